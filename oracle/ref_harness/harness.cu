// harness.cu -- TEST INFRASTRUCTURE ONLY: drives the reference trainer's own
// CUDA functions (visheshnarayan/llm.cu, compiled from its sources where they
// lie; see Makefile) to produce parity fixtures and reference timings.  It is
// never linked into, or called by, libllmcu.so.
//
// The reference trainer (src/train.cu) cannot take injected weights or
// adapters, so this main() replaces only its driver: it allocates the same
// buffers (src/train.cu:112-143), fills MW / LoraWeights from a file, and calls
//   lora_grads_zero -> transformer_forward_lora -> cross_entropy_forward ->
//   transformer_backward_lora -> adamw_step_lora
// exactly as the step loop does (src/train.cu:251-291).  A batch of B
// sequences runs as B forward/backward passes that accumulate into the LoRA
// gradients; each pass normalises by its own (S-1) positions, so the harness
// scales the accumulated gradients by 1/B (with the reference's own
// scale_add_inplace) before AdamW to obtain the batch mean.
//
// The MW / LW structs below restate the layout the reference functions take
// (src/train.cu:10-24); the prototypes restate src/train.cu:27-39.
//
// Modes:
//   harness parity IN OUT     IN: dims, batch, seq, tokens, targets, weights,
//                             adapters, adamw config (see tests/golden/ref_io.py)
//                             OUT: losses[B], grads, post-AdamW adapters
//   harness quantize IN OUT   the reference's quantize_weights on one matrix
//                             (IN: rows, cols, fp32 w; OUT: int8 q, fp32 scales)
//   harness bench B S STEPS WARMUP [TOKENS]
//                             synthetic device-filled weights; B sequences per
//                             step (token windows from the TOKENS file when
//                             given); prints one JSON line with the per-step
//                             time (cudaEvent)
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "config.h"
#include "lora.h"
#include "tensor.h"

typedef struct {
  float* attn_norm;
  float* ffn_norm;
  float* wq; float* wk; float* wv; float* wo;
  float* q_norm; float* k_norm;
  float* w_gate; float* w_up; float* w_down;
  void* _pad[21];
} LW;
typedef struct {
  float* embed_table;
  LW layers[NUM_LAYERS];
  float* final_norm;
  float* lm_head;
  void* _pad[3];
} MW;

void quantize_weights(const float* weight, int8_t* q_weight, float* scales, int rows, int cols);
void transformer_forward_lora(const int*, const MW*, const LoraWeights*, float*, float*, float*, float*, float*,
                              float*, float*, float*, float*, float*, float*, float*, LoraActs*, int);
void transformer_backward_lora(const float*, const MW*, const LoraWeights*, const LoraActs*, LoraGrads*, float*,
                               float*, float*, float*, float*, float*, float*, float*, float*, float*, float*, float*,
                               float*, float*, int);
float cross_entropy_forward(const float* logits, const int* targets, float* dlogits, int seq_len);
void adamw_step_lora(LoraWeights*, const LoraGrads*, float, float, float, float, float, int);
void lora_grads_zero(LoraGrads*);

namespace {

constexpr int Q_DIM = NUM_HEADS * HEAD_DIM;
constexpr int KV_DIM = NUM_KV_HEADS * HEAD_DIM;

struct Ws {
  float *hidden, *residual, *norm_out, *q, *k, *v, *k_exp, *v_exp, *attn_out, *gate_buf, *up_buf, *logits, *dlogits;
  float *d_hidden, *d_hidden2, *d_norm, *d_q, *d_k, *d_v, *d_q_exp, *d_k_exp, *d_v_exp, *d_pre_o, *d_gate, *d_up,
      *dh_tmp, *dx_lora;
};

float* dalloc(size_t n) {
  float* p = nullptr;
  CUDA_CHECK(cudaMalloc(&p, n * sizeof(float)));
  CUDA_CHECK(cudaMemset(p, 0, n * sizeof(float)));
  return p;
}

void alloc_ws(Ws& w, int seq) {
  const size_t S = seq, H = HIDDEN_SIZE, I = INTERMEDIATE_SIZE, V = VOCAB_SIZE;
  w.hidden = dalloc(S * H); w.residual = dalloc(S * H); w.norm_out = dalloc(S * H);
  w.q = dalloc(S * Q_DIM); w.k = dalloc(S * KV_DIM); w.v = dalloc(S * KV_DIM);
  w.k_exp = dalloc(S * Q_DIM); w.v_exp = dalloc(S * Q_DIM); w.attn_out = dalloc(S * Q_DIM);
  w.gate_buf = dalloc(S * I); w.up_buf = dalloc(S * I);
  w.logits = dalloc(S * V); w.dlogits = dalloc(S * V);  // zeroed: the last row is never written (loss.cu:18-21)
  w.d_hidden = dalloc(S * H); w.d_hidden2 = dalloc(S * H); w.d_norm = dalloc(S * H);
  w.d_q = dalloc(S * Q_DIM); w.d_k = dalloc(S * KV_DIM); w.d_v = dalloc(S * KV_DIM);
  w.d_q_exp = dalloc(S * Q_DIM); w.d_k_exp = dalloc(S * Q_DIM); w.d_v_exp = dalloc(S * Q_DIM);
  w.d_pre_o = dalloc(S * Q_DIM); w.d_gate = dalloc(S * I); w.d_up = dalloc(S * I);
  w.dh_tmp = dalloc(S * LORA_RANK); w.dx_lora = dalloc(S * Q_DIM);
}

struct Model {
  MW mw;
  std::vector<float*> bufs;
};

// Weight order in the parity file: embed, final_norm, then per layer
// attn_norm ffn_norm wq wk wv wo q_norm k_norm w_gate w_up w_down.
void alloc_model(MW& m) {
  memset(&m, 0, sizeof(m));
  const size_t H = HIDDEN_SIZE, I = INTERMEDIATE_SIZE, V = VOCAB_SIZE;
  m.embed_table = dalloc(V * H);
  m.final_norm = dalloc(H);
  for (int l = 0; l < NUM_LAYERS; ++l) {
    LW& w = m.layers[l];
    w.attn_norm = dalloc(H); w.ffn_norm = dalloc(H);
    w.wq = dalloc((size_t)Q_DIM * H); w.wk = dalloc((size_t)KV_DIM * H); w.wv = dalloc((size_t)KV_DIM * H);
    w.wo = dalloc(H * Q_DIM); w.q_norm = dalloc(HEAD_DIM); w.k_norm = dalloc(HEAD_DIM);
    w.w_gate = dalloc(I * H); w.w_up = dalloc(I * H); w.w_down = dalloc(H * I);
  }
  m.lm_head = m.embed_table;  // tied (the reference loads a copy of the embedding, scripts/bench_runpod.sh:57)
}

struct Reader {
  FILE* f;
  void read(void* dst, size_t bytes) {
    if (fread(dst, 1, bytes, f) != bytes) { fprintf(stderr, "harness: short read\n"); exit(2); }
  }
  void to_dev(float* d, size_t n) {
    std::vector<float> h(n);
    read(h.data(), n * sizeof(float));
    CUDA_CHECK(cudaMemcpy(d, h.data(), n * sizeof(float), cudaMemcpyHostToDevice));
  }
};

void write_dev(FILE* f, const float* d, size_t n) {
  std::vector<float> h(n);
  CUDA_CHECK(cudaMemcpy(h.data(), d, n * sizeof(float), cudaMemcpyDeviceToHost));
  fwrite(h.data(), sizeof(float), n, f);
}

LoraAdapter* adapter(LoraWeights& lw, int l, int p) {
  return p == 0 ? &lw.wq[l] : p == 1 ? &lw.wk[l] : p == 2 ? &lw.wv[l] : &lw.wo[l];
}
LoraGrad* grad(LoraGrads& g, int l, int p) {
  return p == 0 ? &g.wq[l] : p == 1 ? &g.wk[l] : p == 2 ? &g.wv[l] : &g.wo[l];
}

void step_fwd_bwd(MW& m, LoraWeights& lora, LoraActs& acts, LoraGrads& grads, Ws& w, const int* d_tok,
                  const int* d_tgt, int seq, float* loss) {
  transformer_forward_lora(d_tok, &m, &lora, w.hidden, w.residual, w.norm_out, w.q, w.k, w.v, w.k_exp, w.v_exp,
                           w.attn_out, w.gate_buf, w.up_buf, w.logits, &acts, seq);
  *loss = cross_entropy_forward(w.logits, d_tgt, w.dlogits, seq);
  transformer_backward_lora(w.dlogits, &m, &lora, &acts, &grads, w.d_hidden, w.d_hidden2, w.d_norm, w.d_q, w.d_k,
                            w.d_v, w.d_q_exp, w.d_k_exp, w.d_v_exp, w.d_pre_o, w.d_gate, w.d_up, w.dh_tmp,
                            w.dx_lora, seq);
}

void scale_grads(LoraGrads& g, float s) {
  for (int l = 0; l < NUM_LAYERS; ++l)
    for (int p = 0; p < 4; ++p) {
      LoraGrad* gr = grad(g, l, p);
      const int d_in = p == 3 ? Q_DIM : HIDDEN_SIZE;
      const int d_out = p == 0 ? Q_DIM : (p == 3 ? HIDDEN_SIZE : KV_DIM);
      scale_add_inplace(gr->dA, gr->dA, s - 1.0f, LORA_RANK * d_in);
      scale_add_inplace(gr->dB, gr->dB, s - 1.0f, d_out * LORA_RANK);
    }
}

int parity(const char* in_path, const char* out_path) {
  FILE* f = fopen(in_path, "rb");
  if (!f) { fprintf(stderr, "harness: cannot open %s\n", in_path); return 2; }
  Reader rd{f};
  int32_t hdr[10];
  rd.read(hdr, sizeof(hdr));
  const int32_t want[8] = {HIDDEN_SIZE, NUM_LAYERS, NUM_HEADS, NUM_KV_HEADS, HEAD_DIM, INTERMEDIATE_SIZE, VOCAB_SIZE,
                           LORA_RANK};
  for (int i = 0; i < 8; ++i)
    if (hdr[i] != want[i]) { fprintf(stderr, "harness: dims mismatch at %d (%d vs %d)\n", i, hdr[i], want[i]); return 2; }
  const int B = hdr[8], S = hdr[9];
  std::vector<int32_t> tok(B * S), tgt(B * S);
  rd.read(tok.data(), tok.size() * 4);
  rd.read(tgt.data(), tgt.size() * 4);
  float opt[5];  // lr b1 b2 eps wd
  rd.read(opt, sizeof(opt));

  MW m;
  alloc_model(m);
  const size_t H = HIDDEN_SIZE, I = INTERMEDIATE_SIZE, V = VOCAB_SIZE;
  rd.to_dev(m.embed_table, V * H);
  rd.to_dev(m.final_norm, H);
  for (int l = 0; l < NUM_LAYERS; ++l) {
    LW& w = m.layers[l];
    rd.to_dev(w.attn_norm, H); rd.to_dev(w.ffn_norm, H);
    rd.to_dev(w.wq, (size_t)Q_DIM * H); rd.to_dev(w.wk, (size_t)KV_DIM * H); rd.to_dev(w.wv, (size_t)KV_DIM * H);
    rd.to_dev(w.wo, H * Q_DIM); rd.to_dev(w.q_norm, HEAD_DIM); rd.to_dev(w.k_norm, HEAD_DIM);
    rd.to_dev(w.w_gate, I * H); rd.to_dev(w.w_up, I * H); rd.to_dev(w.w_down, H * I);
  }
  LoraWeights lora;
  lora_weights_init(&lora);
  for (int l = 0; l < NUM_LAYERS; ++l)
    for (int p = 0; p < 4; ++p) {
      LoraAdapter* a = adapter(lora, l, p);
      rd.to_dev(a->A, (size_t)LORA_RANK * a->d_in);
      rd.to_dev(a->B, (size_t)a->d_out * LORA_RANK);
    }
  fclose(f);

  LoraGrads grads;
  lora_grads_alloc(&grads, &lora);
  LoraActs acts;
  lora_acts_alloc(&acts, S);
  Ws w;
  alloc_ws(w, S);
  int *d_tok, *d_tgt;
  CUDA_CHECK(cudaMalloc(&d_tok, S * sizeof(int)));
  CUDA_CHECK(cudaMalloc(&d_tgt, S * sizeof(int)));

  lora_grads_zero(&grads);
  std::vector<float> losses(B);
  for (int b = 0; b < B; ++b) {
    CUDA_CHECK(cudaMemcpy(d_tok, tok.data() + b * S, S * sizeof(int), cudaMemcpyHostToDevice));
    CUDA_CHECK(cudaMemcpy(d_tgt, tgt.data() + b * S, S * sizeof(int), cudaMemcpyHostToDevice));
    step_fwd_bwd(m, lora, acts, grads, w, d_tok, d_tgt, S, &losses[b]);
  }
  if (B > 1) scale_grads(grads, 1.0f / B);
  CUDA_CHECK(cudaDeviceSynchronize());

  FILE* o = fopen(out_path, "wb");
  if (!o) { fprintf(stderr, "harness: cannot write %s\n", out_path); return 2; }
  fwrite(losses.data(), sizeof(float), B, o);
  for (int l = 0; l < NUM_LAYERS; ++l)
    for (int p = 0; p < 4; ++p) {
      LoraAdapter* a = adapter(lora, l, p);
      LoraGrad* g = grad(grads, l, p);
      write_dev(o, g->dA, (size_t)LORA_RANK * a->d_in);
      write_dev(o, g->dB, (size_t)a->d_out * LORA_RANK);
    }
  adamw_step_lora(&lora, &grads, opt[0], opt[1], opt[2], opt[3], opt[4], 1);
  CUDA_CHECK(cudaDeviceSynchronize());
  for (int l = 0; l < NUM_LAYERS; ++l)
    for (int p = 0; p < 4; ++p) {
      LoraAdapter* a = adapter(lora, l, p);
      write_dev(o, a->A, (size_t)LORA_RANK * a->d_in);
      write_dev(o, a->B, (size_t)a->d_out * LORA_RANK);
    }
  fclose(o);
  printf("harness parity: B=%d S=%d loss[0]=%.6f\n", B, S, losses[0]);
  return 0;
}

__global__ void fill_kernel(float* p, size_t n, unsigned seed, float scale) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    unsigned h = (unsigned)i * 2654435761u ^ seed;
    h ^= h >> 15; h *= 2246822519u; h ^= h >> 13; h *= 3266489917u; h ^= h >> 16;
    p[i] = ((h & 0xFFFFFF) / 16777216.0f - 0.5f) * 2.0f * scale;  // uniform, std = scale/sqrt(3)
  }
}

void fill(float* p, size_t n, unsigned seed, float scale) {
  fill_kernel<<<1024, 256>>>(p, n, seed, scale);
  CUDA_CHECK_LAST();
}

int bench(int B, int S, int steps, int warmup, const char* tok_file) {
  MW m;
  alloc_model(m);
  const size_t H = HIDDEN_SIZE, I = INTERMEDIATE_SIZE, V = VOCAB_SIZE;
  const float sc = 0.02f * 1.7320508f;
  unsigned seed = 1;
  fill(m.embed_table, V * H, seed++, sc);
  for (int l = 0; l < NUM_LAYERS; ++l) {
    LW& w = m.layers[l];
    fill(w.wq, (size_t)Q_DIM * H, seed++, sc); fill(w.wk, (size_t)KV_DIM * H, seed++, sc);
    fill(w.wv, (size_t)KV_DIM * H, seed++, sc); fill(w.wo, H * Q_DIM, seed++, sc);
    fill(w.w_gate, I * H, seed++, sc); fill(w.w_up, I * H, seed++, sc); fill(w.w_down, H * I, seed++, sc);
  }
  std::vector<float> ones(H > HEAD_DIM ? H : HEAD_DIM, 1.0f);
  CUDA_CHECK(cudaMemcpy(m.final_norm, ones.data(), H * 4, cudaMemcpyHostToDevice));
  for (int l = 0; l < NUM_LAYERS; ++l) {
    LW& w = m.layers[l];
    CUDA_CHECK(cudaMemcpy(w.attn_norm, ones.data(), H * 4, cudaMemcpyHostToDevice));
    CUDA_CHECK(cudaMemcpy(w.ffn_norm, ones.data(), H * 4, cudaMemcpyHostToDevice));
    CUDA_CHECK(cudaMemcpy(w.q_norm, ones.data(), HEAD_DIM * 4, cudaMemcpyHostToDevice));
    CUDA_CHECK(cudaMemcpy(w.k_norm, ones.data(), HEAD_DIM * 4, cudaMemcpyHostToDevice));
  }
  LoraWeights lora;
  lora_weights_init(&lora);
  LoraGrads grads;
  lora_grads_alloc(&grads, &lora);
  LoraActs acts;
  lora_acts_alloc(&acts, S);
  Ws w;
  alloc_ws(w, S);
  int *d_tok, *d_tgt;
  CUDA_CHECK(cudaMalloc(&d_tok, (size_t)B * S * sizeof(int)));
  CUDA_CHECK(cudaMalloc(&d_tgt, (size_t)B * S * sizeof(int)));
  // B windows of S + 1 ids (inputs = ids[0..S-1], targets = ids[1..S]): from
  // tok_file (int32, written by bench.py with the same draw as its own arm),
  // else an LCG over the vocabulary
  std::vector<int> tok((size_t)B * (S + 1));
  if (tok_file) {
    FILE* f = fopen(tok_file, "rb");
    if (!f || fread(tok.data(), sizeof(int), tok.size(), f) != tok.size()) {
      fprintf(stderr, "cannot read %zu token ids from %s\n", tok.size(), tok_file);
      return 1;
    }
    fclose(f);
    for (int t : tok)
      if (t < 0 || t >= VOCAB_SIZE) {
        fprintf(stderr, "token id %d outside [0, %d)\n", t, VOCAB_SIZE);
        return 1;
      }
  } else {
    unsigned r = 12345;
    for (auto& t : tok) { r = r * 1664525u + 1013904223u; t = (int)(r % VOCAB_SIZE); }
  }
  for (int b = 0; b < B; ++b) {
    CUDA_CHECK(cudaMemcpy(d_tok + b * S, tok.data() + b * (S + 1), S * 4, cudaMemcpyHostToDevice));
    CUDA_CHECK(cudaMemcpy(d_tgt + b * S, tok.data() + b * (S + 1) + 1, S * 4, cudaMemcpyHostToDevice));
  }
  cudaEvent_t e0, e1;
  CUDA_CHECK(cudaEventCreate(&e0));
  CUDA_CHECK(cudaEventCreate(&e1));
  float loss = 0.f, ms_total = 0.f;
  for (int it = 0; it < warmup + steps; ++it) {
    if (it == warmup) CUDA_CHECK(cudaEventRecord(e0));
    lora_grads_zero(&grads);
    for (int b = 0; b < B; ++b) step_fwd_bwd(m, lora, acts, grads, w, d_tok + b * S, d_tgt + b * S, S, &loss);
    if (B > 1) scale_grads(grads, 1.0f / B);
    adamw_step_lora(&lora, &grads, 3e-4f, 0.9f, 0.999f, 1e-8f, 0.01f, it + 1);
  }
  CUDA_CHECK(cudaEventRecord(e1));
  CUDA_CHECK(cudaEventSynchronize(e1));
  CUDA_CHECK(cudaEventElapsedTime(&ms_total, e0, e1));
  const double ms = steps > 0 ? ms_total / steps : 0.0;
  printf("{\"harness\": \"reference\", \"batch\": %d, \"seq\": %d, \"steps\": %d, \"warmup\": %d, "
         "\"ms_per_step\": %.3f, \"tokens_per_s\": %.3f, \"loss\": %.6f}\n",
         B, S, steps, warmup, ms, ms > 0 ? 1000.0 * B * S / ms : 0.0, loss);
  return 0;
}

}  // namespace

// The reference's per-row INT8 quantiser (src/kernels/quantize.cu:8-50, its
// own quantize_weights launch) on one weight matrix.  IN: int32 rows, int32
// cols, float32 w[rows * cols].  OUT: int8 q[rows * cols], float32
// scale[rows].
int quantize(const char* in_path, const char* out_path) {
  FILE* f = fopen(in_path, "rb");
  int dims[2] = {0, 0};
  if (!f || fread(dims, sizeof(int), 2, f) != 2 || dims[0] <= 0 || dims[1] <= 0) {
    fprintf(stderr, "harness: bad quantize input %s\n", in_path);
    return 2;
  }
  const size_t n = static_cast<size_t>(dims[0]) * dims[1];
  std::vector<float> w(n);
  if (fread(w.data(), sizeof(float), n, f) != n) {
    fprintf(stderr, "harness: short read %s\n", in_path);
    return 2;
  }
  fclose(f);
  float *dw, *ds;
  int8_t* dq;
  CUDA_CHECK(cudaMalloc(&dw, n * sizeof(float)));
  CUDA_CHECK(cudaMalloc(&dq, n));
  CUDA_CHECK(cudaMalloc(&ds, dims[0] * sizeof(float)));
  CUDA_CHECK(cudaMemcpy(dw, w.data(), n * sizeof(float), cudaMemcpyHostToDevice));
  quantize_weights(dw, dq, ds, dims[0], dims[1]);
  CUDA_CHECK(cudaDeviceSynchronize());
  std::vector<int8_t> q(n);
  std::vector<float> sc(dims[0]);
  CUDA_CHECK(cudaMemcpy(q.data(), dq, n, cudaMemcpyDeviceToHost));
  CUDA_CHECK(cudaMemcpy(sc.data(), ds, dims[0] * sizeof(float), cudaMemcpyDeviceToHost));
  FILE* o = fopen(out_path, "wb");
  if (!o || fwrite(q.data(), 1, n, o) != n || fwrite(sc.data(), sizeof(float), dims[0], o) != (size_t)dims[0]) {
    fprintf(stderr, "harness: cannot write %s\n", out_path);
    return 2;
  }
  fclose(o);
  return 0;
}

int main(int argc, char** argv) {
  if (argc >= 4 && !strcmp(argv[1], "parity")) return parity(argv[2], argv[3]);
  if (argc >= 4 && !strcmp(argv[1], "quantize")) return quantize(argv[2], argv[3]);
  if (argc >= 6 && !strcmp(argv[1], "bench"))
    return bench(atoi(argv[2]), atoi(argv[3]), atoi(argv[4]), atoi(argv[5]), argc >= 7 ? argv[6] : nullptr);
  fprintf(stderr, "usage: harness parity IN OUT | harness quantize IN OUT | harness bench B S STEPS WARMUP [TOKENS]\n");
  return 2;
}
