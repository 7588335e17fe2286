// llmcu.cu -- the C ABI (include/llmcu.h): context, device arena, weight and
// adapter I/O, the training step schedule and data-parallel plumbing.
//
// Step schedule on the compute stream (reference order, src/train.cu:251-291,
// restated for fused kernels; M = batch * seq rows):
//   lora_merge                         merged q/k/v/o weights W + s B A (+ A, s B pads)
//   embed -> for each layer:
//     rmsnorm(attn) -> h = xn A_cat^T -> qkv = [xn|h][W_qkv|2B]^T
//     -> QK-norm+RoPE -> flash attention -> h_o = o A_o^T
//     -> resid_mid = resid + [o|h_o][W_o|2B_o]^T
//     -> rmsnorm(ffn) -> gate/up GEMM with SwiGLU -> resid_out = resid_mid + act W_d^T
//   final rmsnorm -> lm_head streamed over vocabulary chunks: per chunk the
//   logits GEMM leaves exp(logit - row reference) in an L2-sized chunk buffer,
//   rows that met a new maximum are rescaled, d_xf += chunk values . E_c
//   (split-K) -> LSE, loss, d_xf = exp(ref - lse) d_xf + (p_t - 1) E_t
//   -> final-norm backward -> for each layer, reversed:
//     down dX + SwiGLU bwd -> gate/up dX -> ffn-norm bwd -> dh_o -> o dX (+LoRA)
//     -> LoRA grads (o) -> attention bwd -> RoPE/QK-norm bwd -> dh_qkv
//     -> qkv dX (+LoRA) -> LoRA grads (q,k,v) -> attn-norm bwd
//     [data parallel: allreduce of this layer's adapter gradients on the
//      communication stream, overlapping the layers still to run]
//   AdamW over the flat adapter buffer.
#include <nccl.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

#include "../../include/llmcu.h"
#include "common.cuh"
#include "lora.cuh"

using namespace llmcu;

namespace {

constexpr float kGradScale = 64.0f;   // dlogits are scaled by this power of two (fp16 range)
constexpr int kLmSplitK = 4;          // K (vocabulary) slices of each lm_head dX GEMM
// The lm_head streams over the vocabulary in chunks whose fp16 values
// ([rows, chunk]) fit this many elements (128 MiB: 16384 columns at 4096
// rows; measured on B200 against 8192 / 32768 columns, the shorter chain of
// launches outweighs the part of the chunk that leaves L2)
constexpr size_t kCeChunkElems = static_cast<size_t>(64) << 20;
constexpr int kCeFirstChunk = 2048;  // vocabulary columns of the first chunk
// split-K fix-up workspace of the GEMMs whose tiles fill under half a wave
// (small batches): about one wave of 128 x 256 fp32 partial tiles
constexpr size_t kFxWsFloats = static_cast<size_t>(160) * 128 * 256;
constexpr int kFxCounters = 16384;
// adapter-gradient split partials (lora_grad): enough for the per-layer
// batches at the split counts lora_grad_splits picks (fewer splits otherwise)
constexpr size_t kLgWsFloats = static_cast<size_t>(8) << 20;

struct LayerW {
  __half *wqkv, *wo, *wgu, *wd;  // fp16 base, [out, in] (also read MN-major by the dX GEMMs)
  float *attn_norm, *ffn_norm, *q_norm, *k_norm;
  // INT8 base: q [out, in] per fused weight + per-row scales
  int8_t *q_qkv, *q_o, *q_gu, *q_d;
  float *s_qkv, *s_o, *s_gu, *s_d;
  // merged base + LoRA weights of this step (lora_merge); mgu / md only
  // with MLP targets
  __half *mqkv, *mo, *mgu, *md;
};

struct LayerA {  // forward stash
  float *resid_mid;
  __half *xn, *hq, *qkv, *qkr, *attn, *ho, *xn2, *gu, *act;  // qkr: normed, rotated q | k [M, Q + KV]
  __half *hgu, *hd;  // MLP targets: x A^T of gate | up (segments 0 / 16) and of down, [M, 64]
  float* lse;
};

}  // namespace

struct llmcu_ctx {
  llmcu_model_cfg m;
  llmcu_lora_cfg lc;
  llmcu_run_cfg rc;
  int device = 0;
  int H = 0, Q = 0, KV = 0, QKV = 0, I = 0, V = 0, L = 0, hd = 0, nh = 0, nkv = 0, Mmax = 0;
  LoraDims ld;
  int64_t n_lora = 0;
  std::string err;
  cudaStream_t st = nullptr, comm = nullptr;
  cudaStream_t side = nullptr;  // adapter-gradient launches, overlapped with the backward's main chain
  char* arena = nullptr;
  size_t arena_bytes = 0;

  // base
  __half* E = nullptr;
  float* final_norm = nullptr;
  int8_t *qE = nullptr;
  float* sE = nullptr;
  std::vector<LayerW> lw;
  // int8 dequant scratch (one layer's fp16 weight) and a row-scale temporary
  __half* dq_w = nullptr;
  float* q_scale_tmp = nullptr;
  MergeWeights mw;  // all layers' base weights, for lora_merge

  // lora
  float *lp = nullptr, *lg = nullptr, *lm = nullptr, *lv = nullptr;
  int lpart_amax = 0;

  // activations
  std::vector<float*> resid;  // L + 1 buffers
  std::vector<LayerA> la;
  __half* xf = nullptr;
  // streamed lm_head: per (row, 128-column slot) reference and sum of
  // exp(logit - reference); per-row running reference; one chunk of values
  float *part_ref = nullptr, *part_sum = nullptr, *tgt_logit = nullptr, *lse_ce = nullptr, *row_loss = nullptr;
  float* ce_ref = nullptr;
  uint8_t* valid = nullptr;
  __half* pc = nullptr;  // [rows, chunk] fp16
  size_t pc_elems = 0;
  float* d_xf = nullptr;
  int ce_slots = 0;
  // backward scratch
  float *dres = nullptr, *dq = nullptr, *dk = nullptr, *delta = nullptr;
  float* dq_slabs = nullptr;  // deterministic mode: per-key-tile dQ partials
  __half* dxn = nullptr;  // dX of the normed inputs (fp16, feeds the RMSNorm backward)
  __half *dres16 = nullptr, *dgu = nullptr, *dho = nullptr, *dattn = nullptr, *dqkv = nullptr, *dhq = nullptr;
  __half* dres16m = nullptr;  // fp16 gradient at the attention block's output (the FFN norm backward's)
  __half *dhgu = nullptr, *dhd = nullptr;  // MLP targets: dY s B of gate | up and of down, [M, 64]
  // io
  int *tok = nullptr, *tgt = nullptr, *derr = nullptr;
  float* fx_ws = nullptr;  // split-K fix-up partials (set_gemm_workspace)
  int* fx_cnt = nullptr;
  float* lg_ws = nullptr;  // adapter-gradient split partials
  float* loss_dev = nullptr;   // [0] = mean loss of the last step
  float *rope_cos = nullptr, *rope_sin = nullptr;
  float* stage = nullptr;      // fp32 staging for host uploads
  size_t stage_elems = 0;
  int last_n_valid = 0;
  // decoding (llmcu_generate): K / V cache [L][max_seq][KV] (roped k, v), one
  // position's vectors, split-attention partials, counters and chosen tokens
  __half *kc = nullptr, *vc = nullptr;
  float *dec_x = nullptr, *dec_xmid = nullptr, *dec_logits = nullptr, *dec_part = nullptr, *dec_amax = nullptr;
  __half *dec_qkv = nullptr, *dec_attn = nullptr, *dec_gu = nullptr;
  int *dec_cnt = nullptr, *dec_tok = nullptr, *dec_tickets = nullptr;
  cudaGraphExec_t dec_graph = nullptr;  // one decode step, captured on first use

  // per-kernel-class timing (llmcu_profile_enable)
  bool prof_on = false;
  std::vector<cudaEvent_t> prof_ev;
  std::vector<int> prof_cls;  // class of each recorded (begin, end) event pair
  std::vector<int> prof_k;    // kernels launched between each (begin, end) pair
  int prof_n = 0;             // events used
  double prof_ms[16] = {0};
  int64_t prof_cnt[16] = {0};

  // data parallel
  ncclComm_t nccl = nullptr;
  int rank = 0, world = 1;
  int timeout_ms = 60000;
  std::vector<cudaEvent_t> ev_layer;
  cudaEvent_t ev_comm_done = nullptr, ev_step_done = nullptr;
  cudaEvent_t ev_dq_in = nullptr, ev_dq_done = nullptr;  // dq zeroed on the side stream
  // per layer: main -> side before the MLP and attention adapter gradients,
  // side -> main after each
  std::vector<cudaEvent_t> ev_side;
};

namespace {

llmcu_status fail(llmcu_ctx* c, llmcu_status s, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  if (c) c->err = buf;
  return s;
}

#define CK(expr)                                                                                   \
  do {                                                                                             \
    cudaError_t e_ = (expr);                                                                       \
    if (e_ != cudaSuccess)                                                                         \
      return fail(ctx, LLMCU_ERR_CUDA, "%s failed: %s (%s:%d)", #expr, cudaGetErrorString(e_), __FILE__, \
                  __LINE__);                                                                       \
  } while (0)

enum ProfClass : int {
  P_GEMM = 0, P_ATTN_FWD, P_ATTN_BWD, P_NORM, P_LORA_GRAD, P_LORA_PREP, P_LMHEAD, P_EMBED, P_ADAMW, P_DEQUANT, P_FILL,
  P_DP_WAIT,  // no kernel: the compute stream waiting for the last allreduces after the backward
  P_COUNT
};
const char* kProfNames[P_COUNT] = {"gemm_tc", "attention_fwd", "attention_bwd", "norm_rope", "lora_grad",
                                   "lora_merge", "lm_head", "embed", "adamw", "int8_dequant", "fill_and_loss",
                                   "dp_exposed"};

// Records one event of a (begin, end) pair around `kernels` launches of class `cls`.
void prof_mark(llmcu_ctx* c, int cls, int kernels = 1) {
  if (!c->prof_on || c->prof_n + 1 > static_cast<int>(c->prof_ev.size())) return;
  cudaEventRecord(c->prof_ev[c->prof_n], c->st);
  if ((c->prof_n & 1) == 0) {
    c->prof_cls.push_back(cls);
    c->prof_k.push_back(kernels);
  }
  ++c->prof_n;
}

#define CKS(expr)                                  \
  do {                                             \
    llmcu_status s_ = (expr);                      \
    if (s_ != LLMCU_OK) return s_;                 \
  } while (0)

// `expr` launches `n` kernels of class `cls`
#define TIMEDN(cls, n, expr)    \
  do {                          \
    prof_mark(ctx, cls, n);     \
    CK(expr);                   \
    prof_mark(ctx, cls, n);     \
  } while (0)
#define TIMED(cls, expr) TIMEDN(cls, 1, expr)

Operand op(const __half* p, int rows, int k, int ld) { return Operand{p, rows, k, ld}; }

// ------------------------------------------------------------------ arena
struct Carver {
  size_t off = 0;
  char* base = nullptr;
  template <class T>
  T* take(size_t n) {
    off = (off + 255) / 256 * 256;
    T* p = base ? reinterpret_cast<T*>(base + off) : nullptr;
    off += n * sizeof(T);
    return p;
  }
};

void carve(llmcu_ctx* c, Carver& cv) {
  const size_t H = c->H, Q = c->Q, KV = c->KV, QKV = c->QKV, I = c->I, V = c->V, M = c->Mmax, L = c->L;
  const bool int8 = c->rc.base_dtype == LLMCU_BASE_INT8;
  c->lw.assign(L, LayerW{});
  c->la.assign(L, LayerA{});
  c->resid.assign(L + 1, nullptr);
  // base weights: each kind for all layers in one array (lora_merge indexes layers by stride)
  c->E = cv.take<__half>(V * H);  // INT8: the dequantised table (gather + lm_head)
  if (int8) {
    c->qE = cv.take<int8_t>(V * H);
    c->sE = cv.take<float>(V);
  }
  c->final_norm = cv.take<float>(H);
  c->mw = MergeWeights{};
  if (!int8) {
    __half* wqkv = cv.take<__half>(L * QKV * H);
    __half* wo = cv.take<__half>(L * H * Q);
    __half* wgu = cv.take<__half>(L * 2 * I * H);
    __half* wd = cv.take<__half>(L * H * I);
    for (size_t l = 0; l < L; ++l) {
      LayerW& w = c->lw[l];
      w.wqkv = wqkv ? wqkv + l * QKV * H : nullptr;
      w.wo = wo ? wo + l * H * Q : nullptr;
      w.wgu = wgu ? wgu + l * 2 * I * H : nullptr;
      w.wd = wd ? wd + l * H * I : nullptr;
    }
    c->mw.qkv.w = wqkv;
    c->mw.o.w = wo;
    c->mw.gu.w = wgu;
    c->mw.d.w = wd;
  } else {
    int8_t* q_qkv = cv.take<int8_t>(L * QKV * H);
    int8_t* q_o = cv.take<int8_t>(L * H * Q);
    int8_t* q_gu = cv.take<int8_t>(L * 2 * I * H);
    int8_t* q_d = cv.take<int8_t>(L * H * I);
    float* s_qkv = cv.take<float>(L * QKV);
    float* s_o = cv.take<float>(L * H);
    float* s_gu = cv.take<float>(L * 2 * I);
    float* s_d = cv.take<float>(L * H);
    for (size_t l = 0; l < L; ++l) {
      LayerW& w = c->lw[l];
      w.q_qkv = q_qkv ? q_qkv + l * QKV * H : nullptr;
      w.q_o = q_o ? q_o + l * H * Q : nullptr;
      w.q_gu = q_gu ? q_gu + l * 2 * I * H : nullptr;
      w.q_d = q_d ? q_d + l * H * I : nullptr;
      w.s_qkv = s_qkv ? s_qkv + l * QKV : nullptr;
      w.s_o = s_o ? s_o + l * H : nullptr;
      w.s_gu = s_gu ? s_gu + l * 2 * I : nullptr;
      w.s_d = s_d ? s_d + l * H : nullptr;
    }
    c->mw.qkv.q = q_qkv;
    c->mw.o.q = q_o;
    c->mw.gu.q = q_gu;
    c->mw.d.q = q_d;
    c->mw.qkv.s = s_qkv;
    c->mw.o.s = s_o;
    c->mw.gu.s = s_gu;
    c->mw.d.s = s_d;
    c->mw.qkv.s_layer = static_cast<int64_t>(QKV);
    c->mw.o.s_layer = static_cast<int64_t>(H);
    c->mw.gu.s_layer = static_cast<int64_t>(2 * I);
    c->mw.d.s_layer = static_cast<int64_t>(H);
    const size_t wmax = std::max({QKV * H, H * Q, 2 * I * H, H * I});
    c->dq_w = cv.take<__half>(wmax);
    c->q_scale_tmp = cv.take<float>(std::max({QKV, H, 2 * I}));
  }
  c->mw.qkv.w_layer = static_cast<int64_t>(QKV * H);
  c->mw.o.w_layer = static_cast<int64_t>(H * Q);
  c->mw.gu.w_layer = static_cast<int64_t>(2 * I * H);
  c->mw.d.w_layer = static_cast<int64_t>(H * I);
  const bool mlp = c->ld.has_mlp();
  {
    const int64_t nq = merged_qkv_elems(c->ld), no = merged_o_elems(c->ld);
    const int64_t ng = merged_gu_elems(c->ld), nd = merged_d_elems(c->ld);
    __half* mqkv = cv.take<__half>(L * nq);
    __half* mo = cv.take<__half>(L * no);
    __half* mgu = mlp ? cv.take<__half>(L * ng) : nullptr;
    __half* md = mlp ? cv.take<__half>(L * nd) : nullptr;
    for (size_t l = 0; l < L; ++l) {
      c->lw[l].mqkv = mqkv ? mqkv + l * nq : nullptr;
      c->lw[l].mo = mo ? mo + l * no : nullptr;
      c->lw[l].mgu = mgu ? mgu + l * ng : nullptr;
      c->lw[l].md = md ? md + l * nd : nullptr;
    }
  }
  for (size_t l = 0; l < L; ++l) {
    LayerW& w = c->lw[l];
    w.attn_norm = cv.take<float>(H);
    w.ffn_norm = cv.take<float>(H);
    w.q_norm = cv.take<float>(c->hd);
    w.k_norm = cv.take<float>(c->hd);
  }
  // lora
  const size_t n = static_cast<size_t>(c->n_lora);
  c->lp = cv.take<float>(n);
  c->lg = cv.take<float>(n);
  c->lm = cv.take<float>(n);
  c->lv = cv.take<float>(n);
  c->lpart_amax = static_cast<int>((std::max({H, Q, KV}) + 63) / 64 * 64);

  // activations
  for (size_t l = 0; l <= L; ++l) c->resid[l] = cv.take<float>(M * H);
  const size_t lse_n = static_cast<size_t>(c->rc.max_batch) * c->nh * c->rc.max_seq;
  for (size_t l = 0; l < L; ++l) {
    LayerA& a = c->la[l];
    a.resid_mid = cv.take<float>(M * H);
    a.xn = cv.take<__half>(M * H);
    a.hq = cv.take<__half>(M * 64);
    a.qkv = cv.take<__half>(M * QKV);
    a.qkr = cv.take<__half>(M * (Q + KV));
    a.attn = cv.take<__half>(M * Q);
    a.ho = cv.take<__half>(M * 64);
    a.xn2 = cv.take<__half>(M * H);
    a.gu = cv.take<__half>(M * 2 * I);
    a.act = cv.take<__half>(M * I);
    a.hgu = mlp ? cv.take<__half>(M * 64) : nullptr;
    a.hd = mlp ? cv.take<__half>(M * 64) : nullptr;
    a.lse = cv.take<float>(lse_n);
  }
  c->xf = cv.take<__half>(M * H);
  c->ce_slots = static_cast<int>((V + 127) / 128);
  c->part_ref = cv.take<float>(M * c->ce_slots);
  c->part_sum = cv.take<float>(M * c->ce_slots);
  c->tgt_logit = cv.take<float>(M);
  c->lse_ce = cv.take<float>(M);
  c->row_loss = cv.take<float>(M + 1);
  c->ce_ref = cv.take<float>(M);
  c->valid = cv.take<uint8_t>(M);
  const size_t v_pad = (V + 255) / 256 * 256;
  const size_t chunk = c->rc.lm_head_chunk > 0 ? std::min<size_t>(c->rc.lm_head_chunk, v_pad) : 0;
  c->pc_elems = chunk ? M * chunk : std::min(std::max(kCeChunkElems, M * 256), M * v_pad);
  c->pc = cv.take<__half>(c->pc_elems);  // one vocabulary chunk of the lm_head
  c->d_xf = cv.take<float>(M * H);
  c->dres = cv.take<float>(M * H);
  c->dres16 = cv.take<__half>(M * H);
  c->dres16m = cv.take<__half>(M * H);
  c->dxn = cv.take<__half>(M * H);
  c->dgu = cv.take<__half>(M * 2 * I);
  c->dho = cv.take<__half>(M * 64);
  c->dattn = cv.take<__half>(M * Q);
  c->dq = cv.take<float>(M * Q);
  if (c->rc.deterministic) {
    const size_t nqt = (static_cast<size_t>(c->rc.max_seq) + 127) / 128;
    c->dq_slabs = cv.take<float>(nqt * static_cast<size_t>(c->rc.max_batch) * nqt * 128 * Q);
  }
  c->dk = cv.take<float>(M * KV);
  c->delta = cv.take<float>(lse_n);
  c->dqkv = cv.take<__half>(M * QKV);
  c->dhq = cv.take<__half>(M * 64);
  c->dhgu = mlp ? cv.take<__half>(M * 64) : nullptr;
  c->dhd = mlp ? cv.take<__half>(M * 64) : nullptr;
  c->fx_ws = cv.take<float>(kFxWsFloats);
  c->fx_cnt = cv.take<int>(kFxCounters);
  c->lg_ws = cv.take<float>(kLgWsFloats);
  c->tok = cv.take<int>(M);
  c->tgt = cv.take<int>(M);
  c->derr = cv.take<int>(4);
  c->loss_dev = cv.take<float>(4);
  c->rope_cos = cv.take<float>(static_cast<size_t>(c->rc.max_seq) * (c->hd / 2));
  c->rope_sin = cv.take<float>(static_cast<size_t>(c->rc.max_seq) * (c->hd / 2));
  c->stage_elems = std::max({V * H, 2 * I * H, QKV * H});
  c->stage = cv.take<float>(c->stage_elems);
  const size_t ctxlen = static_cast<size_t>(c->rc.max_seq);
  c->kc = cv.take<__half>(L * ctxlen * KV);
  c->vc = cv.take<__half>(L * ctxlen * KV);
  c->dec_x = cv.take<float>(H);
  c->dec_xmid = cv.take<float>(H);
  c->dec_logits = cv.take<float>(V);
  c->dec_part = cv.take<float>(static_cast<size_t>(c->nh) * decode_attn_splits(c->rc.max_seq) * (c->hd + 2));
  c->dec_qkv = cv.take<__half>(QKV);
  c->dec_attn = cv.take<__half>(Q);
  c->dec_gu = cv.take<__half>(2 * I);
  c->dec_cnt = cv.take<int>(4);
  c->dec_tickets = cv.take<int>(c->nh);
  c->dec_amax = cv.take<float>(decode_argmax_scratch());
  c->dec_tok = cv.take<int>(ctxlen);
}

llmcu_status check_dev_err(llmcu_ctx* ctx) {
  int e = 0;
  CK(cudaMemcpyAsync(&e, ctx->derr, sizeof(int), cudaMemcpyDeviceToHost, ctx->st));
  CK(cudaStreamSynchronize(ctx->st));
  if (e) {
    CK(cudaMemsetAsync(ctx->derr, 0, sizeof(int), ctx->st));
    if (e & kErrTokenRange) return fail(ctx, LLMCU_ERR_INVALID_ARG, "token or target id outside [0, vocab)");
    return fail(ctx, LLMCU_ERR_DEVICE_CHECK, "device-side check failed (error bits 0x%x)", e);
  }
  return LLMCU_OK;
}

// ---------------------------------------------------------- nccl helpers
llmcu_status nccl_wait(llmcu_ctx* ctx, ncclResult_t r, const char* what) {
  const auto t0 = std::chrono::steady_clock::now();
  while (true) {
    if (r == ncclSuccess) return LLMCU_OK;
    if (r != ncclInProgress) {
      return fail(ctx, LLMCU_ERR_NCCL, "%s: %s", what, ncclGetErrorString(r));
    }
    ncclResult_t ar = ncclSuccess;
    ncclCommGetAsyncError(ctx->nccl, &ar);
    r = ar;
    if (r == ncclInProgress) {
      const auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0).count();
      if (ms > ctx->timeout_ms) {
        ncclCommAbort(ctx->nccl);
        ctx->nccl = nullptr;
        ctx->world = 1;
        return fail(ctx, LLMCU_ERR_TIMEOUT, "%s: NCCL did not complete within %d ms; communicator aborted", what,
                    ctx->timeout_ms);
      }
      std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
  }
}

// Wait on the host for `ev` with the context deadline; on expiry abort NCCL.
llmcu_status wait_event(llmcu_ctx* ctx, cudaEvent_t ev) {
  const auto t0 = std::chrono::steady_clock::now();
  while (true) {
    cudaError_t q = cudaEventQuery(ev);
    if (q == cudaSuccess) return LLMCU_OK;
    if (q != cudaErrorNotReady) return fail(ctx, LLMCU_ERR_CUDA, "step failed: %s", cudaGetErrorString(q));
    if (ctx->nccl) {
      ncclResult_t ar = ncclSuccess;
      ncclCommGetAsyncError(ctx->nccl, &ar);
      if (ar != ncclSuccess && ar != ncclInProgress) {
        ncclCommAbort(ctx->nccl);
        ctx->nccl = nullptr;
        ctx->world = 1;
        return fail(ctx, LLMCU_ERR_NCCL, "NCCL error during step: %s", ncclGetErrorString(ar));
      }
    }
    const auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0).count();
    if (ms > ctx->timeout_ms) {
      if (ctx->nccl) {
        ncclCommAbort(ctx->nccl);
        ctx->nccl = nullptr;
        ctx->world = 1;
      }
      return fail(ctx, LLMCU_ERR_TIMEOUT, "step did not complete within %d ms", ctx->timeout_ms);
    }
    std::this_thread::sleep_for(std::chrono::microseconds(100));
  }
}

// ------------------------------------------------------------- INT8 base
__global__ void scale_loss_kernel(const float* total, float inv_n, float* out) { pdl_trigger(); pdl_wait(); out[0] = total[0] * inv_n; }


Operand op_mn(const __half* p, int k_rows, int n_cols, int ld) { return Operand{p, n_cols, k_rows, ld, true}; }

// B operand of one base weight W [rows, cols] ([out, in]): the fp16 copy, or
// the INT8 rows, staged as exact fp16 by the GEMM, with the per-row scales of
// src/kernels/quantize.cu:55-78 applied to the forward's output columns by its
// epilogue (the reference's INT8 GEMM multiplies the sum by scale[n]); for the
// input gradient (MN-major) the caller folds the scales into A.
Operand base_b(const llmcu_ctx* c, const __half* w16, const int8_t* q, const float* s, int rows, int cols, bool mn) {
  Operand o = mn ? op_mn(w16, rows, cols, cols) : op(w16, rows, cols, cols);
  if (c->rc.base_dtype == LLMCU_BASE_INT8) {
    o.ptr = nullptr;
    o.q8 = q;
    o.q8_scale = s;
  }
  return o;
}

// fp16 [rows, cols] copy of one base weight for the GEMM: the fp16 base
// itself, or the INT8 rows dequantised into scratch by one vectorised pass
// (fp16(code * scale), src/kernels/quantize.cu:55-78's per-row scale).
Operand base_dq(llmcu_ctx* c, const __half* w16, const int8_t* q, const float* s, int rows, int cols, bool mn,
                cudaError_t* e) {
  const __half* w = w16;
  if (c->rc.base_dtype == LLMCU_BASE_INT8) {
    prof_mark(c, P_DEQUANT);
    *e = dequant_rows_f16(q, s, rows, cols, c->dq_w, c->st);
    prof_mark(c, P_DEQUANT);
    w = c->dq_w;
  }
  return mn ? op_mn(w, rows, cols, cols) : op(w, rows, cols, cols);
}

// B operand of an MLP base weight under the context's INT8 mode.
Operand mlp_b(llmcu_ctx* c, const __half* w16, const int8_t* q, const float* s, int rows, int cols, bool mn,
              cudaError_t* e) {
  if (c->rc.base_dtype == LLMCU_BASE_INT8 && c->rc.int8_in_gemm) return base_b(c, w16, q, s, rows, cols, mn);
  return base_dq(c, w16, q, s, rows, cols, mn, e);
}

// The context's split-K fix-up workspace for the gemm() calls of one step
// (or prefill) on this thread; counters re-zeroed first, in case an aborted
// launch left some behind.
struct GemmWorkspaceScope {
  explicit GemmWorkspaceScope(llmcu_ctx* c) { set_gemm_workspace(c->fx_ws, kFxWsFloats, c->fx_cnt, kFxCounters); }
  ~GemmWorkspaceScope() { set_gemm_workspace(nullptr, 0, nullptr, 0); }
};

// Merged weights of the current adapters, every layer (lora_merge).
cudaError_t merge_adapters(llmcu_ctx* ctx) {
  MergedOut mo;
  mo.qkv = ctx->lw[0].mqkv;
  mo.o = ctx->lw[0].mo;
  mo.gu = ctx->lw[0].mgu;
  mo.d = ctx->lw[0].md;
  return lora_merge(ctx->lp, ctx->ld, ctx->L, ctx->mw, mo, ctx->st);
}

// ----------------------------------------------------------------- step
// Embedding and every layer's forward over ctx->tok ([B, S] ids on the device),
// leaving each layer's stash and ctx->resid[L] (the pre-final-norm hidden).
// Expects the merged weights of the current adapters (merge_adapters).
llmcu_status forward_layers(llmcu_ctx* ctx, int B, int S) {
  const int M = B * S;
  const int H = ctx->H, Q = ctx->Q, KV = ctx->KV, QKV = ctx->QKV, I = ctx->I, V = ctx->V;
  const float eps = ctx->m.rms_eps;
  cudaStream_t st = ctx->st;
  int* err = ctx->derr;
  const __half* E = ctx->E;
  TIMED(P_EMBED, embed_forward(ctx->tok, E, ctx->resid[0], M, H, V, err, st));

  // ------------------------------------------------------------ forward
  for (int l = 0; l < ctx->L; ++l) {
    LayerW& w = ctx->lw[l];
    LayerA& a = ctx->la[l];
    const float* x = ctx->resid[l];
    TIMED(P_NORM, rmsnorm_forward(x, w.attn_norm, a.xn, M, H, eps, st));
    {  // [q | k | v | h] = xn . mqkv^T; q, k normed and rotated into qkr
      EpiArgs ea;
      ea.out = a.qkv;
      ea.ld_out = QKV;
      ea.n_main = QKV;
      ea.side = a.hq;
      ea.ld_side = 64;
      if (ctx->hd == 128) {  // QK-norm + RoPE in the GEMM epilogue
        ea.rope_out = a.qkr;
        ea.ld_rope = Q + KV;
        ea.q_norm_w = w.q_norm;
        ea.k_norm_w = w.k_norm;
        ea.rope_cos = ctx->rope_cos;
        ea.rope_sin = ctx->rope_sin;
        ea.seq = S;
        ea.n_q_cols = Q;
        ea.n_qk_cols = Q + KV;
        ea.eps = eps;
        TIMED(P_GEMM, gemm(op(a.xn, M, H, H), op(w.mqkv, QKV + 64, H, H + 64), M, QKV + 64, Epi::kQKNormRope, ea, err,
                           st));
      } else {
        TIMED(P_GEMM, gemm(op(a.xn, M, H, H), op(w.mqkv, QKV + 64, H, H + 64), M, QKV + 64, Epi::kStoreF16, ea, err,
                           st));
        TIMED(P_NORM, qknorm_rope_forward(a.qkv, QKV, w.q_norm, w.k_norm, Q + KV, ctx->rope_cos, ctx->rope_sin, a.qkr,
                                          a.qkr + Q, B, S, ctx->nh, ctx->nkv, ctx->hd, eps, st));
      }
    }
    TIMED(P_ATTN_FWD, attention_forward(a.qkr, a.qkr + Q, a.qkv + Q + KV, a.attn, a.lse, B, S, ctx->nh, ctx->nkv, ctx->hd,
                                        Q + KV, Q + KV, QKV, Q, err, st));
    {  // [resid_mid | h_o] = [resid + attn . mo^T | attn . Ao^T]
      EpiArgs ea;
      ea.out = a.resid_mid;
      ea.ld_out = H;
      ea.resid = x;
      ea.n_main = H;
      ea.side = a.ho;
      ea.ld_side = 64;
      TIMED(P_GEMM, gemm(op(a.attn, M, Q, Q), op(w.mo, H + 64, Q, Q + 64), M, H + 64, Epi::kResidF32, ea, err, st));
    }
    TIMED(P_NORM, rmsnorm_forward(a.resid_mid, w.ffn_norm, a.xn2, M, H, eps, st));
    if (ctx->ld.has_mlp()) {
      {  // [gu | act | h_gu] = xn2 . mgu^T: SwiGLU over the merged rows, h of gate / up in the side tile
        EpiArgs ea;
        ea.gu = a.gu;
        ea.ld_gu = 2 * I;
        ea.act = a.act;
        ea.ld_act = I;
        ea.n_main = 2 * I;
        ea.side = a.hgu;
        ea.ld_side = 64;
        TIMED(P_GEMM, gemm(op(a.xn2, M, H, H), op(w.mgu, 2 * I + 64, H, H + 64), M, 2 * I + 64, Epi::kSwiGLU, ea, err,
                           st, 256));
      }
      {  // [resid' | h_d] = [resid_mid + act . md^T | act . Ad^T]
        EpiArgs ea;
        ea.out = ctx->resid[l + 1];
        ea.ld_out = H;
        ea.resid = a.resid_mid;
        ea.n_main = H;
        ea.side = a.hd;
        ea.ld_side = 64;
        TIMED(P_GEMM, gemm(op(a.act, M, I, I), op(w.md, H + 64, I, I + 64), M, H + 64, Epi::kResidF32, ea, err, st));
      }
      continue;
    }
    cudaError_t e = cudaSuccess;
    {
      EpiArgs ea;
      ea.gu = a.gu;
      ea.ld_gu = 2 * I;
      ea.act = a.act;
      ea.ld_act = I;
      const Operand bgu = mlp_b(ctx, w.wgu, w.q_gu, w.s_gu, 2 * I, H, false, &e);
      CK(e);
      TIMED(P_GEMM, gemm(op(a.xn2, M, H, H), bgu, M, 2 * I, Epi::kSwiGLU, ea, err, st, 256));
    }
    {
      EpiArgs ea;
      ea.out = ctx->resid[l + 1];
      ea.ld_out = H;
      ea.resid = a.resid_mid;
      const Operand bd = mlp_b(ctx, w.wd, w.q_d, w.s_d, H, I, false, &e);
      CK(e);
      TIMED(P_GEMM, gemm(op(a.act, M, I, I), bd, M, H, Epi::kResidF32, ea, err, st));
    }
  }

  return LLMCU_OK;
}

llmcu_status run_forward_backward(llmcu_ctx* ctx, int B, int S) {
  const int M = B * S;
  const int H = ctx->H, Q = ctx->Q, KV = ctx->KV, QKV = ctx->QKV, I = ctx->I, V = ctx->V;
  const float eps = ctx->m.rms_eps;
  cudaStream_t st = ctx->st;
  int* err = ctx->derr;
  const LoraDims& d = ctx->ld;
  const int r = ctx->lc.rank;
  const int n_valid_local = ctx->rc.loss_all_positions ? M : B * (S - 1);
  const double n_valid_total = static_cast<double>(n_valid_local) * ctx->world;
  ctx->last_n_valid = n_valid_local;
  const float unscale = static_cast<float>(1.0 / (kGradScale * n_valid_total));

  // the gradients start at zero (lora_grad stores every adapter it trains);
  // this first kernel follows the host's token upload, so it is launched
  // normally and the rest of the step's kernels chain by programmatic
  // dependent launch
  struct PdlScope {
    ~PdlScope() { set_pdl(false); }
  } pdl_scope;
  set_pdl(false);
  GemmWorkspaceScope gws(ctx);
  CK(cudaMemsetAsync(ctx->fx_cnt, 0, sizeof(int) * kFxCounters, st));
  TIMED(P_FILL, fill_f32(ctx->lg, ctx->n_lora, 0.f, st));
  set_pdl(true);
  // merged q/k/v/o weights of this step's adapters, every layer
  TIMEDN(P_LORA_PREP, d.has_mlp() ? 6 : 3, merge_adapters(ctx));
  TIMED(P_FILL, ce_valid_rows(ctx->valid, ctx->tgt, B, S, ctx->rc.loss_all_positions, V, err, st));
  CKS(forward_layers(ctx, B, S));
  const __half* E = ctx->E;

  // ------------------------------------------------------- lm_head + CE
  // Streamed over the vocabulary (no [M, V] tensor): per chunk of columns,
  // logits = xf E_c^T leave as fp16 exp(logit - ref) into the chunk buffer
  // (with per-slot partials), rows that met a new maximum move to a new
  // reference, and d_xf += values . E_c; the last step forms the loss and
  // dX = exp(ref - lse) d_xf + (p_t - 1) E_t (src/kernels/loss.cu:13-91,
  // src/kernels/lora_forward.cu:304, src/kernels/lora_backward.cu:243).
  float* xfinal = ctx->resid[ctx->L];
  TIMED(P_NORM, rmsnorm_forward(xfinal, ctx->final_norm, ctx->xf, M, H, eps, st));
  {
    // chunk width: the configured one, else as wide as the buffer holds at
    // this step's rows; the first chunk is narrower (every row of the first
    // chunk is rescaled once its maximum is known, so it is kept small)
    const int v_pad = (V + 255) / 256 * 256;
    const int vc = ctx->rc.lm_head_chunk > 0
                       ? std::min(v_pad, ctx->rc.lm_head_chunk)
                       : static_cast<int>(std::min<size_t>(v_pad, ctx->pc_elems / static_cast<size_t>(M) / 256 * 256));
    const int vc0 = std::min(vc, kCeFirstChunk);
    // K (vocabulary) slices of each chunk's dX GEMM: kLmSplitK, more when the
    // row tiles are few (small batches), up to about one wave of CTAs; they
    // reduce-add in no fixed order, so the deterministic mode takes none (the
    // GEMM's own ordered split fix-up then fills small batches)
    const int ksplit =
        ctx->rc.deterministic
            ? 1
            : std::max(kLmSplitK, std::min(16, gemm_num_sms() / std::max(1, (M + 127) / 128 * ((H + 255) / 256))));
    int launches = 2;  // + ce_stream_finish's two
    for (int v0 = 0; v0 < V; v0 += (v0 == 0 ? vc0 : vc)) launches += 3;
    // one event pair around the whole section (per-kernel events would break
    // the programmatic-launch overlap of its short kernels)
    prof_mark(ctx, P_LMHEAD, launches);
    for (int v0 = 0; v0 < V;) {
      const int n = std::min(v0 == 0 ? vc0 : vc, V - v0);
      const __half* Ec = E + static_cast<size_t>(v0) * H;
      EpiArgs ea;
      ea.targets = ctx->tgt;
      ea.ce_ref = ctx->ce_ref;
      ea.part_max = ctx->part_ref;
      ea.part_sum = ctx->part_sum;
      ea.tgt_logit = ctx->tgt_logit;
      ea.ce_slots = ctx->ce_slots;
      ea.vocab_off = v0;
      ea.out = ctx->pc;
      ea.ld_out = vc;
      CK(gemm(op(ctx->xf, M, H, H), op(Ec, n, H, H), M, n, Epi::kCEStream, ea, err, st, 256));
      CK(ce_stream_rescale(ctx->pc, vc, ctx->part_ref, ctx->ce_slots, ctx->ce_ref, ctx->d_xf, M, H, v0, n,
                           v0 == 0 ? 1 : 0, st));
      EpiArgs eb;
      eb.out = ctx->d_xf;
      eb.ld_out = H;
      eb.accumulate = 1;
      eb.ksplit = ksplit;
      // d_xf += values . E_c  (E_c [n, H] read MN-major)
      CK(gemm(op(ctx->pc, M, n, vc), op_mn(Ec, n, H, H), M, H, Epi::kStoreF32, eb, err, st));
      v0 += n;
    }
    CK(ce_stream_finish(ctx->part_ref, ctx->part_sum, ctx->tgt_logit, ctx->ce_ref, ctx->valid, ctx->tgt, E, M, H, V,
                        ctx->ce_slots, kGradScale, ctx->lse_ce, ctx->row_loss, ctx->d_xf, st));
    prof_mark(ctx, P_LMHEAD, launches);
  }
  // an INT8 base's down-projection row scales ride in the fp16 gradient that
  // is the next input-gradient GEMM's A operand (the GEMM stages the codes)
  const bool q8_mlp = ctx->rc.base_dtype == LLMCU_BASE_INT8 && ctx->rc.int8_in_gemm && !d.has_mlp();
  TIMED(P_NORM, rmsnorm_backward(ctx->d_xf, xfinal, ctx->final_norm, ctx->dres, ctx->dres16, M, H, eps, 0, st,
                                 q8_mlp ? ctx->lw[ctx->L - 1].s_d : nullptr));

  // ----------------------------------------------------------- backward
  // The adapter gradients of a layer run on ctx->side, beside the main chain:
  // the main stream hands its inputs over with an event, and waits for the
  // side's event only before it overwrites what they read (the MLP batch reads
  // dres16, rewritten by the layer's attention-norm backward; the attention
  // batch reads dres16m, dho, dqkv and dhq, rewritten from the next layer's
  // FFN-norm backward on).  A kernel that follows an event wait is launched
  // without programmatic dependence.  With profiling on, everything stays on
  // the main stream so that the per-class times stay separable.
  cudaStream_t gs = ctx->prof_on ? st : ctx->side;
  const bool split = gs != st;
  auto ev_side = [&](int l, int k) { return ctx->ev_side[4 * l + k]; };  // 0/1 MLP in/out, 2/3 attention in/out
  auto side_grad = [&](int l, int k, LoraGradBatch gb) -> llmcu_status {
    if (split) {
      CK(cudaEventRecord(ev_side(l, k), st));
      CK(cudaStreamWaitEvent(gs, ev_side(l, k), 0));
    }
    gb.ws = ctx->lg_ws;
    gb.ws_floats = kLgWsFloats;
    gb.err = err;
    set_pdl(!split);
    TIMEDN(P_LORA_GRAD, lora_grad_splits(M, gb) > 1 ? 2 : 1, lora_grad(gb, M, gs));
    set_pdl(true);
    if (split) CK(cudaEventRecord(ev_side(l, k + 1), gs));
    return LLMCU_OK;
  };
  // true when the next main-stream kernel follows an event wait
  auto wait_side = [&](int l, int k) -> llmcu_status {
    if (split) {
      CK(cudaStreamWaitEvent(st, ev_side(l, k), 0));
      set_pdl(false);
    }
    return LLMCU_OK;
  };
  // dq (the attention backward's fp32 reduce-add target) is zeroed on the
  // side stream: for the top layer while the lm_head backward runs, for each
  // lower layer once the layer above has read it
  auto zero_dq_side = [&]() -> llmcu_status {
    CK(cudaEventRecord(ctx->ev_dq_in, st));
    CK(cudaStreamWaitEvent(gs, ctx->ev_dq_in, 0));
    set_pdl(false);
    CK(fill_f32_2d(ctx->dq, Q, M, Q, 0.f, gs));
    set_pdl(true);
    CK(cudaEventRecord(ctx->ev_dq_done, gs));
    return LLMCU_OK;
  };
  const bool slabs = ctx->dq_slabs != nullptr;  // deterministic dQ: no zeroing, no reduce-add
  if (split && !slabs) CKS(zero_dq_side());
  for (int l = ctx->L - 1; l >= 0; --l) {
    LayerW& w = ctx->lw[l];
    LayerA& a = ctx->la[l];
    float* G = ctx->lg + d.per_layer * l;
    auto gp = [&](int p, bool b_side) { return d.has(p) ? G + (b_side ? d.offB(p) : d.offA(p)) : nullptr; };
    const float sb = d.scale * unscale;
    if (d.has_mlp()) {
      {  // [d_act | dh_d] = dres . md (MN-major), SwiGLU backward fused into dgu
        EpiArgs ea;
        ea.gu_in = a.gu;
        ea.gu = ctx->dgu;
        ea.ld_gu = 2 * I;
        ea.n_main = I;
        ea.side = ctx->dhd;
        ea.ld_side = 64;
        TIMED(P_GEMM, gemm(op(ctx->dres16, M, H, H), op_mn(w.md, H, I + 64, I + 64), M, I + 64, Epi::kSwiGLUBwd, ea,
                           err, st, 256));
      }
      {  // [dxn2 | dh_gu] = dgu . mgu (MN-major)
        EpiArgs ea;
        ea.out = ctx->dxn;
        ea.ld_out = H;
        ea.n_main = H;
        ea.side = ctx->dhgu;
        ea.ld_side = 64;
        TIMED(P_GEMM, gemm(op(ctx->dgu, M, 2 * I, 2 * I), op_mn(w.mgu, 2 * I, H + 64, H + 64), M, H + 64,
                           Epi::kStoreF16, ea, err, st));
      }
      // the MLP adapters' gradients; dres16 holds the layer-output gradient
      LoraGradBatch gb{};
      // dB_d[h, j] = s sum_m dres[m, h] h_d[m, j];  dA_d[j, i] = sum_m dh_d[m, j] act[m, i]
      if (d.has(kPDown)) {
        gb.p[gb.n++] = LoraGradProb{ctx->dres16, H, a.hd, 64, {gp(kPDown, true)}, 1, r, 1, H, r, sb, 0};
        gb.p[gb.n++] = LoraGradProb{a.act, I, ctx->dhd, 64, {gp(kPDown, false)}, 1, 1, I, I, r, unscale, 0};
      }
      if (d.has(kPGate) || d.has(kPUp)) {
        // dB_gate / dB_up from the interleaved dgu columns against h_gu's segments 0 / 16
        gb.p[gb.n++] = LoraGradProb{ctx->dgu, 2 * I, a.hgu, 64, {gp(kPGate, true), gp(kPUp, true)}, 2, r, 1, 2 * I,
                                    r, sb, 1};
        // dA_gate, dA_up in one pass over the normed input
        gb.p[gb.n++] = LoraGradProb{a.xn2, H, ctx->dhgu, 64, {gp(kPGate, false), gp(kPUp, false)}, 2, 1, H, H, r,
                                    unscale, 0};
      }
      gb.a_max = 0;
      for (int i = 0; i < gb.n; ++i) gb.a_max = std::max(gb.a_max, gb.p[i].A);
      CKS(side_grad(l, 0, gb));
    } else {
      // MLP: d_act = dres . W_down (MN-major), SwiGLU backward fused
      {
        EpiArgs ea;
        ea.gu_in = a.gu;
        ea.gu = ctx->dgu;
        ea.ld_gu = 2 * I;
        ea.gu_out_scale = q8_mlp ? w.s_gu : nullptr;  // the gate/up row scales, for the next GEMM
        cudaError_t e = cudaSuccess;
        const Operand bd = mlp_b(ctx, w.wd, w.q_d, w.s_d, H, I, true, &e);
        CK(e);
        TIMED(P_GEMM, gemm(op(ctx->dres16, M, H, H), bd, M, I, Epi::kSwiGLUBwd, ea, err, st, 256));
      }
      // dxn2 = dgu . W_gate/up (MN-major)
      cudaError_t e = cudaSuccess;
      const Operand bgu = mlp_b(ctx, w.wgu, w.q_gu, w.s_gu, 2 * I, H, true, &e);
      CK(e);
      TIMED(P_GEMM, gemm(op(ctx->dgu, M, 2 * I, 2 * I), bgu, M, H, Epi::kStoreF16, EpiArgs{ctx->dxn, H}, err, st));
    }
    // the layer above's attention-adapter gradients read dres16m, dho, dqkv, dhq
    if (l + 1 < ctx->L) CKS(wait_side(l + 1, 3));
    TIMED(P_NORM, rmsnorm_backward(ctx->dxn, a.resid_mid, w.ffn_norm, ctx->dres, ctx->dres16m, M, H, eps, 1, st));
    set_pdl(true);
    // O projection
    {  // [dattn | dh_o] = dres . mo (MN-major): dres W'_o and dres s B_o, plus delta = rowsum(dO * O) per head
      EpiArgs ea;
      ea.out = ctx->dattn;
      ea.ld_out = Q;
      ea.n_main = Q;
      ea.side = ctx->dho;
      ea.ld_side = 64;
      ea.attn_o = a.attn;
      ea.ld_o = Q;
      ea.delta = ctx->delta;
      ea.seq = S;
      ea.n_heads = ctx->nh;
      ea.head_dim = ctx->hd;
      TIMED(P_GEMM, gemm(op(ctx->dres16m, M, H, H), op_mn(w.mo, H, Q + 64, Q + 64), M, Q + 64, Epi::kStoreF16Delta,
                         ea, err, st));
    }
    // attention
    // (delta came with the O-projection dX GEMM)
    if (split && !slabs) {  // dq was zeroed on the side stream
      CK(cudaStreamWaitEvent(st, ctx->ev_dq_done, 0));
      set_pdl(false);
    }
    TIMEDN(P_ATTN_BWD, split || slabs ? 1 : 2,
           attention_backward_tc(a.qkr, a.qkr + Q, a.qkv + Q + KV, ctx->dattn, a.lse, ctx->delta, ctx->dq, ctx->dk,
                                 ctx->dqkv + Q + KV, B, S, ctx->nh, ctx->nkv, ctx->hd, Q + KV, Q + KV, QKV, Q, Q, KV,
                                 QKV, err, st, split, ctx->dq_slabs));
    set_pdl(true);
    TIMED(P_NORM, qknorm_rope_backward(ctx->dq, ctx->dk, a.qkv, QKV, w.q_norm, w.k_norm, ctx->rope_cos, ctx->rope_sin, ctx->dqkv,
                            B, S, ctx->nh, ctx->nkv, ctx->hd, eps, st, ctx->dq_slabs));
    if (split && !slabs && l > 0) CKS(zero_dq_side());  // for the next layer, once read
    // QKV projection
    {  // [dxn | dh_qkv] = dqkv . mqkv (MN-major)
      EpiArgs ea;
      ea.out = ctx->dxn;
      ea.ld_out = H;
      ea.n_main = H;
      ea.side = ctx->dhq;
      ea.ld_side = 64;
      TIMED(P_GEMM, gemm(op(ctx->dqkv, M, QKV, QKV), op_mn(w.mqkv, QKV, H + 64, H + 64), M, H + 64, Epi::kStoreF16, ea,
                         err, st));
    }
    {
      // the attention adapters' gradients of the layer in one launch
      LoraGradBatch gb{};
      gb.a_max = ctx->lpart_amax;
      if (d.has(kPQ)) gb.p[gb.n++] = LoraGradProb{ctx->dqkv, QKV, a.hq, 64, {gp(kPQ, true)}, 1, r, 1, Q, r, sb, 0};
      if (d.has(kPK))
        gb.p[gb.n++] = LoraGradProb{ctx->dqkv + Q, QKV, a.hq + kSegK, 64, {gp(kPK, true)}, 1, r, 1, KV, r, sb, 0};
      if (d.has(kPV))
        gb.p[gb.n++] = LoraGradProb{ctx->dqkv + Q + KV, QKV, a.hq + kSegV, 64, {gp(kPV, true)}, 1, r, 1, KV, r, sb, 0};
      // dA_q, dA_k, dA_v in one pass over the normed input (column groups 0 / 16 / 32 of dh)
      if (d.has(kPQ) || d.has(kPK) || d.has(kPV))
        gb.p[gb.n++] = LoraGradProb{a.xn, H, ctx->dhq, 64, {gp(kPQ, false), gp(kPK, false), gp(kPV, false)}, 3, 1, H,
                                    H, r, unscale, 0};
      if (d.has(kPO)) {
        // dBo[h, j] = s * sum_m dres[m, h] ho[m, j] (dres at the attention block's output)
        gb.p[gb.n++] = LoraGradProb{ctx->dres16m, H, a.ho, 64, {gp(kPO, true)}, 1, r, 1, H, r, sb, 0};
        // dAo[j, q] = sum_m dho[m, j] attn[m, q]
        gb.p[gb.n++] = LoraGradProb{a.attn, Q, ctx->dho, 64, {gp(kPO, false)}, 1, 1, Q, Q, r, unscale, 0};
      }
      if (gb.n) {
        CKS(side_grad(l, 2, gb));
      } else if (split) {  // keep the layer's "done" event meaningful
        CK(cudaEventRecord(ev_side(l, 2), st));
        CK(cudaStreamWaitEvent(gs, ev_side(l, 2), 0));
        CK(cudaEventRecord(ev_side(l, 3), gs));
      }
    }
    // the MLP batch reads dres16, which the attention-norm backward rewrites
    if (d.has_mlp()) CKS(wait_side(l, 1));
    TIMED(P_NORM, rmsnorm_backward(ctx->dxn, ctx->resid[l], w.attn_norm, ctx->dres, ctx->dres16, M, H, eps, 1, st,
                                   q8_mlp && l > 0 ? ctx->lw[l - 1].s_d : nullptr));
    set_pdl(true);
    if (ctx->nccl) {
      // the layer's gradients are complete once its last side launch is
      cudaEvent_t done = ctx->ev_layer[l];
      if (split) {
        done = ev_side(l, 3);
      } else {
        CK(cudaEventRecord(done, st));
      }
      CK(cudaStreamWaitEvent(ctx->comm, done, 0));
      CKS(nccl_wait(ctx, ncclAllReduce(G, G, static_cast<size_t>(d.per_layer), ncclFloat, ncclSum, ctx->nccl,
                                       ctx->comm),
                    "allreduce of layer gradients"));
    }
  }
  // dp_exposed: compute-stream time from the end of the backward's last
  // kernel until every gradient bucket and the loss are allreduced (the
  // communication the backward did not hide)
  prof_mark(ctx, P_DP_WAIT, 0);
  if (split) CK(cudaStreamWaitEvent(st, ev_side(0, 3), 0));  // every gradient is in place before AdamW
  // loss: sum over valid rows (over all ranks) / number of valid rows; the
  // final kernel may follow an event wait, so it is launched normally
  set_pdl(false);
  float* total = ctx->row_loss + M;
  if (ctx->nccl) {
    CK(cudaEventRecord(ctx->ev_layer[0], st));
    CK(cudaStreamWaitEvent(ctx->comm, ctx->ev_layer[0], 0));
    CKS(nccl_wait(ctx, ncclAllReduce(total, total, 1, ncclFloat, ncclSum, ctx->nccl, ctx->comm), "loss allreduce"));
    CK(cudaEventRecord(ctx->ev_comm_done, ctx->comm));
    CK(cudaStreamWaitEvent(st, ctx->ev_comm_done, 0));
  }
  prof_mark(ctx, P_DP_WAIT, 0);
  prof_mark(ctx, P_FILL);
  scale_loss_kernel<<<1, 1, 0, st>>>(total, static_cast<float>(1.0 / n_valid_total), ctx->loss_dev);
  CK(cudaGetLastError());
  prof_mark(ctx, P_FILL);
  return LLMCU_OK;
}

llmcu_status validate_step(llmcu_ctx* ctx, int B, int S) {
  if (B <= 0 || S <= 1 || B > ctx->rc.max_batch || S > ctx->rc.max_seq)
    return fail(ctx, LLMCU_ERR_INVALID_ARG, "batch %d / seq %d outside [1, %d] x [2, %d]", B, S, ctx->rc.max_batch,
                ctx->rc.max_seq);
  return LLMCU_OK;
}

llmcu_status do_adamw(llmcu_ctx* ctx, const llmcu_adamw_cfg* o, int step) {
  if (!o || step < 1) return fail(ctx, LLMCU_ERR_INVALID_ARG, "adamw: null config or step < 1");
  const float bc1 = 1.0f - powf(o->beta1, static_cast<float>(step));
  const float bc2 = 1.0f - powf(o->beta2, static_cast<float>(step));
  TIMED(P_ADAMW, adamw_flat(ctx->lp, ctx->lg, ctx->lm, ctx->lv, ctx->n_lora, o->lr, o->beta1, o->beta2, o->eps, o->weight_decay,
                bc1, bc2, 1.0f, ctx->st));
  return LLMCU_OK;
}

llmcu_status upload_tokens(llmcu_ctx* ctx, const int32_t* tokens, const int32_t* targets, int M) {
  if (!tokens || !targets) return fail(ctx, LLMCU_ERR_INVALID_ARG, "null token pointer");
  CK(cudaMemcpyAsync(ctx->tok, tokens, sizeof(int) * M, cudaMemcpyHostToDevice, ctx->st));
  CK(cudaMemcpyAsync(ctx->tgt, targets, sizeof(int) * M, cudaMemcpyHostToDevice, ctx->st));
  return LLMCU_OK;
}

llmcu_status read_loss(llmcu_ctx* ctx, float* loss_out) {
  float h = 0.f;
  CK(cudaMemcpyAsync(&h, ctx->loss_dev, sizeof(float), cudaMemcpyDeviceToHost, ctx->st));
  CK(cudaEventRecord(ctx->ev_step_done, ctx->st));
  CKS(wait_event(ctx, ctx->ev_step_done));
  CKS(check_dev_err(ctx));
  if (loss_out) *loss_out = h;
  return LLMCU_OK;
}

}  // namespace

// ====================================================================== ABI

extern "C" {

const char* llmcu_version(void) { return "llmcu 1 sm_100a"; }

const char* llmcu_last_error(const llmcu_ctx* ctx) { return ctx ? ctx->err.c_str() : "null context"; }

size_t llmcu_device_bytes(const llmcu_ctx* ctx) { return ctx ? ctx->arena_bytes : 0; }

void* llmcu_stream(const llmcu_ctx* ctx) { return ctx ? static_cast<void*>(ctx->st) : nullptr; }

int64_t llmcu_lora_param_count(const llmcu_ctx* ctx) { return ctx ? ctx->n_lora : 0; }

int32_t llmcu_lora_targets(const llmcu_ctx* ctx) { return ctx ? static_cast<int32_t>(ctx->ld.targets) : 0; }

llmcu_status llmcu_ctx_create(const llmcu_model_cfg* model, const llmcu_lora_cfg* lora, const llmcu_run_cfg* run,
                              int device, llmcu_ctx** out) {
  if (!model || !lora || !run || !out) return LLMCU_ERR_INVALID_ARG;
  *out = nullptr;
  const llmcu_model_cfg& m = *model;
  if (m.hidden <= 0 || m.n_layers <= 0 || m.n_heads <= 0 || m.n_kv_heads <= 0 || m.vocab <= 0 || m.ffn <= 0)
    return LLMCU_ERR_INVALID_ARG;
  if (m.head_dim != 64 && m.head_dim != 128) return LLMCU_ERR_UNSUPPORTED;
  if (m.n_heads % m.n_kv_heads) return LLMCU_ERR_INVALID_ARG;
  if (m.hidden % 64 || m.ffn % 128 || m.vocab % 8) return LLMCU_ERR_UNSUPPORTED;
  if (lora->rank < 1 || lora->rank > 16) return LLMCU_ERR_UNSUPPORTED;
  const uint32_t targets = lora->targets ? static_cast<uint32_t>(lora->targets) : kTargetsAttn;
  if (targets & ~(kTargetsAttn | kTargetsMlp)) return LLMCU_ERR_INVALID_ARG;
  // the MLP's merged weights put their side columns on 256-column tile boundaries
  if ((targets & kTargetsMlp) && m.ffn % 256) return LLMCU_ERR_UNSUPPORTED;
  if (run->max_batch < 1 || run->max_seq < 2) return LLMCU_ERR_INVALID_ARG;
  if (run->base_dtype != LLMCU_BASE_FP16 && run->base_dtype != LLMCU_BASE_INT8) return LLMCU_ERR_INVALID_ARG;
  if (run->lm_head_chunk < 0 || run->lm_head_chunk % 256) return LLMCU_ERR_INVALID_ARG;
  if (run->deterministic != 0 && run->deterministic != 1) return LLMCU_ERR_INVALID_ARG;

  llmcu_ctx* ctx = new llmcu_ctx();
  ctx->m = m;
  ctx->lc = *lora;
  ctx->lc.targets = static_cast<int32_t>(targets);
  ctx->rc = *run;
  ctx->device = device;
  ctx->H = m.hidden;
  ctx->L = m.n_layers;
  ctx->nh = m.n_heads;
  ctx->nkv = m.n_kv_heads;
  ctx->hd = m.head_dim;
  ctx->Q = m.n_heads * m.head_dim;
  ctx->KV = m.n_kv_heads * m.head_dim;
  ctx->QKV = ctx->Q + 2 * ctx->KV;
  ctx->I = m.ffn;
  ctx->V = m.vocab;
  ctx->Mmax = run->max_batch * run->max_seq;
  ctx->ld = LoraDims::make(lora->rank, ctx->H, ctx->Q, ctx->KV, ctx->I, lora->alpha / static_cast<float>(lora->rank),
                           targets);
  ctx->n_lora = ctx->ld.per_layer * ctx->L;

  auto bail = [&](llmcu_status s) {
    llmcu_ctx_destroy(ctx);
    return s;
  };
  if (cudaSetDevice(device) != cudaSuccess) return bail(LLMCU_ERR_CUDA);
  if (cudaStreamCreateWithFlags(&ctx->st, cudaStreamNonBlocking) != cudaSuccess) return bail(LLMCU_ERR_CUDA);
  if (cudaStreamCreateWithFlags(&ctx->comm, cudaStreamNonBlocking) != cudaSuccess) return bail(LLMCU_ERR_CUDA);
  if (cudaStreamCreateWithFlags(&ctx->side, cudaStreamNonBlocking) != cudaSuccess) return bail(LLMCU_ERR_CUDA);
  Carver probe;
  carve(ctx, probe);
  ctx->arena_bytes = probe.off + 256;
  if (cudaMalloc(&ctx->arena, ctx->arena_bytes) != cudaSuccess) {
    cudaGetLastError();
    ctx->arena = nullptr;
    return bail(LLMCU_ERR_OOM);
  }
  Carver cv;
  cv.base = ctx->arena;
  carve(ctx, cv);
  ctx->ev_layer.assign(ctx->L, nullptr);
  for (auto& ev : ctx->ev_layer)
    if (cudaEventCreateWithFlags(&ev, cudaEventDisableTiming) != cudaSuccess) return bail(LLMCU_ERR_CUDA);
  ctx->ev_side.assign(4 * ctx->L, nullptr);
  for (auto& ev : ctx->ev_side)
    if (cudaEventCreateWithFlags(&ev, cudaEventDisableTiming) != cudaSuccess) return bail(LLMCU_ERR_CUDA);
  if (cudaEventCreateWithFlags(&ctx->ev_comm_done, cudaEventDisableTiming) != cudaSuccess) return bail(LLMCU_ERR_CUDA);
  if (cudaEventCreateWithFlags(&ctx->ev_dq_in, cudaEventDisableTiming) != cudaSuccess) return bail(LLMCU_ERR_CUDA);
  if (cudaEventCreateWithFlags(&ctx->ev_dq_done, cudaEventDisableTiming) != cudaSuccess) return bail(LLMCU_ERR_CUDA);
  if (cudaEventCreateWithFlags(&ctx->ev_step_done, cudaEventDisableTiming) != cudaSuccess) return bail(LLMCU_ERR_CUDA);
  // zero everything once (adapters A = B = 0, moments 0), norms = 1
  if (cudaMemsetAsync(ctx->arena, 0, ctx->arena_bytes, ctx->st) != cudaSuccess) return bail(LLMCU_ERR_CUDA);
  fill_f32(ctx->final_norm, ctx->H, 1.0f, ctx->st);
  for (auto& w : ctx->lw) {
    fill_f32(w.attn_norm, ctx->H, 1.0f, ctx->st);
    fill_f32(w.ffn_norm, ctx->H, 1.0f, ctx->st);
    fill_f32(w.q_norm, ctx->hd, 1.0f, ctx->st);
    fill_f32(w.k_norm, ctx->hd, 1.0f, ctx->st);
  }
  if (rope_tables(ctx->rope_cos, ctx->rope_sin, run->max_seq, ctx->hd, m.rope_theta, ctx->st) != cudaSuccess)
    return bail(LLMCU_ERR_CUDA);
  if (cudaStreamSynchronize(ctx->st) != cudaSuccess) return bail(LLMCU_ERR_CUDA);
  *out = ctx;
  return LLMCU_OK;
}

void llmcu_ctx_destroy(llmcu_ctx* ctx) {
  if (!ctx) return;
  cudaSetDevice(ctx->device);
  if (ctx->st) cudaStreamSynchronize(ctx->st);
  if (ctx->comm) cudaStreamSynchronize(ctx->comm);
  if (ctx->side) cudaStreamSynchronize(ctx->side);
  if (ctx->nccl) ncclCommDestroy(ctx->nccl);
  for (auto ev : ctx->ev_layer)
    if (ev) cudaEventDestroy(ev);
  for (auto ev : ctx->ev_side)
    if (ev) cudaEventDestroy(ev);
  for (auto ev : ctx->prof_ev)
    if (ev) cudaEventDestroy(ev);
  if (ctx->ev_comm_done) cudaEventDestroy(ctx->ev_comm_done);
  if (ctx->ev_dq_in) cudaEventDestroy(ctx->ev_dq_in);
  if (ctx->ev_dq_done) cudaEventDestroy(ctx->ev_dq_done);
  if (ctx->ev_step_done) cudaEventDestroy(ctx->ev_step_done);
  if (ctx->dec_graph) cudaGraphExecDestroy(ctx->dec_graph);
  if (ctx->arena) cudaFree(ctx->arena);
  if (ctx->st) cudaStreamDestroy(ctx->st);
  if (ctx->comm) cudaStreamDestroy(ctx->comm);
  if (ctx->side) cudaStreamDestroy(ctx->side);
  delete ctx;
}

llmcu_status llmcu_synchronize(llmcu_ctx* ctx) {
  if (!ctx) return LLMCU_ERR_INVALID_ARG;
  CK(cudaSetDevice(ctx->device));
  CK(cudaStreamSynchronize(ctx->st));
  CK(cudaStreamSynchronize(ctx->comm));
  CK(cudaStreamSynchronize(ctx->side));
  return LLMCU_OK;
}

// ---------------------------------------------------------------- weights

static llmcu_status upload_stage(llmcu_ctx* ctx, const float* host, size_t n) {
  if (n > ctx->stage_elems) return fail(ctx, LLMCU_ERR_INVALID_ARG, "tensor larger than the staging buffer");
  CK(cudaMemcpyAsync(ctx->stage, host, n * sizeof(float), cudaMemcpyHostToDevice, ctx->st));
  return LLMCU_OK;
}

// Places one fp32 [rows, cols] weight (already in ctx->stage) into the fused
// fp16 layout (row offset / gate-up interleave), or into the INT8 layout
// (per-row quantiser, src/kernels/quantize.cu:8-50).
static llmcu_status place_linear(llmcu_ctx* ctx, int rows, int cols, __half* w, int row_off, int interleave,
                                 int8_t* q, float* s) {
  if (ctx->rc.base_dtype != LLMCU_BASE_INT8) {
    CK(convert_weight(ctx->stage, rows, cols, w, cols, row_off, interleave, nullptr, 0, 0, ctx->st));
    return LLMCU_OK;
  }
  if (interleave) {
    // quantise into a temporary block then scatter 128-row blocks to the interleaved slots
    int8_t* tmp = reinterpret_cast<int8_t*>(ctx->dq_w);
    float* stmp = ctx->q_scale_tmp;
    CK(quantize_rows_int8(ctx->stage, rows, cols, tmp, stmp, ctx->st));
    for (int r0 = 0; r0 < rows; r0 += 128) {
      const int dst_row = (r0 >> 7) * 256 + (interleave == 2 ? 128 : 0);
      const int n = std::min(128, rows - r0);
      CK(cudaMemcpyAsync(q + static_cast<size_t>(dst_row) * cols, tmp + static_cast<size_t>(r0) * cols,
                         static_cast<size_t>(n) * cols, cudaMemcpyDeviceToDevice, ctx->st));
      CK(cudaMemcpyAsync(s + dst_row, stmp + r0, n * sizeof(float), cudaMemcpyDeviceToDevice, ctx->st));
    }
  } else {
    CK(quantize_rows_int8(ctx->stage, rows, cols, q + static_cast<size_t>(row_off) * cols, s + row_off, ctx->st));
  }
  return LLMCU_OK;
}

llmcu_status llmcu_set_base_tensor(llmcu_ctx* ctx, int id, int layer, const float* host) {
  if (!ctx || !host) return fail(ctx, LLMCU_ERR_INVALID_ARG, "null argument");
  CK(cudaSetDevice(ctx->device));
  const int H = ctx->H, Q = ctx->Q, KV = ctx->KV, I = ctx->I, V = ctx->V, hd = ctx->hd;
  const bool per_layer = id >= LLMCU_T_ATTN_NORM && id < LLMCU_T_COUNT;
  if (per_layer && (layer < 0 || layer >= ctx->L)) return fail(ctx, LLMCU_ERR_INVALID_ARG, "layer %d out of range", layer);
  const bool int8 = ctx->rc.base_dtype == LLMCU_BASE_INT8;
  switch (id) {
    case LLMCU_T_EMBED: {
      CKS(upload_stage(ctx, host, static_cast<size_t>(V) * H));
      if (!int8) {
        CK(convert_weight(ctx->stage, V, H, ctx->E, H, 0, 0, nullptr, 0, 0, ctx->st));
      } else {
        CK(quantize_rows_int8(ctx->stage, V, H, ctx->qE, ctx->sE, ctx->st));
        CK(dequant_rows_f16(ctx->qE, ctx->sE, V, H, ctx->E, ctx->st));
      }
      break;
    }
    case LLMCU_T_FINAL_NORM:
      CK(cudaMemcpyAsync(ctx->final_norm, host, H * sizeof(float), cudaMemcpyHostToDevice, ctx->st));
      break;
    case LLMCU_T_ATTN_NORM:
      CK(cudaMemcpyAsync(ctx->lw[layer].attn_norm, host, H * sizeof(float), cudaMemcpyHostToDevice, ctx->st));
      break;
    case LLMCU_T_FFN_NORM:
      CK(cudaMemcpyAsync(ctx->lw[layer].ffn_norm, host, H * sizeof(float), cudaMemcpyHostToDevice, ctx->st));
      break;
    case LLMCU_T_Q_NORM:
      CK(cudaMemcpyAsync(ctx->lw[layer].q_norm, host, hd * sizeof(float), cudaMemcpyHostToDevice, ctx->st));
      break;
    case LLMCU_T_K_NORM:
      CK(cudaMemcpyAsync(ctx->lw[layer].k_norm, host, hd * sizeof(float), cudaMemcpyHostToDevice, ctx->st));
      break;
    case LLMCU_T_WQ:
    case LLMCU_T_WK:
    case LLMCU_T_WV: {
      LayerW& w = ctx->lw[layer];
      const int rows = id == LLMCU_T_WQ ? Q : KV;
      const int off = id == LLMCU_T_WQ ? 0 : (id == LLMCU_T_WK ? Q : Q + KV);
      CKS(upload_stage(ctx, host, static_cast<size_t>(rows) * H));
      CKS(place_linear(ctx, rows, H, w.wqkv, off, 0, w.q_qkv, w.s_qkv));
      break;
    }
    case LLMCU_T_WO: {
      LayerW& w = ctx->lw[layer];
      CKS(upload_stage(ctx, host, static_cast<size_t>(H) * Q));
      CKS(place_linear(ctx, H, Q, w.wo, 0, 0, w.q_o, w.s_o));
      break;
    }
    case LLMCU_T_W_GATE:
    case LLMCU_T_W_UP: {
      LayerW& w = ctx->lw[layer];
      const int il = id == LLMCU_T_W_GATE ? 1 : 2;
      CKS(upload_stage(ctx, host, static_cast<size_t>(I) * H));
      CKS(place_linear(ctx, I, H, w.wgu, 0, il, w.q_gu, w.s_gu));
      break;
    }
    case LLMCU_T_W_DOWN: {
      LayerW& w = ctx->lw[layer];
      CKS(upload_stage(ctx, host, static_cast<size_t>(H) * I));
      CKS(place_linear(ctx, H, I, w.wd, 0, 0, w.q_d, w.s_d));
      break;
    }
    default:
      return fail(ctx, LLMCU_ERR_INVALID_ARG, "unknown tensor id %d", id);
  }
  CK(cudaStreamSynchronize(ctx->st));
  return LLMCU_OK;
}

llmcu_status llmcu_load_base_fp32_files(llmcu_ctx* ctx, const char* dir) {
  if (!ctx || !dir) return fail(ctx, LLMCU_ERR_INVALID_ARG, "null argument");
  const int H = ctx->H, Q = ctx->Q, KV = ctx->KV, I = ctx->I, V = ctx->V, hd = ctx->hd;
  std::vector<float> buf;
  auto load = [&](const std::string& name, size_t n) -> llmcu_status {
    const std::string path = std::string(dir) + "/" + name;
    FILE* f = fopen(path.c_str(), "rb");
    if (!f) return fail(ctx, LLMCU_ERR_IO, "cannot open %s", path.c_str());
    buf.resize(n);
    const size_t got = fread(buf.data(), sizeof(float), n, f);
    fclose(f);
    if (got != n) return fail(ctx, LLMCU_ERR_IO, "short read %s (%zu of %zu floats)", path.c_str(), got, n);
    return LLMCU_OK;
  };
  CKS(load("model.embed_tokens.weight.bin", static_cast<size_t>(V) * H));
  CKS(llmcu_set_base_tensor(ctx, LLMCU_T_EMBED, 0, buf.data()));
  CKS(load("model.norm.weight.bin", H));
  CKS(llmcu_set_base_tensor(ctx, LLMCU_T_FINAL_NORM, 0, buf.data()));
  struct F { const char* n; int id; size_t sz; };
  for (int l = 0; l < ctx->L; ++l) {
    const F fs[] = {
        {"input_layernorm.weight", LLMCU_T_ATTN_NORM, static_cast<size_t>(H)},
        {"post_attention_layernorm.weight", LLMCU_T_FFN_NORM, static_cast<size_t>(H)},
        {"self_attn.q_proj.weight", LLMCU_T_WQ, static_cast<size_t>(Q) * H},
        {"self_attn.k_proj.weight", LLMCU_T_WK, static_cast<size_t>(KV) * H},
        {"self_attn.v_proj.weight", LLMCU_T_WV, static_cast<size_t>(KV) * H},
        {"self_attn.o_proj.weight", LLMCU_T_WO, static_cast<size_t>(H) * Q},
        {"self_attn.q_norm.weight", LLMCU_T_Q_NORM, static_cast<size_t>(hd)},
        {"self_attn.k_norm.weight", LLMCU_T_K_NORM, static_cast<size_t>(hd)},
        {"mlp.gate_proj.weight", LLMCU_T_W_GATE, static_cast<size_t>(I) * H},
        {"mlp.up_proj.weight", LLMCU_T_W_UP, static_cast<size_t>(I) * H},
        {"mlp.down_proj.weight", LLMCU_T_W_DOWN, static_cast<size_t>(H) * I},
    };
    for (const F& f : fs) {
      char name[256];
      snprintf(name, sizeof(name), "model.layers.%d.%s.bin", l, f.n);
      CKS(load(name, f.sz));
      CKS(llmcu_set_base_tensor(ctx, f.id, l, buf.data()));
    }
  }
  return LLMCU_OK;
}

llmcu_status llmcu_init_base_synthetic(llmcu_ctx* ctx, uint64_t seed, float stddev) {
  if (!ctx) return LLMCU_ERR_INVALID_ARG;
  CK(cudaSetDevice(ctx->device));
  const int64_t H = ctx->H, Q = ctx->Q, QKV = ctx->QKV, I = ctx->I, V = ctx->V;
  cudaStream_t st = ctx->st;
  uint64_t k = seed * 1000003ull + 17;
  auto lin = [&](int rows, int cols, __half* w, int8_t* q, float* s) -> llmcu_status {
    const int64_t n = static_cast<int64_t>(rows) * cols;
    if (ctx->rc.base_dtype != LLMCU_BASE_INT8) {
      CK(fill_normal_f16(w, n, k++, stddev, st));
    } else {
      CK(fill_normal_f32(ctx->stage, n, k++, stddev, st));
      CK(quantize_rows_int8(ctx->stage, rows, cols, q, s, st));
    }
    return LLMCU_OK;
  };
  if (ctx->rc.base_dtype != LLMCU_BASE_INT8) {
    CK(fill_normal_f16(ctx->E, V * H, k++, stddev, st));
  } else {
    CK(fill_normal_f32(ctx->stage, V * H, k++, stddev, st));
    CK(quantize_rows_int8(ctx->stage, static_cast<int>(V), static_cast<int>(H), ctx->qE, ctx->sE, st));
    CK(dequant_rows_f16(ctx->qE, ctx->sE, static_cast<int>(V), static_cast<int>(H), ctx->E, st));
  }
  for (auto& w : ctx->lw) {
    CKS(lin(static_cast<int>(QKV), static_cast<int>(H), w.wqkv, w.q_qkv, w.s_qkv));
    CKS(lin(static_cast<int>(H), static_cast<int>(Q), w.wo, w.q_o, w.s_o));
    CKS(lin(static_cast<int>(2 * I), static_cast<int>(H), w.wgu, w.q_gu, w.s_gu));
    CKS(lin(static_cast<int>(H), static_cast<int>(I), w.wd, w.q_d, w.s_d));
  }
  CK(cudaStreamSynchronize(st));
  return LLMCU_OK;
}

// ------------------------------------------------------------------- LoRA

static llmcu_status check_proj(llmcu_ctx* ctx, int layer, int proj) {
  if (layer < 0 || layer >= ctx->L || proj < 0 || proj >= kNumProj)
    return fail(ctx, LLMCU_ERR_INVALID_ARG, "layer %d / proj %d out of range", layer, proj);
  if (!ctx->ld.has(proj))
    return fail(ctx, LLMCU_ERR_INVALID_ARG, "proj %d is not among the targets 0x%x", proj, ctx->ld.targets);
  return LLMCU_OK;
}

llmcu_status llmcu_set_lora(llmcu_ctx* ctx, int layer, int proj, const float* A, const float* B) {
  if (!ctx || !A || !B) return fail(ctx, LLMCU_ERR_INVALID_ARG, "null argument");
  CKS(check_proj(ctx, layer, proj));
  CK(cudaSetDevice(ctx->device));
  const LoraDims& d = ctx->ld;
  float* base = ctx->lp + d.per_layer * layer;
  const size_t nA = static_cast<size_t>(d.r) * d.d_in(proj), nB = static_cast<size_t>(d.d_out(proj)) * d.r;
  CK(cudaMemcpyAsync(base + d.offA(proj), A, nA * sizeof(float), cudaMemcpyHostToDevice, ctx->st));
  CK(cudaMemcpyAsync(base + d.offB(proj), B, nB * sizeof(float), cudaMemcpyHostToDevice, ctx->st));
  CK(cudaStreamSynchronize(ctx->st));
  return LLMCU_OK;
}

static llmcu_status get_pair(llmcu_ctx* ctx, const float* flat, int layer, int proj, float* A, float* B) {
  if (!ctx || !A || !B) return fail(ctx, LLMCU_ERR_INVALID_ARG, "null argument");
  CKS(check_proj(ctx, layer, proj));
  CK(cudaSetDevice(ctx->device));
  const LoraDims& d = ctx->ld;
  const float* base = flat + d.per_layer * layer;
  const size_t nA = static_cast<size_t>(d.r) * d.d_in(proj), nB = static_cast<size_t>(d.d_out(proj)) * d.r;
  CK(cudaStreamSynchronize(ctx->comm));
  CK(cudaMemcpyAsync(A, base + d.offA(proj), nA * sizeof(float), cudaMemcpyDeviceToHost, ctx->st));
  CK(cudaMemcpyAsync(B, base + d.offB(proj), nB * sizeof(float), cudaMemcpyDeviceToHost, ctx->st));
  CK(cudaStreamSynchronize(ctx->st));
  return LLMCU_OK;
}

llmcu_status llmcu_get_lora(llmcu_ctx* ctx, int layer, int proj, float* A, float* B) {
  return get_pair(ctx, ctx ? ctx->lp : nullptr, layer, proj, A, B);
}

llmcu_status llmcu_get_lora_grads(llmcu_ctx* ctx, int layer, int proj, float* dA, float* dB) {
  return get_pair(ctx, ctx ? ctx->lg : nullptr, layer, proj, dA, dB);
}

llmcu_status llmcu_init_lora_synthetic(llmcu_ctx* ctx, uint64_t seed, float b_std) {
  if (!ctx) return LLMCU_ERR_INVALID_ARG;
  CK(cudaSetDevice(ctx->device));
  const LoraDims& d = ctx->ld;
  uint64_t k = seed * 7919ull + 3;
  for (int l = 0; l < ctx->L; ++l) {
    float* base = ctx->lp + d.per_layer * l;
    for (int p = 0; p < kNumProj; ++p) {
      if (!d.has(p)) continue;
      const float bound = 1.0f / sqrtf(static_cast<float>(d.d_in(p)));
      CK(fill_uniform_f32(base + d.offA(p), static_cast<int64_t>(d.r) * d.d_in(p), k++, -bound, bound, ctx->st));
      CK(fill_normal_f32(base + d.offB(p), static_cast<int64_t>(d.d_out(p)) * d.r, k++, b_std, ctx->st));
    }
  }
  CK(cudaStreamSynchronize(ctx->st));
  return LLMCU_OK;
}

llmcu_status llmcu_reset_optimizer(llmcu_ctx* ctx) {
  if (!ctx) return LLMCU_ERR_INVALID_ARG;
  CK(cudaSetDevice(ctx->device));
  CK(cudaMemsetAsync(ctx->lm, 0, ctx->n_lora * sizeof(float), ctx->st));
  CK(cudaMemsetAsync(ctx->lv, 0, ctx->n_lora * sizeof(float), ctx->st));
  CK(cudaStreamSynchronize(ctx->st));
  return LLMCU_OK;
}

// ------------------------------------------------------------------ steps

llmcu_status llmcu_forward_backward(llmcu_ctx* ctx, const int32_t* tokens, const int32_t* targets, int batch, int seq,
                                    float* loss_out) {
  if (!ctx) return LLMCU_ERR_INVALID_ARG;
  CK(cudaSetDevice(ctx->device));
  CKS(validate_step(ctx, batch, seq));
  CKS(upload_tokens(ctx, tokens, targets, batch * seq));
  CKS(run_forward_backward(ctx, batch, seq));
  return read_loss(ctx, loss_out);
}

llmcu_status llmcu_adamw(llmcu_ctx* ctx, const llmcu_adamw_cfg* opt, int step) {
  if (!ctx) return LLMCU_ERR_INVALID_ARG;
  CK(cudaSetDevice(ctx->device));
  CKS(do_adamw(ctx, opt, step));
  CK(cudaStreamSynchronize(ctx->st));
  return LLMCU_OK;
}

llmcu_status llmcu_train_step(llmcu_ctx* ctx, const int32_t* tokens, const int32_t* targets, int batch, int seq,
                              const llmcu_adamw_cfg* opt, int step, float* loss_out) {
  if (!ctx) return LLMCU_ERR_INVALID_ARG;
  CK(cudaSetDevice(ctx->device));
  CKS(validate_step(ctx, batch, seq));
  if (!opt || step < 1) return fail(ctx, LLMCU_ERR_INVALID_ARG, "adamw: null config or step < 1");
  CKS(upload_tokens(ctx, tokens, targets, batch * seq));
  CKS(run_forward_backward(ctx, batch, seq));
  CKS(do_adamw(ctx, opt, step));
  return read_loss(ctx, loss_out);
}

llmcu_status llmcu_train_step_device(llmcu_ctx* ctx, const int32_t* d_tokens, const int32_t* d_targets, int batch,
                                     int seq, const llmcu_adamw_cfg* opt, int step) {
  if (!ctx || !d_tokens || !d_targets) return fail(ctx, LLMCU_ERR_INVALID_ARG, "null argument");
  CK(cudaSetDevice(ctx->device));
  CKS(validate_step(ctx, batch, seq));
  if (!opt || step < 1) return fail(ctx, LLMCU_ERR_INVALID_ARG, "adamw: null config or step < 1");
  const int M = batch * seq;
  CK(cudaMemcpyAsync(ctx->tok, d_tokens, sizeof(int) * M, cudaMemcpyDeviceToDevice, ctx->st));
  CK(cudaMemcpyAsync(ctx->tgt, d_targets, sizeof(int) * M, cudaMemcpyDeviceToDevice, ctx->st));
  CKS(run_forward_backward(ctx, batch, seq));
  CKS(do_adamw(ctx, opt, step));
  return LLMCU_OK;
}

llmcu_status llmcu_read_loss(llmcu_ctx* ctx, float* loss_out) {
  if (!ctx) return LLMCU_ERR_INVALID_ARG;
  CK(cudaSetDevice(ctx->device));
  return read_loss(ctx, loss_out);
}

// ---------------------------------------------------------- checkpointing

// file-name parts of the adapters (the reference's four, then the MLP's, named
// like the base weights they adapt)
static const char* kProjNames[kNumProj] = {"wq", "wk", "wv", "wo", "w_gate", "w_up", "w_down"};

// The adapter files of one step (src/train.cu:146-170's names and layout:
// dir/lora_step{step}_layer{l}_{proj}_{A,B}.bin, raw fp32, A [r, d_in],
// B [d_out, r], no header) from / into the flat host layout of `d`.  `what`
// receives the failing path.
static llmcu_status lora_files_io(const LoraDims& d, int n_layers, float* flat, const char* dir, int step, bool write,
                                  std::string* what) {
  for (int l = 0; l < n_layers; ++l) {
    float* base = flat + d.per_layer * l;
    for (int p = 0; p < kNumProj; ++p) {
      if (!d.has(p)) continue;
      const size_t n[2] = {static_cast<size_t>(d.r) * d.d_in(p), static_cast<size_t>(d.d_out(p)) * d.r};
      float* part[2] = {base + d.offA(p), base + d.offB(p)};
      const char* ab[2] = {"A", "B"};
      for (int i = 0; i < 2; ++i) {
        char path[1024];
        snprintf(path, sizeof(path), "%s/lora_step%d_layer%d_%s_%s.bin", dir, step, l, kProjNames[p], ab[i]);
        *what = path;
        FILE* f = fopen(path, write ? "wb" : "rb");
        if (!f) return LLMCU_ERR_IO;
        const size_t got = write ? fwrite(part[i], sizeof(float), n[i], f) : fread(part[i], sizeof(float), n[i], f);
        const bool closed = fclose(f) == 0;
        if (got != n[i] || !closed) return LLMCU_ERR_IO;
      }
    }
  }
  return LLMCU_OK;
}

static bool layout_dims(const llmcu_lora_layout* lay, LoraDims* d) {
  if (!lay || lay->n_layers <= 0 || lay->hidden <= 0 || lay->q_dim <= 0 || lay->kv_dim <= 0 || lay->ffn <= 0 ||
      lay->rank < 1 || lay->rank > 16)
    return false;
  const uint32_t t = lay->targets ? static_cast<uint32_t>(lay->targets) : kTargetsAttn;
  if (t & ~(kTargetsAttn | kTargetsMlp)) return false;
  *d = LoraDims::make(lay->rank, lay->hidden, lay->q_dim, lay->kv_dim, lay->ffn, 1.0f, t);
  return true;
}

int64_t llmcu_lora_layout_count(const llmcu_lora_layout* lay) {
  LoraDims d;
  return layout_dims(lay, &d) ? d.per_layer * lay->n_layers : 0;
}

llmcu_status llmcu_lora_files_write(const llmcu_lora_layout* lay, const float* flat, const char* dir, int step) {
  LoraDims d;
  if (!flat || !dir || !layout_dims(lay, &d)) return LLMCU_ERR_INVALID_ARG;
  std::string what;
  return lora_files_io(d, lay->n_layers, const_cast<float*>(flat), dir, step, true, &what);
}

llmcu_status llmcu_lora_files_read(const llmcu_lora_layout* lay, float* flat, const char* dir, int step) {
  LoraDims d;
  if (!flat || !dir || !layout_dims(lay, &d)) return LLMCU_ERR_INVALID_ARG;
  std::string what;
  return lora_files_io(d, lay->n_layers, flat, dir, step, false, &what);
}

llmcu_status llmcu_save_lora(llmcu_ctx* ctx, const char* dir, int step) {
  if (!ctx || !dir) return fail(ctx, LLMCU_ERR_INVALID_ARG, "null argument");
  CK(cudaSetDevice(ctx->device));
  std::vector<float> flat(static_cast<size_t>(ctx->n_lora));
  CK(cudaStreamSynchronize(ctx->comm));
  CK(cudaMemcpyAsync(flat.data(), ctx->lp, flat.size() * sizeof(float), cudaMemcpyDeviceToHost, ctx->st));
  CK(cudaStreamSynchronize(ctx->st));
  std::string what;
  if (lora_files_io(ctx->ld, ctx->L, flat.data(), dir, step, true, &what) != LLMCU_OK)
    return fail(ctx, LLMCU_ERR_IO, "cannot write %s", what.c_str());
  return LLMCU_OK;
}

llmcu_status llmcu_load_lora(llmcu_ctx* ctx, const char* dir, int step) {
  if (!ctx || !dir) return fail(ctx, LLMCU_ERR_INVALID_ARG, "null argument");
  CK(cudaSetDevice(ctx->device));
  std::vector<float> flat(static_cast<size_t>(ctx->n_lora));
  std::string what;
  if (lora_files_io(ctx->ld, ctx->L, flat.data(), dir, step, false, &what) != LLMCU_OK)
    return fail(ctx, LLMCU_ERR_IO, "cannot read %s (missing or short)", what.c_str());
  CK(cudaMemcpyAsync(ctx->lp, flat.data(), flat.size() * sizeof(float), cudaMemcpyHostToDevice, ctx->st));
  CK(cudaStreamSynchronize(ctx->st));
  return LLMCU_OK;
}

// ------------------------------------------------------------- generation
namespace {

// One decode step (llm_engine's transformer_decode, src/kernels/forward.cu:340-394)
// for the token dec_cnt[2] at position dec_cnt[0], both read on the device:
// GEMVs over the merged q/k/v/o weights and the base (or, with MLP targets,
// merged) MLP and lm_head rows (INT8 rows with their scales for an INT8
// base), the cache append inside the
// QK-norm/RoPE kernel, split attention over the cache and the argmax that
// chooses the next token.
llmcu_status decode_step(llmcu_ctx* ctx, float* step_logits) {
  const int H = ctx->H, Q = ctx->Q, KV = ctx->KV, QKV = ctx->QKV, I = ctx->I, V = ctx->V;
  const float eps = ctx->m.rms_eps;
  cudaStream_t st = ctx->st;
  const bool int8 = ctx->rc.base_dtype == LLMCU_BASE_INT8;
  const size_t ctxlen = static_cast<size_t>(ctx->rc.max_seq);
  CK(embed_forward(ctx->dec_cnt + 2, ctx->E, ctx->dec_x, 1, H, V, ctx->derr, st));
  for (int l = 0; l < ctx->L; ++l) {
    LayerW& w = ctx->lw[l];
    __half* kc = ctx->kc + l * ctxlen * KV;
    __half* vc = ctx->vc + l * ctxlen * KV;
    CK(decode_gemv(w.mqkv, nullptr, false, H + 64, ctx->dec_x, 1, w.attn_norm, eps, QKV, H, nullptr, nullptr,
                   ctx->dec_qkv, st));
    CK(decode_attention(ctx->dec_qkv, w.q_norm, w.k_norm, ctx->rope_cos, ctx->rope_sin, ctx->dec_cnt, kc, vc,
                        ctx->dec_part, ctx->dec_tickets, ctx->dec_attn, ctx->nh, ctx->nkv, ctx->hd, eps, ctx->rc.max_seq,
                        st));
    CK(decode_gemv(w.mo, nullptr, false, Q + 64, ctx->dec_attn, 0, nullptr, 0.f, H, Q, ctx->dec_x, ctx->dec_xmid,
                   nullptr, st));
    // ffn norm folded into the gate/up GEMV, SwiGLU into the down GEMV; with
    // MLP targets both read the merged fp16 rows (their pads are skipped)
    if (w.mgu) {
      CK(decode_gemv(w.mgu, nullptr, false, H + 64, ctx->dec_xmid, 1, w.ffn_norm, eps, 2 * I, H, nullptr, nullptr,
                     ctx->dec_gu, st));
      CK(decode_gemv(w.md, nullptr, false, I + 64, ctx->dec_gu, 2, nullptr, 0.f, H, I, ctx->dec_xmid, ctx->dec_x,
                     nullptr, st));
      continue;
    }
    if (int8)
      CK(decode_gemv(w.q_gu, w.s_gu, true, H, ctx->dec_xmid, 1, w.ffn_norm, eps, 2 * I, H, nullptr, nullptr,
                     ctx->dec_gu, st));
    else
      CK(decode_gemv(w.wgu, nullptr, false, H, ctx->dec_xmid, 1, w.ffn_norm, eps, 2 * I, H, nullptr, nullptr,
                     ctx->dec_gu, st));
    if (int8)
      CK(decode_gemv(w.q_d, w.s_d, true, I, ctx->dec_gu, 2, nullptr, 0.f, H, I, ctx->dec_xmid, ctx->dec_x, nullptr,
                     st));
    else
      CK(decode_gemv(w.wd, nullptr, false, I, ctx->dec_gu, 2, nullptr, 0.f, H, I, ctx->dec_xmid, ctx->dec_x, nullptr,
                     st));
  }
  if (int8)
    CK(decode_gemv(ctx->qE, ctx->sE, true, H, ctx->dec_x, 1, ctx->final_norm, eps, V, H, nullptr, ctx->dec_logits,
                   nullptr, st));
  else
    CK(decode_gemv(ctx->E, nullptr, false, H, ctx->dec_x, 1, ctx->final_norm, eps, V, H, nullptr, ctx->dec_logits,
                   nullptr, st));
  CK(decode_argmax(ctx->dec_logits, V, ctx->dec_cnt, ctx->dec_tok, step_logits, ctx->dec_amax, st));
  return LLMCU_OK;
}

// The decode step as a CUDA graph (its kernels read the position on the
// device, so one capture serves every token of every generate call).
llmcu_status decode_graph(llmcu_ctx* ctx) {
  if (ctx->dec_graph) return LLMCU_OK;
  CK(cudaStreamBeginCapture(ctx->st, cudaStreamCaptureModeThreadLocal));
  const llmcu_status s = decode_step(ctx, nullptr);
  cudaGraph_t g = nullptr;
  const cudaError_t e = cudaStreamEndCapture(ctx->st, &g);
  if (s != LLMCU_OK) {
    if (g) cudaGraphDestroy(g);
    return s;
  }
  CK(e);
  const cudaError_t ei = cudaGraphInstantiate(&ctx->dec_graph, g, 0);
  cudaGraphDestroy(g);
  CK(ei);
  return LLMCU_OK;
}

constexpr int kQwenEos[2] = {151643, 151645};  // the ids llm_engine stops at (src/main.cu:368)

}  // namespace

llmcu_status llmcu_generate(llmcu_ctx* ctx, const int32_t* prompt, int n_prompt, int n_new, int32_t* out_tokens,
                            int* n_out, float* step_logits, float* decode_ms) {
  if (!ctx || !prompt || !out_tokens || n_prompt < 1 || n_new < 1)
    return fail(ctx, LLMCU_ERR_INVALID_ARG, "generate: null pointer or empty prompt / request");
  if (n_prompt + n_new > ctx->rc.max_seq)
    return fail(ctx, LLMCU_ERR_INVALID_ARG, "generate: %d prompt + %d new tokens exceed max_seq %d", n_prompt, n_new,
                ctx->rc.max_seq);
  CK(cudaSetDevice(ctx->device));
  const int H = ctx->H, Q = ctx->Q, KV = ctx->KV, QKV = ctx->QKV, V = ctx->V, L = ctx->L;
  const size_t ctxlen = static_cast<size_t>(ctx->rc.max_seq);
  cudaStream_t st = ctx->st;
  const float eps = ctx->m.rms_eps;
  CK(cudaMemcpyAsync(ctx->tok, prompt, sizeof(int32_t) * n_prompt, cudaMemcpyHostToDevice, st));
  float* dlog = nullptr;  // logits history, only when the caller asks for it
  if (step_logits) CK(cudaMalloc(&dlog, sizeof(float) * static_cast<size_t>(n_new) * V));
  struct Cleanup {
    float* p;
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    ~Cleanup() {
      set_pdl(false);
      if (p) cudaFree(p);
      if (e0) cudaEventDestroy(e0);
      if (e1) cudaEventDestroy(e1);
    }
  } cleanup{dlog};
  CK(cudaEventCreate(&cleanup.e0));
  CK(cudaEventCreate(&cleanup.e1));
  // merged weights of the current adapters, then the prompt through the batched forward
  set_pdl(false);
  CK(merge_adapters(ctx));
  CK(cudaMemsetAsync(ctx->fx_cnt, 0, sizeof(int) * kFxCounters, st));
  set_pdl(true);
  {
    GemmWorkspaceScope gws(ctx);
    CKS(forward_layers(ctx, 1, n_prompt));
  }
  set_pdl(false);
  for (int l = 0; l < L; ++l) {  // cache rows 0 .. n_prompt - 1: rotated k, raw v
    const LayerA& a = ctx->la[l];
    CK(cudaMemcpy2DAsync(ctx->kc + l * ctxlen * KV, sizeof(__half) * KV, a.qkr + Q, sizeof(__half) * (Q + KV),
                         sizeof(__half) * KV, n_prompt, cudaMemcpyDeviceToDevice, st));
    CK(cudaMemcpy2DAsync(ctx->vc + l * ctxlen * KV, sizeof(__half) * KV, a.qkv + Q + KV, sizeof(__half) * QKV,
                         sizeof(__half) * KV, n_prompt, cudaMemcpyDeviceToDevice, st));
  }
  const int init[4] = {n_prompt - 1, 0, 0, 0};  // the argmax advances the position to n_prompt
  CK(cudaMemcpyAsync(ctx->dec_cnt, init, sizeof(init), cudaMemcpyHostToDevice, st));
  // first token: final norm + lm_head of the prompt's last position
  const float* xlast = ctx->resid[L] + static_cast<size_t>(n_prompt - 1) * H;
  if (ctx->rc.base_dtype == LLMCU_BASE_INT8)
    CK(decode_gemv(ctx->qE, ctx->sE, true, H, xlast, 1, ctx->final_norm, eps, V, H, nullptr, ctx->dec_logits,
                   nullptr, st));
  else
    CK(decode_gemv(ctx->E, nullptr, false, H, xlast, 1, ctx->final_norm, eps, V, H, nullptr, ctx->dec_logits, nullptr,
                   st));
  CK(decode_argmax(ctx->dec_logits, V, ctx->dec_cnt, ctx->dec_tok, dlog, ctx->dec_amax, st));
  if (!dlog && n_new > 1) CKS(decode_graph(ctx));
  CK(cudaEventRecord(cleanup.e0, st));
  set_pdl(true);
  for (int t = 1; t < n_new; ++t) {
    if (dlog)
      CKS(decode_step(ctx, dlog));
    else
      CK(cudaGraphLaunch(ctx->dec_graph, st));
  }
  set_pdl(false);
  CK(cudaEventRecord(cleanup.e1, st));
  CK(cudaEventSynchronize(cleanup.e1));
  CKS(check_dev_err(ctx));
  std::vector<int32_t> toks(n_new);
  CK(cudaMemcpy(toks.data(), ctx->dec_tok, sizeof(int32_t) * n_new, cudaMemcpyDeviceToHost));
  int n = n_new;
  if (V > kQwenEos[1])
    for (int i = 0; i < n_new; ++i)
      if (toks[i] == kQwenEos[0] || toks[i] == kQwenEos[1]) {
        n = i;
        break;
      }
  memcpy(out_tokens, toks.data(), sizeof(int32_t) * n_new);
  if (n_out) *n_out = n;
  if (step_logits) CK(cudaMemcpy(step_logits, dlog, sizeof(float) * static_cast<size_t>(n_new) * V,
                                 cudaMemcpyDeviceToHost));
  if (decode_ms) {
    float ms = 0.f;
    CK(cudaEventElapsedTime(&ms, cleanup.e0, cleanup.e1));
    *decode_ms = n_new > 1 ? ms / static_cast<float>(n_new - 1) : 0.f;
  }
  return LLMCU_OK;
}

// ----------------------------------------------------- optimizer sidecar
// dir/lora_step{N}_adamw.bin: a 64-byte header, then the AdamW first and
// second moments of every adapter in the flat layout (per layer Aq Bq Ak Bk
// Av Bv Ao Bo; A [r, in], B [out, r]), fp32.  The reference saves A and B
// only (src/train.cu:146-170) and cannot resume; with this file and the
// A / B files of the same step a run continues where it stopped.
namespace {
struct AdamwHeader {
  char magic[8];  // "LLMCUADW"
  int32_t version, step, n_layers, rank, hidden, q_dim, kv_dim;
  int32_t targets;  // adapter mask; 0 reads as q/k/v/o
  int64_t n_params;
  int64_t reserved2[2];
};
static_assert(sizeof(AdamwHeader) == 64, "sidecar header is 64 bytes");
constexpr char kAdamwMagic[8] = {'L', 'L', 'M', 'C', 'U', 'A', 'D', 'W'};

void adamw_path(char* path, size_t n, const char* dir, int step) {
  snprintf(path, n, "%s/lora_step%d_adamw.bin", dir, step);
}
}  // namespace

llmcu_status llmcu_save_adamw_state(llmcu_ctx* ctx, const char* dir, int step) {
  if (!ctx || !dir || step < 0) return fail(ctx, LLMCU_ERR_INVALID_ARG, "null argument or negative step");
  const size_t n = static_cast<size_t>(ctx->n_lora);
  std::vector<float> m(n), v(n);
  CK(cudaMemcpyAsync(m.data(), ctx->lm, n * sizeof(float), cudaMemcpyDeviceToHost, ctx->st));
  CK(cudaMemcpyAsync(v.data(), ctx->lv, n * sizeof(float), cudaMemcpyDeviceToHost, ctx->st));
  CK(cudaStreamSynchronize(ctx->st));
  AdamwHeader h{};
  memcpy(h.magic, kAdamwMagic, 8);
  h.version = 1;
  h.step = step;
  h.n_layers = ctx->L;
  h.rank = ctx->ld.r;
  h.hidden = ctx->H;
  h.q_dim = ctx->Q;
  h.kv_dim = ctx->KV;
  h.targets = static_cast<int32_t>(ctx->ld.targets);
  h.n_params = ctx->n_lora;
  char path[1024];
  adamw_path(path, sizeof(path), dir, step);
  FILE* f = fopen(path, "wb");
  if (!f) return fail(ctx, LLMCU_ERR_IO, "cannot write %s", path);
  const bool ok = fwrite(&h, sizeof(h), 1, f) == 1 && fwrite(m.data(), sizeof(float), n, f) == n &&
                  fwrite(v.data(), sizeof(float), n, f) == n;
  const bool closed = fclose(f) == 0;
  if (!ok || !closed) return fail(ctx, LLMCU_ERR_IO, "short write %s", path);
  return LLMCU_OK;
}

llmcu_status llmcu_load_adamw_state(llmcu_ctx* ctx, const char* dir, int step) {
  if (!ctx || !dir || step < 0) return fail(ctx, LLMCU_ERR_INVALID_ARG, "null argument or negative step");
  char path[1024];
  adamw_path(path, sizeof(path), dir, step);
  FILE* f = fopen(path, "rb");
  if (!f) return fail(ctx, LLMCU_ERR_IO, "cannot open %s", path);
  AdamwHeader h{};
  if (fread(&h, sizeof(h), 1, f) != 1 || memcmp(h.magic, kAdamwMagic, 8) != 0 || h.version != 1) {
    fclose(f);
    return fail(ctx, LLMCU_ERR_IO, "%s is not an AdamW state file", path);
  }
  const uint32_t file_targets = h.targets ? static_cast<uint32_t>(h.targets) : kTargetsAttn;
  if (h.step != step || h.n_layers != ctx->L || h.rank != ctx->ld.r || h.hidden != ctx->H || h.q_dim != ctx->Q ||
      h.kv_dim != ctx->KV || h.n_params != ctx->n_lora || file_targets != ctx->ld.targets) {
    fclose(f);
    return fail(ctx, LLMCU_ERR_INVALID_ARG,
                "%s holds step %d, %d layers, rank %d, dims %d/%d/%d, targets 0x%x (%lld params); this context has "
                "%d layers, rank %d, dims %d/%d/%d, targets 0x%x (%lld params)",
                path, h.step, h.n_layers, h.rank, h.hidden, h.q_dim, h.kv_dim, file_targets,
                static_cast<long long>(h.n_params), ctx->L, ctx->ld.r, ctx->H, ctx->Q, ctx->KV, ctx->ld.targets,
                static_cast<long long>(ctx->n_lora));
  }
  const size_t n = static_cast<size_t>(ctx->n_lora);
  std::vector<float> m(n), v(n);
  const bool ok = fread(m.data(), sizeof(float), n, f) == n && fread(v.data(), sizeof(float), n, f) == n;
  fclose(f);
  if (!ok) return fail(ctx, LLMCU_ERR_IO, "short read %s", path);
  CK(cudaMemcpyAsync(ctx->lm, m.data(), n * sizeof(float), cudaMemcpyHostToDevice, ctx->st));
  CK(cudaMemcpyAsync(ctx->lv, v.data(), n * sizeof(float), cudaMemcpyHostToDevice, ctx->st));
  CK(cudaStreamSynchronize(ctx->st));
  return LLMCU_OK;
}

// ------------------------------------------------------------------- INT8

llmcu_status llmcu_quantize_int8_rows(const float* w, int rows, int cols, int8_t* q, float* scale, void* stream) {
  if (!w || !q || !scale || rows <= 0 || cols <= 0) return LLMCU_ERR_INVALID_ARG;
  if (quantize_rows_int8(w, rows, cols, q, scale, static_cast<cudaStream_t>(stream)) != cudaSuccess)
    return LLMCU_ERR_CUDA;
  return LLMCU_OK;
}

// ---------------------------------------------------------- data parallel

llmcu_status llmcu_dp_get_unique_id(void* id128) {
  if (!id128) return LLMCU_ERR_INVALID_ARG;
  static_assert(sizeof(ncclUniqueId) == 128, "NCCL unique id size");
  ncclUniqueId id;
  if (ncclGetUniqueId(&id) != ncclSuccess) return LLMCU_ERR_NCCL;
  memcpy(id128, &id, sizeof(id));
  return LLMCU_OK;
}

llmcu_status llmcu_dp_set_timeout_ms(llmcu_ctx* ctx, int ms) {
  if (!ctx || ms <= 0) return LLMCU_ERR_INVALID_ARG;
  ctx->timeout_ms = ms;
  return LLMCU_OK;
}

llmcu_status llmcu_dp_init(llmcu_ctx* ctx, const void* id128, int rank, int world) {
  if (!ctx || !id128 || world < 1 || rank < 0 || rank >= world) return fail(ctx, LLMCU_ERR_INVALID_ARG, "bad dp args");
  CK(cudaSetDevice(ctx->device));
  if (ctx->nccl) return fail(ctx, LLMCU_ERR_INVALID_ARG, "data parallel group already initialised");
  if (world == 1) return LLMCU_OK;
  ncclUniqueId id;
  memcpy(&id, id128, sizeof(id));
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  ncclComm_t comm = nullptr;
  ncclResult_t r = ncclCommInitRankConfig(&comm, world, id, rank, &cfg);
  ctx->nccl = comm;
  llmcu_status s = nccl_wait(ctx, r, "ncclCommInitRankConfig");
  if (s != LLMCU_OK) {
    if (ctx->nccl) {
      ncclCommAbort(ctx->nccl);
      ctx->nccl = nullptr;
    }
    return s;
  }
  ctx->rank = rank;
  ctx->world = world;
  return LLMCU_OK;
}

// -------------------------------------------------------------- profiling

static void prof_collect(llmcu_ctx* ctx) {
  if (ctx->prof_n == 0) return;
  cudaEventSynchronize(ctx->prof_ev[ctx->prof_n - 1]);
  for (int i = 0; i + 1 < ctx->prof_n; i += 2) {
    float ms = 0.f;
    if (cudaEventElapsedTime(&ms, ctx->prof_ev[i], ctx->prof_ev[i + 1]) == cudaSuccess) {
      const int c = ctx->prof_cls[i / 2];
      ctx->prof_ms[c] += ms;
      ctx->prof_cnt[c] += ctx->prof_k[i / 2];
    }
  }
  ctx->prof_n = 0;
  ctx->prof_cls.clear();
  ctx->prof_k.clear();
}

llmcu_status llmcu_profile_enable(llmcu_ctx* ctx, int on) {
  if (!ctx) return LLMCU_ERR_INVALID_ARG;
  CK(cudaSetDevice(ctx->device));
  if (on && ctx->prof_ev.empty()) {
    ctx->prof_ev.resize(8192);
    for (auto& ev : ctx->prof_ev) CK(cudaEventCreate(&ev));
  }
  if (!on) prof_collect(ctx);
  ctx->prof_on = on != 0;
  return LLMCU_OK;
}

llmcu_status llmcu_profile_read(llmcu_ctx* ctx, char* buf, size_t len, int reset) {
  if (!ctx || !buf || len == 0) return LLMCU_ERR_INVALID_ARG;
  CK(cudaSetDevice(ctx->device));
  prof_collect(ctx);
  std::string out = "{";
  for (int c = 0; c < P_COUNT; ++c) {
    char item[160];
    snprintf(item, sizeof(item), "%s\"%s\": {\"ms\": %.6f, \"launches\": %lld}", c ? ", " : "", kProfNames[c],
             ctx->prof_ms[c], static_cast<long long>(ctx->prof_cnt[c]));
    out += item;
  }
  out += "}";
  if (out.size() + 1 > len) return fail(ctx, LLMCU_ERR_INVALID_ARG, "profile buffer too small");
  memcpy(buf, out.c_str(), out.size() + 1);
  if (reset) {
    for (int c = 0; c < P_COUNT; ++c) {
      ctx->prof_ms[c] = 0;
      ctx->prof_cnt[c] = 0;
    }
  }
  return LLMCU_OK;
}

// ------------------------------------------------------------ kernel test

}  // extern "C"

namespace llmcu {
// The kernel-level entry points' device error word (one per device: every
// device that loads the library holds its own copy).
static __device__ int g_kernel_err;

cudaError_t kernel_err_word(int** out) {
  void* p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_kernel_err);
  *out = static_cast<int*>(p);
  return e;
}
}  // namespace llmcu

namespace {
// cudaErrorInvalidValue comes from the launchers refusing a pointer, stride
// or shape (TMA descriptors need 16-byte aligned bases and strides).
llmcu_status kernel_status(cudaError_t e) {
  return e == cudaSuccess ? LLMCU_OK : (e == cudaErrorInvalidValue ? LLMCU_ERR_UNSUPPORTED : LLMCU_ERR_CUDA);
}
}  // namespace

extern "C" {

llmcu_status llmcu_kernel_checks(void* stream, int* bits) {
  int* w = nullptr;
  if (kernel_err_word(&w) != cudaSuccess) return LLMCU_ERR_CUDA;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int h = 0;
  if (cudaMemcpyAsync(&h, w, sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess) return LLMCU_ERR_CUDA;
  if (cudaStreamSynchronize(st) != cudaSuccess) return LLMCU_ERR_CUDA;
  if (h && cudaMemsetAsync(w, 0, sizeof(int), st) != cudaSuccess) return LLMCU_ERR_CUDA;
  if (h && cudaStreamSynchronize(st) != cudaSuccess) return LLMCU_ERR_CUDA;
  if (bits) *bits = h;
  return h ? LLMCU_ERR_DEVICE_CHECK : LLMCU_OK;
}

llmcu_status llmcu_kernel_wait_selftest(void* stream) {
  int* d_err = nullptr;
  if (kernel_err_word(&d_err) != cudaSuccess) return LLMCU_ERR_CUDA;
  return wait_selftest(d_err, static_cast<cudaStream_t>(stream)) == cudaSuccess ? LLMCU_OK : LLMCU_ERR_CUDA;
}

llmcu_status llmcu_gemm_nt_f16(const void* A, const void* B, float* C, int M, int N, int K, int lda, int ldb, int ldc,
                               void* stream) {
  if (!A || !B || !C || M <= 0 || N <= 0 || K <= 0) return LLMCU_ERR_INVALID_ARG;
  int* d_err = nullptr;
  if (kernel_err_word(&d_err) != cudaSuccess) return LLMCU_ERR_CUDA;
  EpiArgs ea;
  ea.out = C;
  ea.ld_out = ldc;
  cudaError_t e = gemm(op(static_cast<const __half*>(A), M, K, lda), op(static_cast<const __half*>(B), N, K, ldb), M,
                       N, Epi::kStoreF32, ea, d_err, static_cast<cudaStream_t>(stream));
  return kernel_status(e);
}

llmcu_status llmcu_gemm_nn_f16(const void* A, const void* B, float* C, int M, int N, int K, int lda, int ldb, int ldc,
                               void* stream) {
  if (!A || !B || !C || M <= 0 || N <= 0 || K <= 0) return LLMCU_ERR_INVALID_ARG;
  int* d_err = nullptr;
  if (kernel_err_word(&d_err) != cudaSuccess) return LLMCU_ERR_CUDA;
  EpiArgs ea;
  ea.out = C;
  ea.ld_out = ldc;
  cudaError_t e = gemm(op(static_cast<const __half*>(A), M, K, lda), op_mn(static_cast<const __half*>(B), K, N, ldb),
                       M, N, Epi::kStoreF32, ea, d_err, static_cast<cudaStream_t>(stream));
  return kernel_status(e);
}

llmcu_status llmcu_attention_fwd(const void* q, const void* k, const void* v, void* o, float* lse, int batch, int seq,
                                 int n_heads, int n_kv_heads, int head_dim, int ldq, int ldk, int ldv, void* stream) {
  if (!q || !k || !v || !o || !lse || batch <= 0 || seq <= 0 || n_heads <= 0 || n_kv_heads <= 0 ||
      n_heads % n_kv_heads)
    return LLMCU_ERR_INVALID_ARG;
  int* d_err = nullptr;
  if (kernel_err_word(&d_err) != cudaSuccess) return LLMCU_ERR_CUDA;
  cudaError_t e = attention_forward(static_cast<const __half*>(q), static_cast<const __half*>(k),
                                    static_cast<const __half*>(v), static_cast<__half*>(o), lse, batch, seq, n_heads,
                                    n_kv_heads, head_dim, ldq, ldk, ldv, n_heads * head_dim, d_err,
                                    static_cast<cudaStream_t>(stream));
  return kernel_status(e);
}

llmcu_status llmcu_attention_bwd(const void* q, const void* k, const void* v, const void* o, const void* dout,
                                 const float* lse, float* scratch_delta, float* dq, float* dk, void* dv, int batch,
                                 int seq, int n_heads, int n_kv_heads, int head_dim, int ldq, int ldk, int ldv,
                                 int lddv, void* stream) {
  if (!q || !k || !v || !o || !dout || !lse || !scratch_delta || !dq || !dk || !dv || batch <= 0 || seq <= 0 ||
      n_heads <= 0 || n_kv_heads <= 0 || n_heads % n_kv_heads)
    return LLMCU_ERR_INVALID_ARG;
  int* d_err = nullptr;
  if (kernel_err_word(&d_err) != cudaSuccess) return LLMCU_ERR_CUDA;
  const int ldo = n_heads * head_dim;
  cudaError_t e = attention_backward(
      static_cast<const __half*>(q), static_cast<const __half*>(k), static_cast<const __half*>(v),
      static_cast<const __half*>(o), static_cast<const __half*>(dout), lse, scratch_delta, dq, dk,
      static_cast<__half*>(dv), batch, seq, n_heads, n_kv_heads, head_dim, ldq, ldk, ldv, ldo, ldo,
      n_kv_heads * head_dim, lddv, d_err, static_cast<cudaStream_t>(stream));
  return kernel_status(e);
}

}  // extern "C"
