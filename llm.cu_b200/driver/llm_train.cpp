// llm_train -- C++ host driver of the LoRA training step on libllmcu.so.
//
// Keeps the reference trainer's command line (src/train.cu:184-190):
//   --lr 3e-4 --steps 1000 --seq-len 512 --save-every 100 --log-every 10
// its data file (data/train_tokens.bin: int32 count, int32 ids;
// src/train.cu:195-214), its fp32 weight files (weights/<hf name>.bin,
// src/train.cu:56-89) and its adapter output files
// (weights/lora_step{N}_layer{l}_{wq,wk,wv,wo}_{A,B}.bin, src/train.cu:146-170),
// which python/save_lora.py reads unchanged.  The log line keeps the
// reference's "step %4d  loss %.4f  (avg %.4f)" and appends throughput.
//
// Additions: --batch B (sequences per step and GPU), --config tiny|1.7b,
// --synthetic (device-generated N(0,0.02) base and adapters, uniform tokens),
// --int8 (INT8 per-row base), --weights DIR, --data FILE, --out DIR, --seed,
// --resume N (continue after step N from the adapter and AdamW files in --out;
// every save also writes the AdamW sidecar lora_step{N}_adamw.bin),
// --rank R / --alpha A (LoRA rank 1..16 and alpha; default the config's),
// --lora-targets LIST (comma-separated wq,wk,wv,wo,w_gate,w_up,w_down, or
// "attn" = the reference's q/k/v/o, "mlp", "all"; default attn),
// --int8-in-gemm (with --int8: the GEMMs stage the INT8 codes themselves).
// Data parallel: when WORLD_SIZE > 1 (e.g. under torchrun) each process
// drives GPU LOCAL_RANK, rank 0 writes the NCCL id to --dp-id-file and the
// others read it; rank r takes sequences r, r+W, ... of every step window.
#include <unistd.h>

#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <random>
#include <string>
#include <thread>
#include <vector>

#include "llmcu.h"

namespace {

int env_int(const char* k, int d) {
  const char* v = getenv(k);
  return v ? atoi(v) : d;
}

void die(llmcu_ctx* ctx, llmcu_status s, const char* what) {
  fprintf(stderr, "ERROR: %s failed (status %d): %s\n", what, static_cast<int>(s),
          ctx ? llmcu_last_error(ctx) : "");
  exit(1);
}

}  // namespace

int main(int argc, char** argv) {
  float lr = 3e-4f;
  int steps = 1000, seq_len = 512, save_every = 100, log_every = 10, batch = 1, resume = 0;
  const float beta1 = 0.9f, beta2 = 0.999f, eps_adam = 1e-8f, wd = 0.01f;
  std::string config = "1.7b", weights = "weights", data = "data/train_tokens.bin", out = "weights";
  std::string id_file = "/tmp/llmcu_nccl_id";
  bool synthetic = false, int8 = false, int8_in_gemm = false;
  unsigned long long seed = 1234;
  int lora_rank = 0;
  float lora_alpha = 0.f;
  std::string targets_arg = "attn";

  for (int i = 1; i < argc; i++) {
    auto next = [&](const char* flag) -> const char* {
      if (!strcmp(argv[i], flag) && i + 1 < argc) return argv[++i];
      return nullptr;
    };
    const char* v;
    if ((v = next("--lr"))) lr = static_cast<float>(atof(v));
    else if ((v = next("--steps"))) steps = atoi(v);
    else if ((v = next("--seq-len"))) seq_len = atoi(v);
    else if ((v = next("--save-every"))) save_every = atoi(v);
    else if ((v = next("--log-every"))) log_every = atoi(v);
    else if ((v = next("--batch"))) batch = atoi(v);
    else if ((v = next("--config"))) config = v;
    else if ((v = next("--weights"))) weights = v;
    else if ((v = next("--data"))) data = v;
    else if ((v = next("--out"))) out = v;
    else if ((v = next("--seed"))) seed = strtoull(v, nullptr, 10);
    else if ((v = next("--dp-id-file"))) id_file = v;
    else if ((v = next("--resume"))) resume = atoi(v);
    else if ((v = next("--rank"))) lora_rank = atoi(v);
    else if ((v = next("--alpha"))) lora_alpha = static_cast<float>(atof(v));
    else if ((v = next("--lora-targets"))) targets_arg = v;
    else if (!strcmp(argv[i], "--synthetic")) synthetic = true;
    else if (!strcmp(argv[i], "--int8")) int8 = true;
    else if (!strcmp(argv[i], "--int8-in-gemm")) int8_in_gemm = true;
    else if (!strcmp(argv[i], "--help") || !strcmp(argv[i], "-h")) {
      printf("usage: llm_train [--lr F] [--steps N] [--seq-len S] [--save-every N] [--log-every N]\n"
             "                 [--batch B] [--config tiny|1.7b] [--synthetic] [--int8] [--weights DIR]\n"
             "                 [--data FILE] [--out DIR] [--seed N] [--dp-id-file PATH] [--resume N]\n"
             "                 [--rank R] [--alpha A] [--lora-targets attn|mlp|all|wq,wk,...,w_down]\n"
             "                 [--int8-in-gemm]\n");
      return 0;
    }
  }
  if (log_every < 1) log_every = 1;
  if (save_every < 1) save_every = steps;

  const int world = env_int("WORLD_SIZE", 1), rank = env_int("RANK", 0), local = env_int("LOCAL_RANK", 0);

  llmcu_model_cfg mc;
  llmcu_lora_cfg lc;
  if (config == "tiny") {
    mc = {256, 2, 4, 2, 64, 768, 4096, 1.0e6f, 1.0e-6f};
    lc = {4, 8.0f, LLMCU_TARGETS_ATTN};
  } else {
    mc = {2048, 28, 16, 8, 128, 6144, 151936, 1.0e6f, 1.0e-6f};
    lc = {16, 32.0f, LLMCU_TARGETS_ATTN};
  }
  if (lora_rank > 0) lc.rank = lora_rank;
  if (lora_alpha > 0.f) lc.alpha = lora_alpha;
  {
    static const char* kNames[LLMCU_P_COUNT] = {"wq", "wk", "wv", "wo", "w_gate", "w_up", "w_down"};
    int mask = 0;
    if (targets_arg == "attn") mask = LLMCU_TARGETS_ATTN;
    else if (targets_arg == "mlp") mask = LLMCU_TARGETS_MLP;
    else if (targets_arg == "all") mask = LLMCU_TARGETS_ALL;
    else {
      size_t pos = 0;
      while (pos <= targets_arg.size()) {
        const size_t comma = targets_arg.find(',', pos);
        const std::string name = targets_arg.substr(pos, comma == std::string::npos ? std::string::npos : comma - pos);
        int p = 0;
        while (p < LLMCU_P_COUNT && name != kNames[p]) ++p;
        if (p == LLMCU_P_COUNT) {
          fprintf(stderr, "ERROR: unknown --lora-targets entry '%s'\n", name.c_str());
          return 1;
        }
        mask |= 1 << p;
        if (comma == std::string::npos) break;
        pos = comma + 1;
      }
    }
    lc.targets = mask;
  }
  llmcu_run_cfg rc = {batch, seq_len, int8 ? LLMCU_BASE_INT8 : LLMCU_BASE_FP16, 0, int8_in_gemm ? 1 : 0, 0, 0};
  if (rank == 0)
    printf("Training config: lr=%.2e steps=%d seq_len=%d batch=%d world=%d model=%s base=%s lora rank=%d "
           "alpha=%g targets=0x%x\n",
           lr, steps, seq_len, batch, world, config.c_str(), int8 ? "int8" : "fp16", lc.rank, lc.alpha, lc.targets);

  // training data (src/train.cu:195-214): int32 count + ids
  std::vector<int32_t> train;
  if (!synthetic) {
    FILE* f = fopen(data.c_str(), "rb");
    if (!f) {
      fprintf(stderr, "ERROR: %s not found. Tokenize training data first:\n"
              "  python python/tokenize_input.py --train <text_file>\n", data.c_str());
      return 1;
    }
    int32_t n = 0;
    if (fread(&n, sizeof(int32_t), 1, f) != 1 || n <= 0) {
      fprintf(stderr, "ERROR: bad header in %s\n", data.c_str());
      fclose(f);
      return 1;
    }
    train.resize(n);
    const size_t got = fread(train.data(), sizeof(int32_t), n, f);
    fclose(f);
    if (got != static_cast<size_t>(n)) {
      fprintf(stderr, "ERROR: short read %s\n", data.c_str());
      return 1;
    }
    if (rank == 0) printf("Loaded %d training tokens\n", n);
  }
  const int num_seqs = synthetic ? 1 << 30 : static_cast<int>(train.size() / (seq_len + 1));
  if (num_seqs == 0) {
    fprintf(stderr, "ERROR: need at least %d tokens, got %zu\n", seq_len + 1, train.size());
    return 1;
  }

  llmcu_ctx* ctx = nullptr;
  llmcu_status s = llmcu_ctx_create(&mc, &lc, &rc, local, &ctx);
  if (s != LLMCU_OK) die(ctx, s, "llmcu_ctx_create");

  if (world > 1) {
    unsigned char id[128];
    if (rank == 0) {
      if ((s = llmcu_dp_get_unique_id(id)) != LLMCU_OK) die(ctx, s, "llmcu_dp_get_unique_id");
      const std::string tmp = id_file + ".tmp";
      FILE* f = fopen(tmp.c_str(), "wb");
      if (!f || fwrite(id, 1, 128, f) != 128) die(ctx, LLMCU_ERR_IO, "writing NCCL id");
      fclose(f);
      rename(tmp.c_str(), id_file.c_str());
    } else {
      bool ok = false;
      for (int t = 0; t < 6000 && !ok; ++t) {
        FILE* f = fopen(id_file.c_str(), "rb");
        if (f) {
          ok = fread(id, 1, 128, f) == 128;
          fclose(f);
        }
        if (!ok) std::this_thread::sleep_for(std::chrono::milliseconds(10));
      }
      if (!ok) die(ctx, LLMCU_ERR_TIMEOUT, "reading NCCL id file");
    }
    if ((s = llmcu_dp_init(ctx, id, rank, world)) != LLMCU_OK) die(ctx, s, "llmcu_dp_init");
  }

  if (synthetic) {
    if ((s = llmcu_init_base_synthetic(ctx, seed, 0.02f)) != LLMCU_OK) die(ctx, s, "llmcu_init_base_synthetic");
  } else {
    if ((s = llmcu_load_base_fp32_files(ctx, weights.c_str())) != LLMCU_OK) die(ctx, s, "llmcu_load_base_fp32_files");
  }
  // adapters as BASELINE configs: A ~ U(+-1/sqrt(in)), B ~ N(0, 0.01); identical on every rank
  if ((s = llmcu_init_lora_synthetic(ctx, seed + 1, 0.01f)) != LLMCU_OK) die(ctx, s, "llmcu_init_lora_synthetic");
  if (resume > 0) {  // adapters and AdamW moments of step `resume` from --out; continue at resume + 1
    if ((s = llmcu_load_lora(ctx, out.c_str(), resume)) != LLMCU_OK) die(ctx, s, "llmcu_load_lora");
    if ((s = llmcu_load_adamw_state(ctx, out.c_str(), resume)) != LLMCU_OK) die(ctx, s, "llmcu_load_adamw_state");
    if (rank == 0) printf("Resumed from step %d (%s)\n", resume, out.c_str());
  }
  if (rank == 0)
    printf("LoRA adapters initialized (rank=%d, alpha=%.0f, scale=%.1f, %lld params)\n", lc.rank, lc.alpha,
           lc.alpha / lc.rank, static_cast<long long>(llmcu_lora_param_count(ctx)));

  const int M = batch * seq_len;
  std::vector<int32_t> tok(M), tgt(M);
  std::mt19937_64 rng(seed * 31 + rank);
  // the synthetic stream draws seq_len + 1 ids per sequence: skip the steps already taken
  if (synthetic && resume > 0) rng.discard(static_cast<unsigned long long>(resume) * batch * (seq_len + 1));
  const llmcu_adamw_cfg opt = {lr, beta1, beta2, eps_adam, wd};
  if (rank == 0) printf("\n=== Training ===\n");
  float running = 0.f;
  int count = 0;
  auto t_log = std::chrono::steady_clock::now();
  for (int step = resume + 1; step <= steps; ++step) {
    for (int b = 0; b < batch; ++b) {
      if (synthetic) {
        for (int i = 0; i < seq_len; ++i) {
          tok[b * seq_len + i] = static_cast<int32_t>(rng() % static_cast<uint64_t>(mc.vocab));
          if (i > 0) tgt[b * seq_len + i - 1] = tok[b * seq_len + i];
        }
        tgt[b * seq_len + seq_len - 1] = static_cast<int32_t>(rng() % static_cast<uint64_t>(mc.vocab));
      } else {
        // deterministic non-overlapping windows (src/train.cu:251-258), sharded over ranks
        const long long w = (static_cast<long long>(step - 1) * batch * world + static_cast<long long>(b) * world + rank) %
                            num_seqs;
        const int32_t* start = train.data() + w * (seq_len + 1);
        memcpy(&tok[b * seq_len], start, sizeof(int32_t) * seq_len);
        memcpy(&tgt[b * seq_len], start + 1, sizeof(int32_t) * seq_len);
      }
    }
    float loss = 0.f;
    if ((s = llmcu_train_step(ctx, tok.data(), tgt.data(), batch, seq_len, &opt, step, &loss)) != LLMCU_OK)
      die(ctx, s, "llmcu_train_step");
    running += loss;
    ++count;
    if (step % log_every == 0 && rank == 0) {
      const auto now = std::chrono::steady_clock::now();
      const double sec = std::chrono::duration<double>(now - t_log).count();
      t_log = now;
      const double tps = static_cast<double>(count) * M * world / sec;
      printf("step %4d  loss %.4f  (avg %.4f)  tok/s %.0f  ms/step %.2f\n", step, loss, running / count, tps,
             1000.0 * sec / count);
      fflush(stdout);
      running = 0.f;
      count = 0;
    }
    if (step % save_every == 0 && rank == 0) {
      if ((s = llmcu_save_lora(ctx, out.c_str(), step)) != LLMCU_OK) die(ctx, s, "llmcu_save_lora");
      if ((s = llmcu_save_adamw_state(ctx, out.c_str(), step)) != LLMCU_OK) die(ctx, s, "llmcu_save_adamw_state");
      printf("Saved LoRA weights at step %d\n", step);
    }
  }
  if (rank == 0) {
    if ((s = llmcu_save_lora(ctx, out.c_str(), steps)) != LLMCU_OK) die(ctx, s, "llmcu_save_lora");
    if ((s = llmcu_save_adamw_state(ctx, out.c_str(), steps)) != LLMCU_OK) die(ctx, s, "llmcu_save_adamw_state");
    printf("Saved LoRA weights at step %d\n\nTraining complete.\n", steps);
  }
  llmcu_ctx_destroy(ctx);
  return 0;
}
