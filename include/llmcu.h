/*
 * llmcu.h -- C ABI of the B200-native Qwen3 LoRA training step (libllmcu.so).
 *
 * The reference (visheshnarayan/llm.cu) has no library API: its trainer calls
 * C++-linkage functions whose signatures are re-declared by hand in each file
 * (src/train.cu:27-39, include/lora.h:66-90) and exits on any CUDA error
 * (include/utils.h:10-27).  This header is the drop-in boundary that replaces
 * that call surface.  Each entry point names the reference function(s) it
 * stands in for.
 *
 * Conventions
 *   - Plain C: pointers, sizes, PODs.  No torch or C++ types.
 *   - Every call returns an llmcu_status and never calls exit(); the text of
 *     the last failure on a context is llmcu_last_error(ctx).
 *   - The library owns all device memory.  llmcu_ctx_create() allocates one
 *     arena sized for (max_batch, max_seq); no call made during a training
 *     step allocates device memory.
 *   - One context per device per host thread.  Work runs on context-owned
 *     streams (one compute stream, one communication stream).
 *   - "host" pointers are ordinary CPU memory (pinned or not); "device"
 *     pointers are CUDA device addresses on the context's device.
 *   - Token ids are int32 [batch, seq] row-major; targets are the inputs
 *     shifted by one (src/train.cu:253-258).
 */
#ifndef LLMCU_H
#define LLMCU_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define LLMCU_ABI_VERSION 2

typedef enum {
    LLMCU_OK = 0,
    LLMCU_ERR_INVALID_ARG = 1,   /* bad size, id, pointer or state           */
    LLMCU_ERR_CUDA = 2,          /* a CUDA runtime call failed               */
    LLMCU_ERR_OOM = 3,           /* device arena could not be allocated      */
    LLMCU_ERR_IO = 4,            /* file missing, short read or short write  */
    LLMCU_ERR_NCCL = 5,          /* a NCCL call failed or a peer aborted     */
    LLMCU_ERR_TIMEOUT = 6,       /* a host-side deadline expired             */
    LLMCU_ERR_DEVICE_CHECK = 7,  /* a kernel's own check failed (bounded wait
                                    expired, id out of range); the context
                                    stays usable                             */
    LLMCU_ERR_UNSUPPORTED = 8    /* shape/config this build does not handle */
} llmcu_status;

/* Model dimensions: the runtime form of the reference's compile-time macros
 * (include/config.h:5-21, include/lora.h:6-8). */
typedef struct {
    int32_t hidden;        /* HIDDEN_SIZE            2048  */
    int32_t n_layers;      /* NUM_LAYERS             28    */
    int32_t n_heads;       /* NUM_HEADS              16    */
    int32_t n_kv_heads;    /* NUM_KV_HEADS           8     */
    int32_t head_dim;      /* HEAD_DIM               128 (64 and 128 supported) */
    int32_t ffn;           /* INTERMEDIATE_SIZE      6144  */
    int32_t vocab;         /* VOCAB_SIZE             151936 */
    float   rope_theta;    /* ROPE_THETA             1e6   */
    float   rms_eps;       /* RMS_NORM_EPS           1e-6  */
} llmcu_model_cfg;

typedef struct {
    int32_t rank;          /* LORA_RANK   16 (1..16 supported) */
    float   alpha;         /* LORA_ALPHA  32 -> scale alpha/rank */
    int32_t targets;       /* adapted projections: bit p set = llmcu_proj p has
                              an adapter; 0 = LLMCU_TARGETS_ATTN, the reference's
                              fixed set (include/lora.h:22-27)                 */
} llmcu_lora_cfg;

typedef enum { LLMCU_BASE_FP16 = 0, LLMCU_BASE_INT8 = 1 } llmcu_base_dtype;

typedef struct {
    int32_t max_batch;          /* sequences per step on this device            */
    int32_t max_seq;            /* tokens per sequence                          */
    int32_t base_dtype;         /* llmcu_base_dtype                             */
    int32_t loss_all_positions; /* 0 = reference convention: positions 0..S-2
                                   of each sequence (src/kernels/loss.cu:18-21);
                                   1 = every position                           */
    int32_t int8_in_gemm;       /* INT8 base, MLP weights: 0 = each weight
                                   dequantised to fp16 by one vectorised pass
                                   just before its GEMM (the faster on B200);
                                   1 = the GEMM stages the INT8 codes itself
                                   (converter warps expand them in shared
                                   memory; row scales in the epilogue / folded
                                   into the input-gradient GEMM's A operand)    */
    int32_t lm_head_chunk;      /* vocabulary columns per lm_head chunk (the
                                   lm_head streams over the vocabulary; a
                                   multiple of 256); 0 = as many as fit 128 MiB
                                   of fp16 values at the step's rows           */
    int32_t deterministic;      /* 1 = every sum has a fixed order, so the same
                                   step gives the same bits every time: the
                                   attention backward stores each key tile's dQ
                                   partial in its own slab (+ B * ceil(S/128)^2
                                   * 128 * nh * hd floats of memory) and they
                                   are summed in order; 0 = dQ is reduce-added
                                   by the key tiles in no fixed order (faster).
                                   The adapter gradients' sums are ordered
                                   either way                                   */
} llmcu_run_cfg;

typedef struct {
    float lr, beta1, beta2, eps, weight_decay;   /* src/train.cu:174-183 */
} llmcu_adamw_cfg;

/* Base tensor ids for llmcu_set_base_tensor (file names of
 * src/train.cu:56-89 / python/export_weights.py:19-25). */
typedef enum {
    LLMCU_T_EMBED = 0,       /* model.embed_tokens.weight   [V, H] (lm_head tied) */
    LLMCU_T_FINAL_NORM = 1,  /* model.norm.weight           [H]                   */
    LLMCU_T_ATTN_NORM = 2,   /* layers.l.input_layernorm    [H]                   */
    LLMCU_T_FFN_NORM = 3,    /* layers.l.post_attention_layernorm [H]             */
    LLMCU_T_WQ = 4,          /* self_attn.q_proj   [nh*hd, H]  */
    LLMCU_T_WK = 5,          /* self_attn.k_proj   [nkv*hd, H] */
    LLMCU_T_WV = 6,          /* self_attn.v_proj   [nkv*hd, H] */
    LLMCU_T_WO = 7,          /* self_attn.o_proj   [H, nh*hd]  */
    LLMCU_T_Q_NORM = 8,      /* self_attn.q_norm   [hd]        */
    LLMCU_T_K_NORM = 9,      /* self_attn.k_norm   [hd]        */
    LLMCU_T_W_GATE = 10,     /* mlp.gate_proj      [I, H]      */
    LLMCU_T_W_UP = 11,       /* mlp.up_proj        [I, H]      */
    LLMCU_T_W_DOWN = 12,     /* mlp.down_proj      [H, I]      */
    LLMCU_T_COUNT = 13
} llmcu_tensor_id;

/* LoRA projection ids: q/k/v/o in the order of include/lora.h:22-27, then
 * the MLP projections (gate_proj, up_proj, down_proj), which the reference
 * does not adapt.  Adapter shapes: A [rank, d_in], B [d_out, rank] with
 * (d_out, d_in) = q (nh*hd, H), k / v (nkv*hd, H), o (H, nh*hd),
 * gate / up (I, H), down (H, I). */
typedef enum {
    LLMCU_P_Q = 0, LLMCU_P_K = 1, LLMCU_P_V = 2, LLMCU_P_O = 3,
    LLMCU_P_GATE = 4, LLMCU_P_UP = 5, LLMCU_P_DOWN = 6,
    LLMCU_P_COUNT = 7
} llmcu_proj;
#define LLMCU_TARGETS_ATTN 0x0F   /* q, k, v, o (the reference)      */
#define LLMCU_TARGETS_MLP  0x70   /* gate, up, down                  */
#define LLMCU_TARGETS_ALL  0x7F

typedef struct llmcu_ctx llmcu_ctx;

/* ---------------------------------------------------------------- context */

/* Replaces load-time setup of src/train.cu:217-242 (lora_weights_init,
 * lora_grads_alloc, lora_acts_alloc, alloc_train_ws): validates the config and
 * allocates the whole arena on `device`.  LoRA adapters start as A = 0, B = 0. */
llmcu_status llmcu_ctx_create(const llmcu_model_cfg* model, const llmcu_lora_cfg* lora,
                              const llmcu_run_cfg* run, int device, llmcu_ctx** out);
/* Replaces lora_weights_free / lora_grads_free / lora_acts_free. */
void llmcu_ctx_destroy(llmcu_ctx* ctx);
/* Text of the last failure on ctx (never NULL; "" if none). */
const char* llmcu_last_error(const llmcu_ctx* ctx);
/* Library version string, e.g. "llmcu 1 sm_100a". */
const char* llmcu_version(void);
/* Bytes of device memory the context holds. */
size_t llmcu_device_bytes(const llmcu_ctx* ctx);
/* The compute stream (a cudaStream_t) -- for callers that order their own
 * device work after a step. */
void* llmcu_stream(const llmcu_ctx* ctx);
llmcu_status llmcu_synchronize(llmcu_ctx* ctx);

/* ------------------------------------------------------------ base weights */

/* Replaces load_weight() for one tensor (src/train.cu:42-54): `host` holds
 * fp32 data with the tensor's reference shape; it is converted to the base
 * dtype (fp16, or INT8 + per-row fp32 scales) on the device.  `layer` is
 * ignored for EMBED / FINAL_NORM. */
llmcu_status llmcu_set_base_tensor(llmcu_ctx* ctx, int tensor_id, int layer, const float* host);
/* Replaces load_model() (src/train.cu:56-89): reads the reference's fp32
 * weight files from `dir` (model.embed_tokens.weight.bin, ...); the separate
 * lm_head.weight.bin is not read because the head is tied to the embedding. */
llmcu_status llmcu_load_base_fp32_files(llmcu_ctx* ctx, const char* dir);
/* Synthetic base for benchmarks: every linear ~ N(0, std) drawn on the device
 * from a counter-based generator keyed by `seed`, norm gains 1. */
llmcu_status llmcu_init_base_synthetic(llmcu_ctx* ctx, uint64_t seed, float std);

/* ------------------------------------------------------------------ LoRA */

/* A is [rank, d_in] and B is [d_out, rank], fp32 row-major, host memory --
 * the layout of include/lora.h:13-20 and of the lora_step files.  `proj`
 * must be one of the context's targets (LLMCU_ERR_INVALID_ARG otherwise). */
llmcu_status llmcu_set_lora(llmcu_ctx* ctx, int layer, int proj, const float* A, const float* B);
llmcu_status llmcu_get_lora(llmcu_ctx* ctx, int layer, int proj, float* A, float* B);
/* Gradients of the last llmcu_forward_backward / llmcu_train_step. */
llmcu_status llmcu_get_lora_grads(llmcu_ctx* ctx, int layer, int proj, float* dA, float* dB);
/* Synthetic adapters on the device: A ~ U(+-1/sqrt(d_in)), B ~ N(0, b_std). */
llmcu_status llmcu_init_lora_synthetic(llmcu_ctx* ctx, uint64_t seed, float b_std);
/* Zero the AdamW moments (m, v). */
llmcu_status llmcu_reset_optimizer(llmcu_ctx* ctx);
/* Total LoRA parameter count (A and B of every adapter). */
int64_t llmcu_lora_param_count(const llmcu_ctx* ctx);
/* The context's target mask (llmcu_lora_cfg.targets with 0 resolved). */
int32_t llmcu_lora_targets(const llmcu_ctx* ctx);

/* ------------------------------------------------------------------ steps */

/* One full step: lora_grads_zero + transformer_forward_lora +
 * cross_entropy_forward + transformer_backward_lora + adamw_step_lora
 * (src/train.cu:251-291).  tokens/targets are HOST int32 [batch, seq];
 * *loss_out receives the mean NLL (over all ranks when data parallel).
 *
 * Argument rules of every step entry point: batch in [1, max_batch] and seq
 * in [2, max_seq] of the context's llmcu_run_cfg, else LLMCU_ERR_INVALID_ARG
 * before any work.  Ids are checked on the device: a token outside
 * [0, vocab) embeds as id 0 and a target outside it scores nothing, the step
 * runs to its end, and the call that reads the loss (this one, or
 * llmcu_read_loss after llmcu_train_step_device) returns
 * LLMCU_ERR_INVALID_ARG; the context stays usable. */
llmcu_status llmcu_train_step(llmcu_ctx* ctx, const int32_t* tokens, const int32_t* targets,
                              int batch, int seq, const llmcu_adamw_cfg* opt, int step,
                              float* loss_out);
/* The same step with DEVICE token buffers; the loss stays on the device
 * (read it with llmcu_read_loss).  Nothing is copied to or from the host. */
llmcu_status llmcu_train_step_device(llmcu_ctx* ctx, const int32_t* d_tokens,
                                     const int32_t* d_targets, int batch, int seq,
                                     const llmcu_adamw_cfg* opt, int step);
/* Mean loss of the last step (synchronises the compute stream). */
llmcu_status llmcu_read_loss(llmcu_ctx* ctx, float* loss_out);
/* Forward + loss + backward only (gradients left in place, no optimizer);
 * the split form of the step used by the parity tests.  It stands in for the
 * reference's transformer_forward_lora + cross_entropy_forward +
 * transformer_backward_lora (src/train.cu:262-285) together: there is no
 * forward-only or backward-only entry, because the vocabulary-streamed
 * lm_head forms the logits' gradient in the same pass as the loss. */
llmcu_status llmcu_forward_backward(llmcu_ctx* ctx, const int32_t* tokens, const int32_t* targets,
                                    int batch, int seq, float* loss_out);
/* AdamW over all adapters with the gradients in place (adamw_step_lora,
 * src/kernels/lora.cu:235-246); bias corrections use `step` (1-based). */
llmcu_status llmcu_adamw(llmcu_ctx* ctx, const llmcu_adamw_cfg* opt, int step);

/* --------------------------------------------------------- checkpointing */

/* Replaces save_lora (src/train.cu:146-170): writes
 * dir/lora_step{step}_layer{l}_{wq,wk,wv,wo}_{A,B}.bin, raw fp32, A [r, d_in],
 * B [d_out, r], no header -- the files python/save_lora.py reads.  The MLP
 * targets, when enabled, add ..._{w_gate,w_up,w_down}_{A,B}.bin the same way
 * (names of the base weights they adapt). */
llmcu_status llmcu_save_lora(llmcu_ctx* ctx, const char* dir, int step);
/* Reads the same files back (e.g. those written by save_lora.py --from-hf). */
llmcu_status llmcu_load_lora(llmcu_ctx* ctx, const char* dir, int step);

/* The same adapter files on the host alone, no device or context needed (the
 * file side of llmcu_save_lora / llmcu_load_lora, which call the same code
 * after / before their device copy): for converters and checkpoint tools that
 * run where there is no GPU.  `flat` is the library's adapter layout: per
 * layer, for each target projection in llmcu_proj order, A [rank, d_in] then
 * B [d_out, rank], fp32 -- llmcu_lora_layout_count floats in all (0 for an
 * invalid layout).  Same file names and contents as save_lora
 * (src/train.cu:146-170); LLMCU_ERR_IO for a missing, short or unwritable
 * file, LLMCU_ERR_INVALID_ARG for a null pointer or invalid layout. */
typedef struct {
    int32_t n_layers, hidden, q_dim, kv_dim, ffn;
    int32_t rank;     /* 1..16 */
    int32_t targets;  /* as llmcu_lora_cfg.targets (0 = q, k, v, o) */
} llmcu_lora_layout;
int64_t llmcu_lora_layout_count(const llmcu_lora_layout* layout);
llmcu_status llmcu_lora_files_write(const llmcu_lora_layout* layout, const float* flat, const char* dir, int step);
llmcu_status llmcu_lora_files_read(const llmcu_lora_layout* layout, float* flat, const char* dir, int step);

/* Greedy generation with a KV cache (llm_engine --generate, src/main.cu:340-385,
 * on the training context's weights and current adapters): the prompt (one
 * sequence of n_prompt host ids) runs through the batched forward and fills the
 * cache, then n_new tokens are chosen by argmax (the lowest id on ties).  The
 * decode steps replay one CUDA graph per token.  n_prompt + n_new <= max_seq.
 * out_tokens[n_new] receives every chosen id; *n_out (nullable) the count
 * before Qwen3's end ids 151643 / 151645 (as llm_engine stops there; n_new
 * when the vocabulary has no such ids).  step_logits (nullable, host
 * [n_new, vocab] fp32): the logits each token was chosen from (then the steps
 * run without the graph).  decode_ms (nullable): device time per decoded token
 * after the first. */
llmcu_status llmcu_generate(llmcu_ctx* ctx, const int32_t* prompt, int n_prompt, int n_new,
                            int32_t* out_tokens, int* n_out, float* step_logits, float* decode_ms);

/* Optimizer sidecar for resuming (no reference counterpart: the reference
 * saves A / B only, src/train.cu:146-170): dir/lora_step{step}_adamw.bin holds
 * a 64-byte header ("LLMCUADW", version 1, step, layers, rank, hidden, q and
 * kv dims, parameter count) and the AdamW first and second moments, fp32, in
 * the flat adapter layout.  Together with llmcu_save_lora's A / B files of the
 * same step, llmcu_load_lora + llmcu_load_adamw_state restore the training
 * state; the next llmcu_train_step then takes step + 1.  Loading checks every
 * header field against the context (LLMCU_ERR_INVALID_ARG on a mismatch). */
llmcu_status llmcu_save_adamw_state(llmcu_ctx* ctx, const char* dir, int step);
llmcu_status llmcu_load_adamw_state(llmcu_ctx* ctx, const char* dir, int step);

/* --------------------------------------------------------------- INT8 */

/* Per-row symmetric quantiser, bit-exact with quantize_kernel
 * (src/kernels/quantize.cu:8-50): scale = absmax/127, q = rint(clamp(w/scale)).
 * DEVICE pointers: w fp32 [rows, cols], q int8 [rows, cols], scale fp32 [rows];
 * `stream` is a cudaStream_t (NULL = legacy default stream). */
llmcu_status llmcu_quantize_int8_rows(const float* w, int rows, int cols, int8_t* q,
                                      float* scale, void* stream);

/* -------------------------------------------------------- data parallel */

/* NCCL unique id of 128 bytes for rank 0 to broadcast out of band. */
llmcu_status llmcu_dp_get_unique_id(void* id128);
/* Joins a data-parallel group of `world` ranks (one per GPU).  After this
 * call every step allreduces the LoRA gradients (sum, fp32) per layer on the
 * communication stream, overlapped with the rest of the backward pass, and
 * the loss is averaged over ranks.  The reference is single-GPU only. */
llmcu_status llmcu_dp_init(llmcu_ctx* ctx, const void* id128, int rank, int world);
/* Host deadline for each NCCL wait; on expiry the communicator is aborted and
 * LLMCU_ERR_TIMEOUT is returned (default 60000 ms). */
llmcu_status llmcu_dp_set_timeout_ms(llmcu_ctx* ctx, int ms);

/* ------------------------------------------------------------- profiling */

/* Per-kernel-class timing.  While enabled, every step records CUDA events on
 * the compute stream around each kernel launch (classes: gemm_tc,
 * attention_fwd, attention_bwd, norm_rope, lora_grad, lora_merge, lm_head
 * (the vocabulary-streamed logits, cross-entropy and d_xf: its GEMMs are not
 * in gemm_tc), embed, adamw, int8_dequant, fill_and_loss) and, data parallel,
 * around the
 * compute stream's wait for the allreduces the backward did not hide
 * (dp_exposed, no kernel); the adapter gradients then run on the compute
 * stream.  The reference has no counterpart (its
 * per-component timers exist only in the inference bench,
 * src/kernels/forward.cu:207-335). */
llmcu_status llmcu_profile_enable(llmcu_ctx* ctx, int on);
/* Writes {"class": {"ms": total, "launches": n}, ...} accumulated since the
 * last reset into buf (NUL-terminated); reset != 0 clears the totals. */
llmcu_status llmcu_profile_read(llmcu_ctx* ctx, char* buf, size_t len, int reset);

/* ------------------------------------------------------------ kernel test
 * Single-kernel entry points on DEVICE pointers, used by the kernel-level
 * parity tests.  `stream` is a cudaStream_t; results are asynchronous.  The
 * returned status covers the launch: LLMCU_ERR_INVALID_ARG for a null pointer
 * or a non-positive size, LLMCU_ERR_UNSUPPORTED for a base address or row
 * stride the TMA descriptors refuse (they need 16-byte alignment) or an
 * unsupported head_dim, LLMCU_ERR_CUDA for a failed launch.  What the kernels
 * find while they run (a bounded wait that gave up, leaving a partial result)
 * is reported afterwards by llmcu_kernel_checks. */

/* Device-side checks of the kernel-level entry points below: their kernels OR
 * an error bit into one word per device, held by the library, when a bounded
 * wait gives up (and then leave their outputs partly written).  This call
 * synchronises `stream`, reads the current device's word, clears it, and
 * returns LLMCU_ERR_DEVICE_CHECK if any bit was set since the last call
 * (LLMCU_OK otherwise); *bits (nullable) receives the raw bits.  No reference
 * counterpart: the reference's kernels have no device-side checks. */
llmcu_status llmcu_kernel_checks(void* stream, int* bits);

/* Failure-path self-test: launches one CTA on `stream` whose single wait is
 * never satisfied, so it gives up after the kernels' bounded-wait limit
 * (4 s), raises its abort flag and sets the same error bit a stalled pipeline
 * would; llmcu_kernel_checks then returns LLMCU_ERR_DEVICE_CHECK, and the
 * device stays usable.  Nothing faults, traps or hangs.  No reference
 * counterpart. */
llmcu_status llmcu_kernel_wait_selftest(void* stream);

/* C[M,N] (fp32) = A[M,K] . B[N,K]^T, fp16 inputs, K-major rows with leading
 * dims lda/ldb/ldc in elements -- the NT product of matmul_kernel
 * (src/kernels/matmul.cu:8-51) on the tcgen05 path. */
llmcu_status llmcu_gemm_nt_f16(const void* A, const void* B, float* C, int M, int N, int K,
                               int lda, int ldb, int ldc, void* stream);
/* C[M,N] (fp32) = A[M,K] . B[K,N], B row-major [K, N] (ldb elements between
 * rows) -- the NN product of matmul_nn_forward (src/kernels/matmul.cu:55-98),
 * the input-gradient GEMMs' form (B read MN-major, no transposed copy). */
llmcu_status llmcu_gemm_nn_f16(const void* A, const void* B, float* C, int M, int N, int K,
                               int lda, int ldb, int ldc, void* stream);
/* Causal GQA attention forward: q [B*S, nh*hd], k/v [B*S, nkv*hd] fp16 with
 * row strides ldq/ldk/ldv; o [B*S, nh*hd] fp16, lse [B, nh, S] fp32
 * (replaces naive_attn_kernel, src/kernels/lora_forward.cu:48-135). */
llmcu_status llmcu_attention_fwd(const void* q, const void* k, const void* v, void* o, float* lse,
                                 int batch, int seq, int n_heads, int n_kv_heads, int head_dim,
                                 int ldq, int ldk, int ldv, void* stream);
/* Its backward (replaces attn_backward_kernel + expand/contract,
 * src/kernels/lora_backward.cu:104-208): dq [B*S, nh*hd] fp32, dk [B*S,
 * nkv*hd] fp32, dv written fp16 with row stride lddv.  `scratch_delta` is
 * fp32 [B, nh, S]. */
llmcu_status llmcu_attention_bwd(const void* q, const void* k, const void* v, const void* o,
                                 const void* dout, const float* lse, float* scratch_delta,
                                 float* dq, float* dk, void* dv, int batch, int seq,
                                 int n_heads, int n_kv_heads, int head_dim, int ldq, int ldk,
                                 int ldv, int lddv, void* stream);

/* The attention backward above with no scratch argument and no allocation.
 * No counterpart in the reference (its backward cudaMallocs and frees
 * temporaries on every call, src/kernels/lora_backward.cu:330-346).
 * For callers that must not allocate device memory themselves: code running
 * under a caching allocator that owns the device's memory (a cudaMalloc beside
 * it fragments memory and escapes its accounting), or a latency-critical loop
 * where cudaMalloc's implicit device synchronisation would stall other streams.
 * The row sums it needs live in a 4 MiB array inside this library, which every
 * GPU that loads the library holds until the process exits:
 *   - batch * n_heads * seq must be <= 1,048,576, else LLMCU_ERR_UNSUPPORTED
 *     and nothing is launched;
 *   - all calls share the one array: calls that overlap on the GPU (different
 *     streams, or several host threads) race and give wrong results; calls on
 *     one stream are ordered and safe.  Every entry the kernels read is written
 *     earlier in the same call, so stale contents from a previous call are
 *     never used;
 *   - each call looks up the current device's copy of the array (so make the
 *     call with the intended device current);
 *   - a bounded wait that gives up inside the kernels is reported, as for the
 *     other kernel-level entry points, by llmcu_kernel_checks.
 * Same arguments, layouts, statuses and results as llmcu_attention_bwd
 * otherwise. */
llmcu_status llmcu_attention_bwd_noalloc(const void* q, const void* k, const void* v, const void* o,
                                         const void* dout, const float* lse, float* dq, float* dk, void* dv,
                                         int batch, int seq, int n_heads, int n_kv_heads, int head_dim,
                                         int ldq, int ldk, int ldv, int lddv, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* LLMCU_H */
