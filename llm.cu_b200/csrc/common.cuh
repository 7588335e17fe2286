// common.cuh -- declarations shared by the kernel translation units.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>

#include "sm100.cuh"

namespace llmcu {

// Runs `set` (cudaFuncSetAttribute calls for one kernel) once on each device
// the process launches that kernel on: function attributes apply per device,
// so a process-wide flag would leave a second device without them.  `mask`
// holds one bit per device ordinal (devices past 63 run `set` every time).
template <class F>
inline cudaError_t once_per_device(std::atomic<unsigned long long>& mask, F&& set) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return set();
  const unsigned long long bit = 1ull << dev;
  if (mask.load(std::memory_order_acquire) & bit) return cudaSuccess;
  e = set();  // two threads may both get here; setting an attribute twice is harmless
  if (e == cudaSuccess) mask.fetch_or(bit, std::memory_order_acq_rel);
  return e;
}

// Device error word of the kernel-level entry points (llmcu_gemm_*,
// llmcu_attention_*): one int per device, held by the library, into which
// their kernels OR the DeviceErr bits of bounded waits that gave up.  The
// address belongs to the current device and is looked up on every call.
cudaError_t kernel_err_word(int** out);

// Programmatic dependent launch for the calling host thread: on while a
// training step issues its chain of kernels (each awaits its predecessor in
// pdl_wait), off otherwise, so a kernel that follows a copy, a memset, an
// event wait or another library's work is launched normally.
bool pdl_enabled();
void set_pdl(bool on);

// Launch `kern`, with programmatic stream serialization when pdl_enabled().
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}


// ---- attention.cu
cudaError_t attention_forward(const __half* q, const __half* k, const __half* v, __half* o, float* lse, int B, int S,
                              int nh, int nkv, int hd, int ldq, int ldk, int ldv, int ldo, int* err, cudaStream_t st);
// ---- attention_tc.cu
cudaError_t attention_forward_tc(const __half* q, const __half* k, const __half* v, __half* o, float* lse, int B,
                                 int S, int nh, int nkv, int hd, int ldq, int ldk, int ldv, int ldo, int* err,
                                 cudaStream_t st);
// dO.O row sums into `delta`, then attention_backward_tc (dq is overwritten).
cudaError_t attention_backward(const __half* q, const __half* k, const __half* v, const __half* o,
                               const __half* dout, const float* lse, float* delta, float* dq, float* dk, __half* dv,
                               int B, int S, int nh, int nkv, int hd, int ldq, int ldk, int ldv, int ldo, int lddq,
                               int lddk, int lddv, int* err, cudaStream_t st);
// dq accumulates with reduce-adds: it is zeroed first unless the caller
// already did (dq_zeroed).  With dq_slabs (deterministic mode) dq is not
// touched: key tile kt stores its partial into slab kt of dq_slabs
// [nqt][B * nqt * 128][nh * hd] fp32 (nqt = ceil(S / 128), each sequence's
// rows padded to whole tiles), for qknorm_rope_backward to sum in order.
cudaError_t attention_backward_tc(const __half* q, const __half* k, const __half* v, const __half* dout,
                                  const float* lse, const float* delta, float* dq, float* dk, __half* dv, int B, int S,
                                  int nh, int nkv, int hd, int ldq, int ldk, int ldv, int ldo, int lddq, int lddk,
                                  int lddv, int* err, cudaStream_t st, bool dq_zeroed = false,
                                  float* dq_slabs = nullptr);

// ---- gemm.cu
// Column slices per GEMM tile (epilogue warps per TMEM lane quadrant); the
// lm_head epilogue writes one (reference, sum) partial per 128-column slice.
constexpr int kGemmEpiGroups = 2;
// Tensor operand for the GEMM: fp16, K-major rows (K contiguous), `ld`
// elements between rows; `rows` x `k` valid extent.
// Tensor operand for the GEMM, fp16.  K-major (mn == false): `rows` rows of
// `k` contiguous elements, `ld` elements between rows.  MN-major (mn == true,
// B only): the [k, rows] matrix stored row-major -- k rows of `rows`
// contiguous elements -- e.g. a weight [out, in] used as B of dY . W.
struct Operand {
  const __half* ptr;
  int rows;
  int k;
  int ld;
  bool mn = false;
  // B only: INT8 codes instead of fp16 (ptr unused), the same [rows, k] /
  // [k, rows] layout with ld bytes between rows; the GEMM stages them as exact
  // fp16.  K-major (x W^T): q8_scale holds the weight's per-row scales, which
  // the epilogue applies to the output columns.  MN-major (dY W): the scales
  // run along K, so the caller folds them into A (q8_scale unused).
  const int8_t* q8 = nullptr;
  const float* q8_scale = nullptr;
};

enum class Epi : int {
  kStoreF16 = 0,
  kStoreF32 = 1,
  kResidF32 = 2,
  kSwiGLU = 3,
  kSwiGLUBwd = 4,
  kStoreF16Delta = 6,  // fp16 dO + the attention backward's per-(row, head) dO.O sums
  kQKNormRope = 7,     // fp16 q/k/v + (head_dim 128) per-head RMSNorm and RoPE of q and k into rope_out
  kCEStream = 8,       // lm_head forward over one vocabulary chunk: exp(l - ref) into the chunk buffer + partials
};

struct EpiArgs {
  // generic outputs
  void* out = nullptr;
  int ld_out = 0;
  int accumulate = 0;
  int ksplit = 1;  // kStoreF32 with accumulate: K slices that reduce-add into the same output
  // kStoreF16Delta: O [M, n_main] (row stride ld_o) and the delta output [B, n_heads, seq]
  const __half* attn_o = nullptr;
  int ld_o = 0;
  float* delta = nullptr;
  int seq = 0, n_heads = 0, head_dim = 0;
  // side output (kStoreF16, kStoreF16Delta, kResidF32): columns [n_main, N) as fp16 [M, N - n_main]
  int n_main = 0;  // 0: no side output
  __half* side = nullptr;
  int ld_side = 0;
  const float* resid = nullptr;
  // SwiGLU
  __half* gu = nullptr;       // interleaved [M, 2I]
  const __half* gu_in = nullptr;
  int ld_gu = 0;
  const float* gu_out_scale = nullptr;  // kSwiGLUBwd: per dgu column factors (null: none)
  __half* act = nullptr;      // [M, I]
  int ld_act = 0;
  // kQKNormRope: q heads are columns [0, n_q_cols), k heads [n_q_cols,
  // n_qk_cols); their normed, rotated copies go to rope_out (same columns,
  // row stride ld_rope); cos/sin tables [seq, 64]
  __half* rope_out = nullptr;
  int ld_rope = 0;
  const float* q_norm_w = nullptr;
  const float* k_norm_w = nullptr;
  const float* rope_cos = nullptr;
  const float* rope_sin = nullptr;
  int n_q_cols = 0, n_qk_cols = 0;
  float eps = 0.f;
  // cross-entropy
  const int* targets = nullptr;
  float* part_max = nullptr;   // kCEStream: the reference of each (row, 128-column slot)
  float* part_sum = nullptr;
  float* tgt_logit = nullptr;
  // kCEStream: per-row reference ce_ref [M], vocabulary index of the chunk's
  // first column (a multiple of 128) and slots per row in part_max / part_sum
  const float* ce_ref = nullptr;
  int vocab_off = 0;
  int ce_slots = 0;
};

// C[M,N] = A . B^T (B K-major) or A . B (B MN-major) with the given
// epilogue.  A.rows = M, B.rows = N, A.k == B.k == K.
cudaError_t gemm(const Operand& A, const Operand& B, int M, int N, Epi epi, const EpiArgs& ea, int* err,
                 cudaStream_t st, int bn_hint = 0);
int gemm_num_sms();
// Split-K fix-up workspace for the calling thread's gemm() calls (null: off):
// ws_floats fp32 partials and cnt_n counters that must be zero (the GEMMs
// leave them zero).  GEMMs whose tiles fill under half a wave then run as K
// splits whose last arrival per tile finishes it.
void set_gemm_workspace(float* ws, size_t ws_floats, int* cnt, int cnt_n);
// fp16 [rows, cols] row-major (row stride ld elements), 128-byte swizzle,
// box 64 columns x box_rows rows.
bool encode_tma_2d_f16(CUtensorMap* map, const void* ptr, int rows, int cols, int ld, int box_rows);

// ---- decode.cu (single-sequence KV-cache decoding; the position is read from
// counters[0] on the device so a decode step can be replayed as a CUDA graph)
int decode_attn_splits(int max_ctx);
// x: xmode 0 = fp16 [K]; 1 = fp32 row [K] RMSNorm'd with `gain` / eps on the
// way in; 2 = fp16 gate/up row [2K] (128-row interleave), SwiGLU on the way in
cudaError_t decode_gemv(const void* W, const float* scale, bool int8, int ldw, const void* x, int xmode,
                        const float* gain, float eps, int N, int K, const float* resid, float* out32, __half* out16,
                        cudaStream_t st);
// raw q/k/v row -> QK-norm + RoPE, cache append at *d_pos, attention over
// rows [0, *d_pos], fp16 output [nh, hd]; part: nh * decode_attn_splits(max_ctx)
// * (hd + 2) floats; tickets: nh ints, zero between calls
cudaError_t decode_attention(const __half* qkv, const float* qn_w, const float* kn_w, const float* cos_t,
                             const float* sin_t, const int* d_pos, __half* k_cache, __half* v_cache, float* part,
                             int* tickets, __half* out, int nh, int nkv, int hd, float eps, int max_ctx,
                             cudaStream_t st);
// counters: [0] position of the next input token, [1] tokens chosen so far, [2] the next input token,
// [3] the argmax blocks' ticket (0 between steps); scratch: decode_argmax_scratch() floats
int decode_argmax_scratch();
cudaError_t decode_argmax(const float* logits, int V, int* counters, int* tokens, float* step_logits, float* scratch,
                          cudaStream_t st);

// ---- kernels.cu
cudaError_t embed_forward(const int* tokens, const __half* E, float* out, int M, int H, int V, int* err,
                          cudaStream_t st);
cudaError_t rmsnorm_forward(const float* x, const float* w, __half* out, int M, int H, float eps, cudaStream_t st);
// dres (+)= rmsnorm_bwd(dy, x, w); dres16 = fp16(dres)
// s16 (optional): per-column factors applied to the fp16 copy dres16 only.
cudaError_t rmsnorm_backward(const float* dy, const float* x, const float* w, float* dres, __half* dres16, int M,
                             int H, float eps, int accumulate, cudaStream_t st, const float* s16 = nullptr);
cudaError_t rmsnorm_backward(const __half* dy, const float* x, const float* w, float* dres, __half* dres16, int M,
                             int H, float eps, int accumulate, cudaStream_t st, const float* s16 = nullptr);
cudaError_t qknorm_rope_forward(const __half* qkv, int ld_qkv, const float* qn_w, const float* kn_w, int ld_out,
                                const float* cos_t, const float* sin_t, __half* q_out, __half* k_out, int B, int S,
                                int nh, int nkv, int hd, float eps, cudaStream_t st);
// dq_slabs (deterministic mode): dq is read as the sum, in key-tile order, of
// the attention backward's per-key-tile slabs (see attention_backward_tc).
cudaError_t qknorm_rope_backward(const float* dq, const float* dk, const __half* qkv, int ld_qkv, const float* qn_w,
                                 const float* kn_w, const float* cos_t, const float* sin_t, __half* dqkv, int B,
                                 int S, int nh, int nkv, int hd, float eps, cudaStream_t st,
                                 const float* dq_slabs = nullptr);
cudaError_t rope_tables(float* cos_t, float* sin_t, int S, int hd, float theta, cudaStream_t st);
cudaError_t ce_valid_rows(uint8_t* valid, const int* targets, int B, int S, int all_positions, int V, int* err,
                          cudaStream_t st);
// Streamed cross-entropy over vocabulary chunks (the lm_head never holds an
// [M, V] tensor).  After the kCEStream GEMM of the chunk [v0, v0 + n): rows
// whose chunk brought a slot above ref + kCeSlotRange move their reference to
// (that max - kCeRefBelowMax), rescaling the row's fp16 chunk values and its
// fp32 d_xf accumulator (first = the first chunk: reference -inf, d_xf rows
// set to 0).  Rows of other chunks are left alone.
constexpr float kCeSlotRange = 11.0f;    // exp(11) < 65504: an unflagged slot's values stay fp16
constexpr float kCeRefBelowMax = 10.0f;  // a new reference sits this far below the row's max
cudaError_t ce_stream_rescale(__half* pc, int ldp, const float* part_ref, int slots, float* ref, float* d_xf, int M,
                              int H, int v0, int n, int first, cudaStream_t st);
// After the last chunk: lse and row losses (+ their sum at row_loss[M]) from
// the slot partials; d_xf -> gscale * (exp(ref - lse) d_xf + (p_t - 1) E_t)
// for rows in the loss, 0 for the others (src/kernels/loss.cu:62-69).
cudaError_t ce_stream_finish(const float* part_ref, const float* part_sum, const float* tgt_logit, const float* ref,
                             const uint8_t* valid, const int* targets, const __half* E, int M, int H, int V,
                             int slots, float gscale, float* lse, float* row_loss_and_sum, float* d_xf,
                             cudaStream_t st);
cudaError_t adamw_flat(float* p, const float* g, float* m, float* v, int64_t n, float lr, float b1, float b2,
                       float eps, float wd, float bc1, float bc2, float gscale, cudaStream_t st);
cudaError_t fill_f32_2d(float* p, int ld, int rows, int cols, float v, cudaStream_t st);
cudaError_t fill_f32(float* p, int64_t n, float v, cudaStream_t st);
cudaError_t fill_normal_f16(__half* p, int64_t n, uint64_t seed, float stddev, cudaStream_t st);
cudaError_t fill_normal_f32(float* p, int64_t n, uint64_t seed, float stddev, cudaStream_t st);
cudaError_t fill_uniform_f32(float* p, int64_t n, uint64_t seed, float lo, float hi, cudaStream_t st);
// dst[r, c] (fp16) = src[r, c] with dst row = row_map(r), optionally transposed
cudaError_t convert_weight(const float* src, int rows, int cols, __half* dst, int ld_dst, int row_off,
                           int interleave, __half* dst_t, int ld_t, int col_off_t, cudaStream_t st);
cudaError_t transpose_f16(const __half* src, int rows, int cols, int ld_src, __half* dst, int ld_dst,
                          cudaStream_t st);
cudaError_t quantize_rows_int8(const float* w, int rows, int cols, int8_t* q, float* scale, cudaStream_t st);
// One CTA whose single wait is never satisfied: it gives up after the
// kernels' bounded-wait limit and ORs kErrWaitProducer into err.
cudaError_t wait_selftest(int* err, cudaStream_t st);
cudaError_t dequant_rows_f16(const int8_t* q, const float* scale, int rows, int cols, __half* out, cudaStream_t st);

}  // namespace llmcu
