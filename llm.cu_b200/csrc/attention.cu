// attention.cu -- host entry points of the causal GQA flash attention.
//
// Replaces the reference's naive_attn_kernel (which writes the full
// probability tensor P [nh, S, S] to HBM, src/kernels/lora_forward.cu:48-135)
// and attn_backward_kernel + expand/contract (global atomics into expanded
// K/V gradients, src/kernels/lora_backward.cu:104-208).  The kernels are the
// tcgen05 ones in attention_tc.cu; this file holds the dO.O row sums of the
// backward, the dispatch, and the allocation-free backward entry point.
#include "../../include/llmcu.h"
#include "common.cuh"

namespace llmcu {

namespace {

// delta[b, h, s] = sum_d dO * O  (fp32), one warp per (row, head)
template <int HD>
__global__ void attn_delta_kernel(const __half* __restrict__ o, const __half* __restrict__ dout,
                                  float* __restrict__ delta, int B, int S, int nh, int ld) {
  pdl_trigger();
  pdl_wait();
  const int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= B * S * nh) return;
  const int h = w % nh;
  const int m = w / nh;  // b * S + s
  const __half* orow = o + static_cast<size_t>(m) * ld + h * HD;
  const __half* drow = dout + static_cast<size_t>(m) * ld + h * HD;
  float acc = 0.f;
  for (int d = lane * 2; d < HD; d += 64) {
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(orow + d));
    const float2 c = __half22float2(*reinterpret_cast<const __half2*>(drow + d));
    acc += a.x * c.x + a.y * c.y;
  }
  acc = warp_sum(acc);
  if (lane == 0) {
    const int b = m / S, s = m % S;
    delta[(static_cast<size_t>(b) * nh + h) * S + s] = acc;
  }
}

template <int HD>
void attn_delta_launch(const __half* o, const __half* dout, float* delta, int B, int S, int nh, int ldo,
                       cudaStream_t st) {
  const int warps = B * S * nh;
  launch_pdl(attn_delta_kernel<HD>, (warps + 7) / 8, 256, 0, st, o, dout, delta, B, S, nh, ldo);
}

}  // namespace

cudaError_t attention_forward(const __half* q, const __half* k, const __half* v, __half* o, float* lse, int B, int S,
                              int nh, int nkv, int hd, int ldq, int ldk, int ldv, int ldo, int* err, cudaStream_t st) {
  return attention_forward_tc(q, k, v, o, lse, B, S, nh, nkv, hd, ldq, ldk, ldv, ldo, err, st);
}

cudaError_t attention_backward(const __half* q, const __half* k, const __half* v, const __half* o,
                               const __half* dout, const float* lse, float* delta, float* dq, float* dk, __half* dv,
                               int B, int S, int nh, int nkv, int hd, int ldq, int ldk, int ldv, int ldo, int lddq,
                               int lddk, int lddv, int* err, cudaStream_t st) {
  if (hd == 128)
    attn_delta_launch<128>(o, dout, delta, B, S, nh, ldo, st);
  else if (hd == 64)
    attn_delta_launch<64>(o, dout, delta, B, S, nh, ldo, st);
  else
    return cudaErrorInvalidValue;
  return attention_backward_tc(q, k, v, dout, lse, delta, dq, dk, dv, B, S, nh, nkv, hd, ldq, ldk, ldv, ldo, lddq,
                               lddk, lddv, err, st);
}

}  // namespace llmcu

namespace llmcu {

// ------------------------------------------- allocation-free backward variant
// File-scope scratch for the row-wise dO.O sums of llmcu_attention_bwd_noalloc.
// Every device that loads this library holds it (4 MiB) until the process
// exits.  In host code the name is only a stand-in; the device address comes
// from cudaGetSymbolAddress with the device current, looked up on every call
// (so it is never stale, e.g. after cudaDeviceReset reloads the module).
namespace {
constexpr int64_t kNoAllocDeltaFloats = 1 << 20;  // batch * n_heads * seq <= 1,048,576
__device__ __align__(256) float g_noalloc_delta[kNoAllocDeltaFloats];

cudaError_t noalloc_scratch(float** out) {
  void* p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_delta);
  *out = static_cast<float*>(p);
  return e;
}
}  // namespace

}  // namespace llmcu

extern "C" llmcu_status llmcu_attention_bwd_noalloc(const void* q, const void* k, const void* v, const void* o,
                                                    const void* dout, const float* lse, float* dq, float* dk,
                                                    void* dv, int batch, int seq, int n_heads, int n_kv_heads,
                                                    int head_dim, int ldq, int ldk, int ldv, int lddv,
                                                    void* stream) {
  using namespace llmcu;
  if (!q || !k || !v || !o || !dout || !lse || !dq || !dk || !dv || batch <= 0 || seq <= 0 || n_heads <= 0 ||
      n_kv_heads <= 0 || n_heads % n_kv_heads)
    return LLMCU_ERR_INVALID_ARG;
  if (static_cast<int64_t>(batch) * n_heads * seq > kNoAllocDeltaFloats) return LLMCU_ERR_UNSUPPORTED;
  if (head_dim != 64 && head_dim != 128) return LLMCU_ERR_UNSUPPORTED;
  float* delta = nullptr;
  int* err = nullptr;  // the kernel-level entry points' error word (llmcu_kernel_checks)
  if (noalloc_scratch(&delta) != cudaSuccess || kernel_err_word(&err) != cudaSuccess) return LLMCU_ERR_CUDA;
  const int ldo = n_heads * head_dim;
  const cudaError_t e = attention_backward(
      static_cast<const __half*>(q), static_cast<const __half*>(k), static_cast<const __half*>(v),
      static_cast<const __half*>(o), static_cast<const __half*>(dout), lse, delta, dq, dk, static_cast<__half*>(dv),
      batch, seq, n_heads, n_kv_heads, head_dim, ldq, ldk, ldv, ldo, ldo, n_kv_heads * head_dim, lddv, err,
      static_cast<cudaStream_t>(stream));
  // as llmcu_attention_bwd: a refused pointer / stride (TMA descriptor) is UNSUPPORTED
  return e == cudaSuccess ? LLMCU_OK : (e == cudaErrorInvalidValue ? LLMCU_ERR_UNSUPPORTED : LLMCU_ERR_CUDA);
}
