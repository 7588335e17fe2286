// decode.cu -- single-sequence KV-cache decoding on the training step's
// weights (inference reuse; the reference's llm_engine, src/main.cu:340-420
// with transformer_decode, src/kernels/forward.cu:340-394):
//   * GEMV for every projection, fp16 rows or INT8 rows with per-row scales
//     (one warp per output row, 16-byte coalesced row reads, the input vector
//     staged once per block in shared memory; optional residual add);
//   * one kernel from the raw q/k/v row to the attention output: QK-norm +
//     RoPE of the position, the K / V cache append, attention split over key
//     ranges (partial max / sum / output each) and the merge of the splits;
//   * the RMSNorms and the SwiGLU folded into the GEMVs' input staging;
//   * greedy argmax (lowest id on ties, as the reference's host loop).
// The position being decoded lives in device memory (`d_pos`) and every
// kernel reads it there, so one decode step is captured once into a CUDA
// graph and replayed per token.
#include "common.cuh"

namespace llmcu {

namespace {

constexpr int kGemvThreads = 256;  // 8 warps; a warp owns one output row at a time

// How a GEMV forms its fp16 input vector in shared memory:
enum : int {
  kXHalf = 0,    // x is the fp16 vector itself
  kXNorm = 1,    // x is an fp32 row: RMSNorm with gain g (each block forms the row's rstd)
  kXSwiGLU = 2,  // x is the fp16 gate/up row [2K], interleaved in 128-row groups: silu(g) * u
};

// y[n] = s[n] * sum_k W[n, k] x[k] for W fp16 (s = 1) or INT8 [N, K] (row
// stride ldw), x as kX says.  out32 (nullable) = resid[n] (nullable: 0) + y;
// out16 (nullable) = fp16(y).  The fused input forms repeat the separate
// kernels' arithmetic (rmsnorm_fwd_row_kernel, the SwiGLU of one row), so a
// norm or activation costs no launch of its own.
template <bool kInt8, int kX>
__global__ void __launch_bounds__(kGemvThreads) gemv_kernel(const void* __restrict__ W, const float* __restrict__ scale,
                                                            int ldw, const void* __restrict__ xin,
                                                            const float* __restrict__ gain, float eps, int N, int K,
                                                            const float* __restrict__ resid, float* __restrict__ out32,
                                                            __half* __restrict__ out16) {
  pdl_trigger();
  extern __shared__ __align__(16) __half gv_x[];
  __shared__ float gv_red[kGemvThreads / 32];
  pdl_wait();
  if constexpr (kX == kXHalf) {
    const __half* x = static_cast<const __half*>(xin);
    for (int i = threadIdx.x * 8; i < K; i += blockDim.x * 8)
      *reinterpret_cast<uint4*>(gv_x + i) = *reinterpret_cast<const uint4*>(x + i);
  } else if constexpr (kX == kXNorm) {
    // the thread's share of x and the gain, all loads issued before any use
    // (K <= 4 * 4 * blockDim.x: at most four float4 per thread)
    const float* x = static_cast<const float*>(xin);
    float4 v[4], g[4];
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int i = (threadIdx.x + j * blockDim.x) * 4;
      v[j] = i < K ? *reinterpret_cast<const float4*>(x + i) : make_float4(0.f, 0.f, 0.f, 0.f);
      g[j] = i < K ? *reinterpret_cast<const float4*>(gain + i) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) ss += v[j].x * v[j].x + v[j].y * v[j].y + v[j].z * v[j].z + v[j].w * v[j].w;
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) gv_red[threadIdx.x >> 5] = ss;
    __syncthreads();
    ss = 0.f;
#pragma unroll
    for (int w = 0; w < kGemvThreads / 32; ++w) ss += gv_red[w];
    const float r = rsqrtf(ss / static_cast<float>(K) + eps);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int i = (threadIdx.x + j * blockDim.x) * 4;
      if (i < K) {
        uint2 u;
        u.x = pack_half2(v[j].x * r * g[j].x, v[j].y * r * g[j].y);
        u.y = pack_half2(v[j].z * r * g[j].z, v[j].w * r * g[j].w);
        *reinterpret_cast<uint2*>(gv_x + i) = u;
      }
    }
  } else {
    // eight activations per chunk from 16-byte gate and up loads, every
    // chunk's loads issued first (K <= 4 * 8 * blockDim.x)
    const __half* gu = static_cast<const __half*>(xin);
    uint4 gq[4], uq[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int i = (threadIdx.x + j * blockDim.x) * 8;
      const int grp = i >> 7, jj = i & 127;
      gq[j] = i < K ? *reinterpret_cast<const uint4*>(gu + grp * 256 + jj) : make_uint4(0u, 0u, 0u, 0u);
      uq[j] = i < K ? *reinterpret_cast<const uint4*>(gu + grp * 256 + 128 + jj) : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int i = (threadIdx.x + j * blockDim.x) * 8;
      if (i < K) {
        const __half2* hg = reinterpret_cast<const __half2*>(&gq[j]);
        const __half2* hu = reinterpret_cast<const __half2*>(&uq[j]);
        uint32_t o[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 fg = __half22float2(hg[e]), fu = __half22float2(hu[e]);
          o[e] = pack_half2(fg.x / (1.0f + __expf(-fg.x)) * fu.x, fg.y / (1.0f + __expf(-fg.y)) * fu.y);
        }
        *reinterpret_cast<uint4*>(gv_x + i) = make_uint4(o[0], o[1], o[2], o[3]);
      }
    }
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int warps = gridDim.x * (blockDim.x >> 5);
  for (int n = blockIdx.x * (blockDim.x >> 5) + warp; n < N; n += warps) {
    float acc = 0.f;
    if constexpr (kInt8) {
      const int8_t* row = static_cast<const int8_t*>(W) + static_cast<size_t>(n) * ldw;
#pragma unroll 4
      for (int k = lane * 16; k < K; k += 32 * 16) {
        const int4 q = __ldg(reinterpret_cast<const int4*>(row + k));
        const int8_t* qb = reinterpret_cast<const int8_t*>(&q);
        const uint4 xa = *reinterpret_cast<const uint4*>(gv_x + k);
        const uint4 xb = *reinterpret_cast<const uint4*>(gv_x + k + 8);
        const __half2* ha = reinterpret_cast<const __half2*>(&xa);
        const __half2* hb = reinterpret_cast<const __half2*>(&xb);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 fa = __half22float2(ha[j]), fb = __half22float2(hb[j]);
          acc = fmaf(static_cast<float>(qb[2 * j]), fa.x, acc);
          acc = fmaf(static_cast<float>(qb[2 * j + 1]), fa.y, acc);
          acc = fmaf(static_cast<float>(qb[8 + 2 * j]), fb.x, acc);
          acc = fmaf(static_cast<float>(qb[8 + 2 * j + 1]), fb.y, acc);
        }
      }
    } else {
      const __half* row = static_cast<const __half*>(W) + static_cast<size_t>(n) * ldw;
#pragma unroll 4
      for (int k = lane * 8; k < K; k += 32 * 8) {
        const uint4 w = __ldg(reinterpret_cast<const uint4*>(row + k));
        const uint4 xv = *reinterpret_cast<const uint4*>(gv_x + k);
        const __half2* hw = reinterpret_cast<const __half2*>(&w);
        const __half2* hx = reinterpret_cast<const __half2*>(&xv);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 fw = __half22float2(hw[j]), fx = __half22float2(hx[j]);
          acc = fmaf(fw.x, fx.x, acc);
          acc = fmaf(fw.y, fx.y, acc);
        }
      }
    }
    acc = warp_sum(acc);
    if (lane == 0) {
      const float y = kInt8 ? acc * scale[n] : acc;
      if (out32) out32[n] = (resid ? resid[n] : 0.f) + y;
      if (out16) out16[n] = __float2half_rn(y);
    }
  }
}

// Per-head RMSNorm (gain g) and rotation of pairs (d, d + HD/2) at position
// pos for the warp's head row src -- the arithmetic of
// qknorm_rope_fwd_vec_kernel -- rounded to fp16; lane holds pairs
// d = lane + 32 p, in y0 (d) and y1 (d + HD/2).
template <int HD>
__device__ __forceinline__ void rope_head(const __half* src, const float* g, const float* cos_t, const float* sin_t,
                                          int pos, float eps, int lane, __half (&y0)[HD / 64], __half (&y1)[HD / 64]) {
  constexpr int kHalf = HD / 2, kP = HD / 64;
  float a[kP], b[kP];
  float ss = 0.f;
#pragma unroll
  for (int p = 0; p < kP; ++p) {
    a[p] = __half2float(src[lane + 32 * p]);
    b[p] = __half2float(src[lane + 32 * p + kHalf]);
    ss += a[p] * a[p] + b[p] * b[p];
  }
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / static_cast<float>(HD) + eps);
#pragma unroll
  for (int p = 0; p < kP; ++p) {
    const int d = lane + 32 * p;
    const float c = cos_t[pos * kHalf + d], s = sin_t[pos * kHalf + d];
    const float x = a[p] * r * g[d], y = b[p] * r * g[d + kHalf];
    y0[p] = __float2half_rn(x * c - y * s);
    y1[p] = __float2half_rn(y * c + x * s);
  }
}

// Attention of one position over the cache, everything between the q/k/v
// GEMV and the o-projection in one launch.  Block (h, sp) takes the kDecT
// keys [sp * kDecT, ...) of the cache rows [0, pos] (pos = *d_pos):
//   * warp 0 forms the head's q (QK-norm + RoPE) from the raw q/k/v row;
//   * the block whose range holds pos forms that position's k (QK-norm +
//     RoPE) and v, appends them to the cache (both query heads of a KV group
//     write the same bytes) and uses them directly; older rows are staged
//     from the cache with 16-byte loads through L2, all in flight at once;
//   * scores, max, exp2 and the partial output {o[HD], m, l} (log2 domain)
//     go to part[h][sp]; the last block of the head to finish (a ticket per
//     head) merges the splits into the fp16 output row.
constexpr int kDecT = 32;
template <int HD>
__global__ void __launch_bounds__(128) decode_attn_kernel(const __half* __restrict__ qkv, const float* __restrict__ qn_w,
                                                          const float* __restrict__ kn_w,
                                                          const float* __restrict__ cos_t,
                                                          const float* __restrict__ sin_t,
                                                          const int* __restrict__ d_pos, __half* __restrict__ k_cache,
                                                          __half* __restrict__ v_cache, float* __restrict__ part,
                                                          int* __restrict__ tickets, __half* __restrict__ out, int nh,
                                                          int nkv, float eps, float scale_log2) {
  pdl_trigger();
  __shared__ __align__(16) __half ks[kDecT][HD + 8];
  __shared__ __align__(16) __half vs[kDecT][HD + 8];
  __shared__ float qs[HD];
  __shared__ float ps[kDecT];
  __shared__ float stat[2];
  __shared__ int last;
  pdl_wait();
  constexpr int kHalf = HD / 2, kP = HD / 64;
  const int h = blockIdx.x, sp = blockIdx.y, splits = gridDim.y;
  const int kvh = h / (nh / nkv);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int pos = __ldcg(d_pos);  // written by the previous step's argmax: read through L2
  const int L = pos + 1;
  const int t0 = sp * kDecT;
  const size_t kv_stride = static_cast<size_t>(nkv) * HD;
  float* dst = part + (static_cast<size_t>(h) * splits + sp) * (HD + 2);
  if (t0 < L) {  // block-uniform
    const int n = min(kDecT, L - t0);
    const bool mine = pos < t0 + kDecT;  // this block holds the new row pos - t0
    constexpr int kC = HD / 8;           // 16-byte chunks per row
    for (int i = threadIdx.x; i < n * kC; i += blockDim.x) {
      const int r = i / kC, c = i % kC;
      if (t0 + r == pos) continue;
      const size_t off = static_cast<size_t>(t0 + r) * kv_stride + kvh * HD + c * 8;
      *reinterpret_cast<uint4*>(&ks[r][c * 8]) = __ldcg(reinterpret_cast<const uint4*>(k_cache + off));
      *reinterpret_cast<uint4*>(&vs[r][c * 8]) = __ldcg(reinterpret_cast<const uint4*>(v_cache + off));
    }
    if (warp == 0) {
      __half y0[kP], y1[kP];
      rope_head<HD>(qkv + static_cast<size_t>(h) * HD, qn_w, cos_t, sin_t, pos, eps, lane, y0, y1);
#pragma unroll
      for (int p = 0; p < kP; ++p) {
        qs[lane + 32 * p] = __half2float(y0[p]) * scale_log2;
        qs[lane + 32 * p + kHalf] = __half2float(y1[p]) * scale_log2;
      }
    } else if (mine && warp == 1) {
      __half y0[kP], y1[kP];
      rope_head<HD>(qkv + static_cast<size_t>(nh + kvh) * HD, kn_w, cos_t, sin_t, pos, eps, lane, y0, y1);
      __half* kc = k_cache + static_cast<size_t>(pos) * kv_stride + kvh * HD;
#pragma unroll
      for (int p = 0; p < kP; ++p) {
        const int d = lane + 32 * p;
        ks[pos - t0][d] = y0[p];
        ks[pos - t0][d + kHalf] = y1[p];
        kc[d] = y0[p];
        kc[d + kHalf] = y1[p];
      }
    } else if (mine && warp == 2) {
      const __half* src = qkv + static_cast<size_t>(nh + nkv + kvh) * HD;
      __half* vc = v_cache + static_cast<size_t>(pos) * kv_stride + kvh * HD;
      for (int d = lane; d < HD; d += 32) {
        vs[pos - t0][d] = src[d];
        vc[d] = src[d];
      }
    }
    __syncthreads();
#pragma unroll
    for (int j = 0; j < kDecT / 4; ++j) {  // warp w: keys 8w .. 8w + 7
      const int r = warp * (kDecT / 4) + j;
      if (r < n) {
        float sc = 0.f;
#pragma unroll
        for (int d = lane; d < HD; d += 32) sc = fmaf(qs[d], __half2float(ks[r][d]), sc);
        sc = warp_sum(sc);
        if (lane == 0) ps[r] = sc;
      }
    }
    __syncthreads();
    if (warp == 0) {
      const float v = lane < n ? ps[lane] : -INFINITY;
      const float m = warp_max(v);
      const float p = lane < n ? exp2f(v - m) : 0.f;
      const float l = warp_sum(p);
      if (lane < n) ps[lane] = p;
      if (lane == 0) {
        stat[0] = m;
        stat[1] = l;
      }
    }
    __syncthreads();
    for (int d = threadIdx.x; d < HD; d += blockDim.x) {
      float o = 0.f;
      for (int r = 0; r < n; ++r) o = fmaf(ps[r], __half2float(vs[r][d]), o);
      __stcg(dst + d, o);
    }
    if (threadIdx.x == 0) {
      __stcg(dst + HD, stat[0]);
      __stcg(dst + HD + 1, stat[1]);
    }
  } else {  // no keys here
    for (int d = threadIdx.x; d < HD; d += blockDim.x) __stcg(dst + d, 0.f);
    if (threadIdx.x == 0) {
      __stcg(dst + HD, -INFINITY);
      __stcg(dst + HD + 1, 0.f);
    }
  }
  // the head's last block merges: out[h][d] = sum 2^(m - M) o[d] / sum 2^(m - M) l
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) last = atomicAdd(tickets + h, 1) == splits - 1;
  __syncthreads();
  if (!last) return;
  __threadfence();
  const float* ph = part + static_cast<size_t>(h) * splits * (HD + 2);
  float M = -INFINITY;
  for (int s2 = 0; s2 < splits; ++s2) M = fmaxf(M, __ldcg(ph + s2 * (HD + 2) + HD));
  for (int d = threadIdx.x; d < HD; d += blockDim.x) {
    float num = 0.f, den = 0.f;
    for (int s2 = 0; s2 < splits; ++s2) {
      const float m = __ldcg(ph + s2 * (HD + 2) + HD);
      if (m == -INFINITY) continue;
      const float f = exp2f(m - M);
      num = fmaf(f, __ldcg(ph + s2 * (HD + 2) + d), num);
      den = fmaf(f, __ldcg(ph + s2 * (HD + 2) + HD + 1), den);
    }
    out[static_cast<size_t>(h) * HD + d] = __float2half_rn(den > 0.f ? num / den : 0.f);
  }
  if (threadIdx.x == 0) __stcg(tickets + h, 0);  // for the next step
}

// (value, id) pair order of the greedy choice: larger value, then lower id
__device__ __forceinline__ void amax_merge(float& best, int& idx, float v2, int i2) {
  if (v2 > best || (v2 == best && i2 < idx)) {
    best = v2;
    idx = i2;
  }
}
__device__ __forceinline__ void amax_warp(float& best, int& idx) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
    amax_merge(best, idx, __shfl_xor_sync(0xffffffffu, best, o), __shfl_xor_sync(0xffffffffu, idx, o));
}

// Greedy choice over logits [V] (the first maximum, as the reference's host
// loop), spread over kAmaxBlocks blocks: each leaves its chunk's best in
// (pval, pidx); the last block to finish (a ticket in counters[3]) picks the
// overall best: tokens[step] = next = argmax, then the step and the position
// advance.  step_logits (nullable) row `step` receives the logits.
constexpr int kAmaxBlocks = 128;
__global__ void __launch_bounds__(256) decode_argmax_kernel(const float* __restrict__ logits, int V,
                                                            int* __restrict__ counters, int* __restrict__ tokens,
                                                            float* __restrict__ step_logits, float* __restrict__ pval,
                                                            int* __restrict__ pidx) {
  pdl_trigger();
  pdl_wait();
  __shared__ float bv[8];
  __shared__ int bi[8];
  __shared__ int last;
  const int step = __ldcg(counters + 1);  // the counters change every step: L2 only
  float best = -INFINITY;
  int idx = 0x7fffffff;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < V; i += gridDim.x * blockDim.x) {
    const float v = logits[i];
    amax_merge(best, idx, v, i);
    if (step_logits) step_logits[static_cast<size_t>(step) * V + i] = v;
  }
  amax_warp(best, idx);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    bv[warp] = best;
    bi[warp] = idx;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < static_cast<int>(blockDim.x >> 5); ++w) amax_merge(best, idx, bv[w], bi[w]);
    __stcg(pval + blockIdx.x, best);
    __stcg(pidx + blockIdx.x, idx);
    __threadfence();
    last = atomicAdd(counters + 3, 1) == static_cast<int>(gridDim.x) - 1;
  }
  __syncthreads();
  if (!last || warp != 0) return;
  __threadfence();
  best = -INFINITY;
  idx = 0x7fffffff;
  for (int b = lane; b < static_cast<int>(gridDim.x); b += 32) amax_merge(best, idx, __ldcg(pval + b), __ldcg(pidx + b));
  amax_warp(best, idx);
  if (lane == 0) {
    if (idx == 0x7fffffff) idx = 0;  // every logit NaN
    tokens[step] = idx;
    __stcg(counters + 2, idx);  // the next step's input token
    __stcg(counters + 1, step + 1);
    __stcg(counters, __ldcg(counters) + 1);  // its position
    __stcg(counters + 3, 0);                 // ticket for the next step
  }
}

}  // namespace

int decode_attn_splits(int max_ctx) { return max_ctx < 1 ? 1 : (max_ctx + kDecT - 1) / kDecT; }

cudaError_t decode_gemv(const void* W, const float* scale, bool int8, int ldw, const void* x, int xmode,
                        const float* gain, float eps, int N, int K, const float* resid, float* out32, __half* out16,
                        cudaStream_t st) {
  if (K % (int8 ? 16 : 8) || ldw % (int8 ? 16 : 8) || reinterpret_cast<uintptr_t>(W) % 16 ||
      reinterpret_cast<uintptr_t>(x) % 16 || (int8 && !scale) || (xmode == kXNorm && !gain) ||
      (xmode == kXSwiGLU && K % 128) || xmode < 0 || xmode > 2 ||
      (xmode == kXNorm && (K > 16 * kGemvThreads || K % 4)) || (xmode == kXSwiGLU && K > 32 * kGemvThreads))
    return cudaErrorInvalidValue;
  const int rows_per_block = kGemvThreads / 32;
  int blocks = (N + rows_per_block - 1) / rows_per_block;
  const int cap = 8 * gemm_num_sms();
  if (blocks > cap) blocks = cap;
  const size_t smem = static_cast<size_t>(K) * sizeof(__half);
#define LLMCU_GEMV(I8, XM)                                                                                     \
  launch_pdl(gemv_kernel<I8, XM>, blocks, kGemvThreads, smem, st, W, scale, ldw, x, gain, eps, N, K, resid, out32, \
             out16)
  if (int8) {
    if (xmode == kXHalf) LLMCU_GEMV(true, kXHalf);
    else if (xmode == kXNorm) LLMCU_GEMV(true, kXNorm);
    else LLMCU_GEMV(true, kXSwiGLU);
  } else {
    if (xmode == kXHalf) LLMCU_GEMV(false, kXHalf);
    else if (xmode == kXNorm) LLMCU_GEMV(false, kXNorm);
    else LLMCU_GEMV(false, kXSwiGLU);
  }
#undef LLMCU_GEMV
  return cudaGetLastError();
}

cudaError_t decode_attention(const __half* qkv, const float* qn_w, const float* kn_w, const float* cos_t,
                             const float* sin_t, const int* d_pos, __half* k_cache, __half* v_cache, float* part,
                             int* tickets, __half* out, int nh, int nkv, int hd, float eps, int max_ctx,
                             cudaStream_t st) {
  if (nkv <= 0 || nh % nkv) return cudaErrorInvalidValue;
  const dim3 grid(nh, decode_attn_splits(max_ctx));
  const float scale_log2 = kLog2e / sqrtf(static_cast<float>(hd));
  if (hd == 128)
    launch_pdl(decode_attn_kernel<128>, grid, 128, 0, st, qkv, qn_w, kn_w, cos_t, sin_t, d_pos, k_cache, v_cache,
               part, tickets, out, nh, nkv, eps, scale_log2);
  else if (hd == 64)
    launch_pdl(decode_attn_kernel<64>, grid, 128, 0, st, qkv, qn_w, kn_w, cos_t, sin_t, d_pos, k_cache, v_cache, part,
               tickets, out, nh, nkv, eps, scale_log2);
  else
    return cudaErrorInvalidValue;
  return cudaGetLastError();
}

int decode_argmax_scratch() { return 2 * kAmaxBlocks; }

cudaError_t decode_argmax(const float* logits, int V, int* counters, int* tokens, float* step_logits, float* scratch,
                          cudaStream_t st) {
  launch_pdl(decode_argmax_kernel, kAmaxBlocks, 256, 0, st, logits, V, counters, tokens, step_logits, scratch,
             reinterpret_cast<int*>(scratch + kAmaxBlocks));
  return cudaGetLastError();
}

}  // namespace llmcu
