// decode.cu -- single-sequence KV-cache decoding on the training step's
// weights (inference reuse; the reference's llm_engine, src/main.cu:340-420
// with transformer_decode, src/kernels/forward.cu:340-394):
//   * GEMV for every projection, fp16 rows or INT8 rows with per-row scales
//     (one warp per output row, 16-byte coalesced row reads, the input vector
//     staged once per block in shared memory; optional residual add);
//   * QK-norm + RoPE of one position, writing K and V into the cache;
//   * attention of one query over the cache, split over key ranges (each
//     split a partial max / sum / output, then one combine per head);
//   * SwiGLU of one row (gate/up interleaved in 128-row groups, as stored);
//   * greedy argmax (lowest id on ties, as the reference's host loop).
// The position being decoded lives in device memory (`d_pos`) and every
// kernel reads it there, so one decode step is captured once into a CUDA
// graph and replayed per token.
#include "common.cuh"

namespace llmcu {

namespace {

constexpr int kGemvThreads = 256;  // 8 warps; a warp owns one output row at a time

// y[n] = s[n] * sum_k W[n, k] x[k] for W fp16 (s = 1) or INT8 [N, K] (row
// stride ldw); x fp16 [K].  out32 (nullable) = resid[n] (nullable: 0) + y;
// out16 (nullable) = fp16(y).
template <bool kInt8>
__global__ void __launch_bounds__(kGemvThreads) gemv_kernel(const void* __restrict__ W, const float* __restrict__ scale,
                                                            int ldw, const __half* __restrict__ x, int N, int K,
                                                            const float* __restrict__ resid, float* __restrict__ out32,
                                                            __half* __restrict__ out16) {
  pdl_trigger();
  extern __shared__ __align__(16) __half gv_x[];
  pdl_wait();
  for (int i = threadIdx.x * 8; i < K; i += blockDim.x * 8)
    *reinterpret_cast<uint4*>(gv_x + i) = *reinterpret_cast<const uint4*>(x + i);
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

// One warp per head of [q heads | k heads | v heads] of the position *d_pos:
// q and k get the per-head RMSNorm (gain q_norm / k_norm) and the rotation of
// pairs (d, d + hd/2) -- the arithmetic of qknorm_rope_fwd_vec_kernel -- q
// into q_out, k into the K cache row; v is copied into the V cache row.
template <int HD>
__global__ void decode_qk_rope_kernel(const __half* __restrict__ qkv, const float* __restrict__ qn_w,
                                      const float* __restrict__ kn_w, const float* __restrict__ cos_t,
                                      const float* __restrict__ sin_t, const int* __restrict__ d_pos,
                                      __half* __restrict__ q_out, __half* __restrict__ k_cache,
                                      __half* __restrict__ v_cache, int nh, int nkv, float eps) {
  pdl_trigger();
  pdl_wait();
  constexpr int kHalf = HD / 2, kP = kHalf / 32;  // rotation pairs per lane
  const int w = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (w >= nh + 2 * nkv) return;  // whole warp
  const int pos = __ldcg(d_pos);  // written by the previous step's argmax: read through L2
  if (w >= nh + nkv) {  // v head
    const int vh = w - nh - nkv;
    const __half* src = qkv + static_cast<size_t>(nh + nkv) * HD + vh * HD;
    __half* dst = v_cache + static_cast<size_t>(pos) * nkv * HD + vh * HD;
    for (int d = lane; d < HD; d += 32) dst[d] = src[d];
    return;
  }
  const bool isq = w < nh;
  const __half* src = qkv + static_cast<size_t>(w) * HD;  // q heads, then k heads
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
  const float* gw = isq ? qn_w : kn_w;
  __half* dst = isq ? q_out + static_cast<size_t>(w) * HD
                    : k_cache + static_cast<size_t>(pos) * nkv * HD + (w - nh) * HD;
#pragma unroll
  for (int p = 0; p < kP; ++p) {
    const int d = lane + 32 * p;
    const float c = cos_t[pos * kHalf + d], s = sin_t[pos * kHalf + d];
    const float x = a[p] * r * gw[d], y = b[p] * r * gw[d + kHalf];
    dst[d] = __float2half_rn(x * c - y * s);
    dst[d + kHalf] = __float2half_rn(y * c + x * s);
  }
}

// Attention of the query heads over cache rows [0, *d_pos]: block (h, sp)
// takes the kDecT keys [sp * kDecT, ...), stages their K and V rows in shared
// memory with 16-byte loads (all in flight at once), and leaves its partial
// output, max and sum (log2 domain) in part[h][sp] = {o[HD], m, l}.
constexpr int kDecT = 32;
template <int HD>
__global__ void __launch_bounds__(128) decode_attn_kernel(const __half* __restrict__ q,
                                                          const __half* __restrict__ k_cache,
                                                          const __half* __restrict__ v_cache,
                                                          const int* __restrict__ d_pos, float* __restrict__ part,
                                                          int nh, int nkv, float scale_log2) {
  pdl_trigger();
  __shared__ __align__(16) __half ks[kDecT][HD + 8];
  __shared__ __align__(16) __half vs[kDecT][HD + 8];
  __shared__ float qs[HD];
  __shared__ float ps[kDecT];
  __shared__ float stat[2];
  pdl_wait();
  const int h = blockIdx.x, sp = blockIdx.y, splits = gridDim.y;
  const int kvh = h / (nh / nkv);
  const int L = __ldcg(d_pos) + 1;
  const int t0 = sp * kDecT;
  float* dst = part + (static_cast<size_t>(h) * splits + sp) * (HD + 2);
  if (t0 >= L) {  // whole block: no keys here
    for (int d = threadIdx.x; d < HD; d += blockDim.x) dst[d] = 0.f;
    if (threadIdx.x == 0) {
      dst[HD] = -INFINITY;
      dst[HD + 1] = 0.f;
    }
    return;
  }
  const int n = min(kDecT, L - t0);
  const size_t kv_stride = static_cast<size_t>(nkv) * HD;
  constexpr int kC = HD / 8;  // 16-byte chunks per row
  for (int i = threadIdx.x; i < n * kC; i += blockDim.x) {
    const int r = i / kC, c = i % kC;
    const size_t off = static_cast<size_t>(t0 + r) * kv_stride + kvh * HD + c * 8;
    *reinterpret_cast<uint4*>(&ks[r][c * 8]) = __ldg(reinterpret_cast<const uint4*>(k_cache + off));
    *reinterpret_cast<uint4*>(&vs[r][c * 8]) = __ldg(reinterpret_cast<const uint4*>(v_cache + off));
  }
  for (int d = threadIdx.x; d < HD; d += blockDim.x) qs[d] = __half2float(q[static_cast<size_t>(h) * HD + d]) * scale_log2;
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
  for (int j = 0; j < kDecT / 4; ++j) {  // warp w: keys 8w .. 8w + 7
    const int r = warp * (kDecT / 4) + j;
    if (r < n) {
      float s = 0.f;
#pragma unroll
      for (int d = lane; d < HD; d += 32) s = fmaf(qs[d], __half2float(ks[r][d]), s);
      s = warp_sum(s);
      if (lane == 0) ps[r] = s;
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
    dst[d] = o;
  }
  if (threadIdx.x == 0) {
    dst[HD] = stat[0];
    dst[HD + 1] = stat[1];
  }
}

// out[h][d] = sum_sp 2^(m_sp - M) o_sp[d] / sum_sp 2^(m_sp - M) l_sp (fp16)
template <int HD>
__global__ void decode_attn_combine_kernel(const float* __restrict__ part, __half* __restrict__ out, int splits) {
  pdl_trigger();
  pdl_wait();
  const int h = blockIdx.x, d = threadIdx.x;
  const float* ph = part + static_cast<size_t>(h) * splits * (HD + 2);
  float M = -INFINITY;
  for (int sp = 0; sp < splits; ++sp) M = fmaxf(M, ph[sp * (HD + 2) + HD]);
  float num = 0.f, den = 0.f;
  for (int sp = 0; sp < splits; ++sp) {
    const float m = ph[sp * (HD + 2) + HD];
    if (m == -INFINITY) continue;
    const float f = exp2f(m - M);
    num = fmaf(f, ph[sp * (HD + 2) + d], num);
    den = fmaf(f, ph[sp * (HD + 2) + HD + 1], den);
  }
  out[static_cast<size_t>(h) * HD + d] = __float2half_rn(den > 0.f ? num / den : 0.f);
}

// act[i] = silu(g) * u for the gate/up rows stored interleaved in 128-row
// groups (row group j: gate rows j*128.., then the matching up rows)
__global__ void decode_swiglu_kernel(const __half* __restrict__ gu, __half* __restrict__ act, int I) {
  pdl_trigger();
  pdl_wait();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= I) return;
  const int grp = i >> 7, j = i & 127;
  const float g = __half2float(gu[grp * 256 + j]), u = __half2float(gu[grp * 256 + 128 + j]);
  act[i] = __float2half_rn(g / (1.0f + __expf(-g)) * u);
}

// Greedy choice over logits [V] (the first maximum, as the reference's host
// loop): tokens[*d_step] = next = argmax; step_logits (nullable) row *d_step
// receives the logits; then the step and the position advance.
__global__ void __launch_bounds__(1024) decode_argmax_kernel(const float* __restrict__ logits, int V,
                                                             int* __restrict__ counters, int* __restrict__ tokens,
                                                             float* __restrict__ step_logits) {
  pdl_trigger();
  pdl_wait();
  __shared__ float bv[32];
  __shared__ int bi[32];
  const int step = __ldcg(counters + 1);  // the counters change every step: L2 only
  float best = -INFINITY;
  int idx = 0x7fffffff;
  for (int i = threadIdx.x; i < V; i += blockDim.x) {
    const float v = logits[i];
    if (v > best || (v == best && i < idx)) {
      best = v;
      idx = i;
    }
    if (step_logits) step_logits[static_cast<size_t>(step) * V + i] = v;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float v2 = __shfl_xor_sync(0xffffffffu, best, o);
    const int i2 = __shfl_xor_sync(0xffffffffu, idx, o);
    if (v2 > best || (v2 == best && i2 < idx)) {
      best = v2;
      idx = i2;
    }
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    bv[warp] = best;
    bi[warp] = idx;
  }
  __syncthreads();
  if (warp == 0) {
    best = lane < (blockDim.x >> 5) ? bv[lane] : -INFINITY;
    idx = lane < (blockDim.x >> 5) ? bi[lane] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float v2 = __shfl_xor_sync(0xffffffffu, best, o);
      const int i2 = __shfl_xor_sync(0xffffffffu, idx, o);
      if (v2 > best || (v2 == best && i2 < idx)) {
        best = v2;
        idx = i2;
      }
    }
    if (lane == 0) {
      if (idx == 0x7fffffff) idx = 0;  // every logit NaN
      tokens[step] = idx;
      __stcg(counters + 2, idx);  // the next step's input token
      __stcg(counters + 1, step + 1);
      __stcg(counters, __ldcg(counters) + 1);  // its position
    }
  }
}

}  // namespace

int decode_attn_splits(int max_ctx) { return max_ctx < 1 ? 1 : (max_ctx + kDecT - 1) / kDecT; }

cudaError_t decode_gemv(const void* W, const float* scale, bool int8, int ldw, const __half* x, int N, int K,
                        const float* resid, float* out32, __half* out16, cudaStream_t st) {
  if (K % (int8 ? 16 : 8) || ldw % (int8 ? 16 : 8) || reinterpret_cast<uintptr_t>(W) % 16 ||
      reinterpret_cast<uintptr_t>(x) % 16 || (int8 && !scale))
    return cudaErrorInvalidValue;
  const int rows_per_block = kGemvThreads / 32;
  int blocks = (N + rows_per_block - 1) / rows_per_block;
  const int cap = 8 * gemm_num_sms();
  if (blocks > cap) blocks = cap;
  const size_t smem = static_cast<size_t>(K) * sizeof(__half);
  if (int8)
    launch_pdl(gemv_kernel<true>, blocks, kGemvThreads, smem, st, W, scale, ldw, x, N, K, resid, out32, out16);
  else
    launch_pdl(gemv_kernel<false>, blocks, kGemvThreads, smem, st, W, scale, ldw, x, N, K, resid, out32, out16);
  return cudaGetLastError();
}

cudaError_t decode_qk_rope(const __half* qkv, const float* qn_w, const float* kn_w, const float* cos_t,
                           const float* sin_t, const int* d_pos, __half* q_out, __half* k_cache, __half* v_cache,
                           int nh, int nkv, int hd, float eps, cudaStream_t st) {
  const int warps = nh + 2 * nkv;
  const int blocks = (warps + 3) / 4;
  if (hd == 128)
    launch_pdl(decode_qk_rope_kernel<128>, blocks, 128, 0, st, qkv, qn_w, kn_w, cos_t, sin_t, d_pos, q_out, k_cache,
               v_cache, nh, nkv, eps);
  else if (hd == 64)
    launch_pdl(decode_qk_rope_kernel<64>, blocks, 128, 0, st, qkv, qn_w, kn_w, cos_t, sin_t, d_pos, q_out, k_cache,
               v_cache, nh, nkv, eps);
  else
    return cudaErrorInvalidValue;
  return cudaGetLastError();
}

cudaError_t decode_attention(const __half* q, const __half* k_cache, const __half* v_cache, const int* d_pos,
                             float* part, __half* out, int nh, int nkv, int hd, int max_ctx, cudaStream_t st) {
  if (nkv <= 0 || nh % nkv) return cudaErrorInvalidValue;
  const int splits = decode_attn_splits(max_ctx);
  const float scale_log2 = kLog2e / sqrtf(static_cast<float>(hd));
  const dim3 grid(nh, splits);
  if (hd == 128) {
    launch_pdl(decode_attn_kernel<128>, grid, 128, 0, st, q, k_cache, v_cache, d_pos, part, nh, nkv, scale_log2);
    launch_pdl(decode_attn_combine_kernel<128>, nh, 128, 0, st, part, out, splits);
  } else if (hd == 64) {
    launch_pdl(decode_attn_kernel<64>, grid, 128, 0, st, q, k_cache, v_cache, d_pos, part, nh, nkv, scale_log2);
    launch_pdl(decode_attn_combine_kernel<64>, nh, 64, 0, st, part, out, splits);
  } else {
    return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t decode_swiglu(const __half* gu, __half* act, int I, cudaStream_t st) {
  if (I % 128) return cudaErrorInvalidValue;
  launch_pdl(decode_swiglu_kernel, (I + 255) / 256, 256, 0, st, gu, act, I);
  return cudaGetLastError();
}

cudaError_t decode_argmax(const float* logits, int V, int* counters, int* tokens, float* step_logits,
                          cudaStream_t st) {
  launch_pdl(decode_argmax_kernel, 1, 1024, 0, st, logits, V, counters, tokens, step_logits);
  return cudaGetLastError();
}

}  // namespace llmcu
