// lora.cu -- LoRA operand preparation and the adapter-gradient kernel.
//
// Adapters live in one flat fp32 buffer (per layer: Aq Bq Ak Bk Av Bv Ao Bo,
// A [r, d_in], B [d_out, r] as include/lora.h:13-20 of the reference), so
// AdamW and the data-parallel allreduce each touch one contiguous range.
//
// lora_prep builds, per layer and per step, the fp16 operands the tcgen05
// GEMMs consume as their 64-wide second K-segment (rank padded to 64):
//   acat  [64, H]   rows 0.. = Aq, 16.. = Ak, 32.. = Av (r rows each) (and acatT)
//   bblk  [QKV, 64] block-diagonal s*Bq | s*Bk | s*Bv, same columns  (and bblkT)
// (each rank segment starts on a 16-column boundary so every operand view
// h + 16*i stays 32-byte aligned for the 16-byte async copies)
//   ao    [64, Q]   rows 0..r-1 = Ao                               (and aoT)
//   bo    [H, 64]   cols 0..r-1 = s*Bo                             (and boT)
// with s = alpha / r folded into B (src/kernels/lora.cu:190-198).
//
// lora_grad computes C[a, b] = scale * sum_m U[m, a] * W[m, b] (b < 16) for a
// batch of problems -- the reference's matmul_tn + scale_add
// (src/kernels/lora_backward.cu:50-90, src/kernels/matmul.cu:102-139):
//   dB = s * dY^T h     (a over d_out, b over r)
//   dA = dh^T x         (computed as (x^T dh)^T: a over d_in, b over r)
// split over m, mma.sync m16n8k16, partials reduced in a fixed order.
#include "common.cuh"
#include "lora.cuh"

namespace llmcu {

namespace {

__global__ void lora_prep_kernel(const float* __restrict__ flat, LoraDims d, __half* __restrict__ derived) {
  const int l = blockIdx.y;
  const float* P = flat + static_cast<int64_t>(l) * d.per_layer;
  __half* D = derived + static_cast<int64_t>(l) * d.derived_per_layer;
  const int r = d.r, H = d.H, Q = d.Q, KV = d.KV, QKV = Q + 2 * KV;
  const float s = d.scale;
  const int64_t n_acat = 64LL * H, n_bblk = 64LL * QKV, n_ao = 64LL * Q, n_bo = 64LL * H;
  const int64_t total = n_acat + n_bblk + n_ao + n_bo;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    int64_t k = i;
    if (k < n_acat) {  // acat[j, c]
      const int j = static_cast<int>(k / H), c = static_cast<int>(k % H);
      float v = 0.f;
      if (j < r) v = P[d.oAq + j * H + c];
      else if (j >= kSegK && j < kSegK + r) v = P[d.oAk + (j - kSegK) * H + c];
      else if (j >= kSegV && j < kSegV + r) v = P[d.oAv + (j - kSegV) * H + c];
      const __half hv = __float2half_rn(v);
      D[d.d_acat + k] = hv;
      D[d.d_acatT + static_cast<int64_t>(c) * 64 + j] = hv;
      continue;
    }
    k -= n_acat;
    if (k < n_bblk) {  // bblk[n, j]
      const int n = static_cast<int>(k / 64), j = static_cast<int>(k % 64);
      float v = 0.f;
      if (n < Q) {
        if (j < r) v = s * P[d.oBq + n * r + j];
      } else if (n < Q + KV) {
        if (j >= kSegK && j < kSegK + r) v = s * P[d.oBk + (n - Q) * r + (j - kSegK)];
      } else {
        if (j >= kSegV && j < kSegV + r) v = s * P[d.oBv + (n - Q - KV) * r + (j - kSegV)];
      }
      const __half hv = __float2half_rn(v);
      D[d.d_bblk + k] = hv;
      D[d.d_bblkT + static_cast<int64_t>(j) * QKV + n] = hv;
      continue;
    }
    k -= n_bblk;
    if (k < n_ao) {  // ao[j, c]
      const int j = static_cast<int>(k / Q), c = static_cast<int>(k % Q);
      const float v = j < r ? P[d.oAo + j * Q + c] : 0.f;
      const __half hv = __float2half_rn(v);
      D[d.d_ao + k] = hv;
      D[d.d_aoT + static_cast<int64_t>(c) * 64 + j] = hv;
      continue;
    }
    k -= n_ao;
    {  // bo[h, j]
      const int h = static_cast<int>(k / 64), j = static_cast<int>(k % 64);
      const float v = j < r ? s * P[d.oBo + h * r + j] : 0.f;
      const __half hv = __float2half_rn(v);
      D[d.d_bo + k] = hv;
      D[d.d_boT + static_cast<int64_t>(j) * H + h] = hv;
    }
  }
}

constexpr int kLgThreads = 128;
constexpr int kLgA = 64;   // a-rows per CTA (4 warps x 16)
constexpr int kLgM = 64;   // m per smem stage

__device__ __forceinline__ uint32_t uoff(int m, int c) {  // [64 m][64 cols] tile, 8 chunks per row
  return static_cast<uint32_t>((m * 8 + (c ^ (m & 7))) * 16);
}

__global__ void __launch_bounds__(kLgThreads) lora_grad_kernel(const LoraGradBatch batch, int M, int splits,
                                                              float* __restrict__ part) {
  __shared__ __align__(128) uint8_t su[2][kLgM * kLgA * 2];
  __shared__ __align__(128) uint8_t sw[2][kLgM * 64 * 2];
  const LoraGradProb& pb = batch.p[blockIdx.y];
  const int a0 = blockIdx.x * kLgA;
  if (a0 >= pb.A) return;
  const int split = blockIdx.z;
  const int m_per = ((M + splits - 1) / splits + kLgM - 1) / kLgM * kLgM;
  const int m_begin = split * m_per;
  const int m_end = min(M, m_begin + m_per);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ng = pb.groups;

  auto load = [&](int buf, int m0) {
    const uint32_t su_b = smem_u32(su[buf]);
    const uint32_t sw_b = smem_u32(sw[buf]);
    for (int i = threadIdx.x; i < kLgM * 8; i += kLgThreads) {
      const int mm = i >> 3, c = i & 7;
      const int m = m0 + mm;
      const bool ok = m < m_end && (a0 + c * 8) < pb.A;
      const __half* src = pb.U + static_cast<size_t>(ok ? m : m_begin) * pb.ldu + (ok ? a0 + c * 8 : 0);
      cp_async_16(su_b + uoff(mm, c), src, ok ? 16 : 0);
      const bool okw = m < m_end && c < 2 * ng;
      const __half* srcw = pb.W + static_cast<size_t>(okw ? m : m_begin) * pb.ldw + (okw ? c * 8 : 0);
      cp_async_16(sw_b + uoff(mm, c), srcw, okw ? 16 : 0);
    }
  };

  float acc[8][4];
#pragma unroll
  for (int n = 0; n < 8; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.f;
  const int nsteps = m_end > m_begin ? (m_end - m_begin + kLgM - 1) / kLgM : 0;
  if (nsteps > 0) load(0, m_begin);
  cp_async_commit();
  for (int s = 0; s < nsteps; ++s) {
    const int buf = s & 1;
    if (s + 1 < nsteps) load(buf ^ 1, m_begin + (s + 1) * kLgM);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    const uint32_t su_b = smem_u32(su[buf]);
    const uint32_t sw_b = smem_u32(sw[buf]);
#pragma unroll
    for (int kk = 0; kk < kLgM / 16; ++kk) {
      const int mi = lane >> 3;
      uint32_t a[4];
      ldmatrix_x4_trans(su_b + uoff(kk * 16 + (mi >> 1) * 8 + (lane & 7), warp * 2 + (mi & 1)), a[0], a[1], a[2],
                        a[3]);
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        if (g < ng) {
          uint32_t b0, b1, b2, b3;
          ldmatrix_x4_trans(sw_b + uoff(kk * 16 + (mi & 1) * 8 + (lane & 7), 2 * g + (mi >> 1)), b0, b1, b2, b3);
          mma_16816(acc[2 * g], a, b0, b1);
          mma_16816(acc[2 * g + 1], a, b2, b3);
        }
      }
    }
    __syncthreads();
  }
  cp_async_wait<0>();

  // partial tile [64 a][64 b] for (split, problem, a-block)
  const int gq = lane >> 2, t = lane & 3;
  float* pp = part + ((static_cast<size_t>(split) * batch.n + blockIdx.y) * batch.a_max + a0) * 64;
#pragma unroll
  for (int n = 0; n < 8; ++n) {
    if (n < 2 * ng) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int a = warp * 16 + gq + (e >> 1) * 8;
        const int b = n * 8 + 2 * t + (e & 1);
        pp[a * 64 + b] = acc[n][e];
      }
    }
  }
}

__global__ void lora_grad_reduce_kernel(const LoraGradBatch batch, int splits, const float* __restrict__ part) {
  const LoraGradProb& pb = batch.p[blockIdx.y];
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;  // a * 64 + (16 g + b)
  const int a = idx >> 6, gb = idx & 63, g = gb >> 4, b = gb & 15;
  if (a >= pb.A || g >= pb.groups || b >= pb.Bn) return;
  float s = 0.f;
  for (int sp = 0; sp < splits; ++sp)
    s += part[((static_cast<size_t>(sp) * batch.n + blockIdx.y) * batch.a_max + a) * 64 + gb];
  pb.out[g][static_cast<size_t>(a) * pb.sa + static_cast<size_t>(b) * pb.sb] = s * pb.scale;
}

}  // namespace

cudaError_t lora_prep(const float* flat, const LoraDims& d, int n_layers, __half* derived, cudaStream_t st) {
  const int64_t total = 64LL * (2 * d.H + d.Q + 2 * d.KV + d.Q);
  int gx = static_cast<int>((total + 255) / 256);
  if (gx > 512) gx = 512;
  dim3 grid(gx, n_layers);
  lora_prep_kernel<<<grid, 256, 0, st>>>(flat, d, derived);
  return cudaGetLastError();
}

int lora_grad_splits(int M, int a_max, int n) {
  const int tiles = (a_max + kLgA - 1) / kLgA * n;
  int s = (2 * gemm_num_sms() + tiles - 1) / tiles;
  const int max_s = (M + 255) / 256;
  if (s > max_s) s = max_s;
  if (s > kLoraMaxSplits) s = kLoraMaxSplits;
  if (s < 1) s = 1;
  return s;
}

cudaError_t lora_grad(const LoraGradBatch& batch, int M, float* part, cudaStream_t st) {
  if (batch.n <= 0 || batch.n > kLoraMaxProbs) return cudaErrorInvalidValue;
  const int splits = lora_grad_splits(M, batch.a_max, batch.n);
  dim3 grid((batch.a_max + kLgA - 1) / kLgA, batch.n, splits);
  lora_grad_kernel<<<grid, kLgThreads, 0, st>>>(batch, M, splits, part);
  dim3 g2((batch.a_max * 64 + 255) / 256, batch.n);
  lora_grad_reduce_kernel<<<g2, 256, 0, st>>>(batch, splits, part);
  return cudaGetLastError();
}

}  // namespace llmcu
