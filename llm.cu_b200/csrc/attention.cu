// attention.cu -- causal GQA flash attention, forward and backward.
//
// Replaces the reference's naive_attn_kernel (which writes the full
// probability tensor P [nh, S, S] to HBM, src/kernels/lora_forward.cu:48-135)
// and attn_backward_kernel + expand/contract (global atomics into expanded
// K/V gradients, src/kernels/lora_backward.cu:104-208).
//
//   forward : O = softmax(scale * Q K^T, causal) V, plus the per-row
//             log-sum-exp; P never leaves registers.
//   backward: recomputes P per tile from Q, K and the LSE.
//             delta = rowsum(dO * O); dK/dV for a KV head accumulate all Q
//             heads of its group inside one CTA (no expansion, no atomics);
//             dQ comes from a second kernel, so every reduction is a plain
//             register accumulation and the result is deterministic.
//
// Tiles: 64 query rows x 64 key rows, 4 warps x 16 rows, fp16 operands in
// XOR-swizzled shared memory fed by cp.async, mma.sync m16n8k16 with fp32
// accumulation.  head_dim 64 and 128.
#include <mutex>

#include "../../include/llmcu.h"
#include "common.cuh"

namespace llmcu {

namespace {

constexpr int kBQ = 64;   // query rows per tile
constexpr int kBK = 64;   // key rows per tile
constexpr int kAttnThreads = 128;

// byte offset of 16-byte chunk `c` of row `r` in a [rows][HD] fp16 tile
template <int HD>
__device__ __forceinline__ uint32_t toff(int r, int c) {
  constexpr int kCPR = HD / 8;
  return static_cast<uint32_t>((r * kCPR + (c ^ (r & 7))) * 16);
}

// rows [r0, r0+ROWS) of a row-major fp16 matrix (row stride ld elements,
// already offset to the head's first column) -> swizzled smem tile; rows
// >= rmax are zero-filled.
template <int HD, int ROWS>
__device__ __forceinline__ void load_tile(uint32_t sbase, const __half* g, int ld, int r0, int rmax) {
  constexpr int kCPR = HD / 8;
  for (int i = threadIdx.x; i < ROWS * kCPR; i += kAttnThreads) {
    const int r = i / kCPR, c = i % kCPR;
    const int gr = r0 + r;
    const int cr = gr < rmax ? gr : (rmax > 0 ? rmax - 1 : 0);
    cp_async_16(sbase + toff<HD>(r, c), g + static_cast<size_t>(cr) * ld + c * 8, gr < rmax ? 16 : 0);
  }
}

// A fragment (16x16, rows r0.., k-step kk) from a [rows][HD] tile
template <int HD>
__device__ __forceinline__ void lda_frag(uint32_t sbase, int r0, int kk, uint32_t (&a)[4]) {
  const int l = threadIdx.x & 31;
  const int r = r0 + (l & 7) + ((l >> 3) & 1) * 8;
  const int c = kk * 2 + (l >> 4);
  ldmatrix_x4(sbase + toff<HD>(r, c), a[0], a[1], a[2], a[3]);
}

// B fragments for n-tiles (n0, n0+1) at k-step kk, tile stored [n][k]
template <int HD>
__device__ __forceinline__ void ldb_nk(uint32_t sbase, int n0, int kk, uint32_t& b0, uint32_t& b1,
                                       uint32_t& b2, uint32_t& b3) {
  const int l = threadIdx.x & 31;
  const int m = l >> 3;
  const int r = n0 * 8 + (m >> 1) * 8 + (l & 7);
  const int c = kk * 2 + (m & 1);
  ldmatrix_x4(sbase + toff<HD>(r, c), b0, b1, b2, b3);
}

// B fragments for n-tiles (nd, nd+1) at k-step j, tile stored [k][n]
template <int HD>
__device__ __forceinline__ void ldb_kn(uint32_t sbase, int nd, int j, uint32_t& b0, uint32_t& b1,
                                       uint32_t& b2, uint32_t& b3) {
  const int l = threadIdx.x & 31;
  const int m = l >> 3;
  const int r = j * 16 + (m & 1) * 8 + (l & 7);
  const int c = nd + (m >> 1);
  ldmatrix_x4_trans(sbase + toff<HD>(r, c), b0, b1, b2, b3);
}

// ---------------------------------------------------------------- forward
template <int HD>
__global__ void __launch_bounds__(kAttnThreads)
    attn_fwd_kernel(const __half* __restrict__ q, const __half* __restrict__ k, const __half* __restrict__ v,
                    __half* __restrict__ o, float* __restrict__ lse, int S, int nh, int nkv, int ldq, int ldk,
                    int ldv, int ldo, float scale_log2) {
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr int kTile = kBQ * HD * 2;
  const uint32_t sQ = smem_u32(smem);
  const uint32_t sK0 = sQ + kTile;
  const uint32_t sV0 = sK0 + 2 * kTile;

  const int qb = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int kvh = h / (nh / nkv);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;

  const __half* qg = q + static_cast<size_t>(b) * S * ldq + h * HD;
  const __half* kg = k + static_cast<size_t>(b) * S * ldk + kvh * HD;
  const __half* vg = v + static_cast<size_t>(b) * S * ldv + kvh * HD;

  load_tile<HD, kBQ>(sQ, qg, ldq, qb * kBQ, S);
  load_tile<HD, kBK>(sK0, kg, ldk, 0, S);
  load_tile<HD, kBK>(sV0, vg, ldv, 0, S);
  cp_async_commit();

  float acc[HD / 8][4];
#pragma unroll
  for (int i = 0; i < HD / 8; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
  float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};
  uint32_t qf[HD / 16][4];

  const int q_lo = qb * kBQ + warp * 16 + g;  // rows q_lo and q_lo + 8
  const int nkb = qb + 1;                      // causal: key blocks 0..qb
  for (int kb = 0; kb < nkb; ++kb) {
    const int buf = kb & 1;
    if (kb + 1 < nkb) {
      load_tile<HD, kBK>(sK0 + (buf ^ 1) * kTile, kg, ldk, (kb + 1) * kBK, S);
      load_tile<HD, kBK>(sV0 + (buf ^ 1) * kTile, vg, ldv, (kb + 1) * kBK, S);
    }
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    if (kb == 0) {
#pragma unroll
      for (int kk = 0; kk < HD / 16; ++kk) lda_frag<HD>(sQ, warp * 16, kk, qf[kk]);
    }
    const uint32_t sK = sK0 + buf * kTile, sV = sV0 + buf * kTile;

    float s[kBK / 8][4];
#pragma unroll
    for (int n = 0; n < kBK / 8; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < HD / 16; ++kk) {
#pragma unroll
      for (int n = 0; n < kBK / 8; n += 2) {
        uint32_t b0, b1, b2, b3;
        ldb_nk<HD>(sK, n, kk, b0, b1, b2, b3);
        mma_16816(s[n], qf[kk], b0, b1);
        mma_16816(s[n + 1], qf[kk], b2, b3);
      }
    }
    // scale, mask, online softmax
    float mnew[2] = {mrow[0], mrow[1]};
#pragma unroll
    for (int n = 0; n < kBK / 8; ++n) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int qi = q_lo + (e >> 1) * 8;
        const int ki = kb * kBK + n * 8 + 2 * t + (e & 1);
        float x = s[n][e] * scale_log2;
        if (ki > qi || ki >= S) x = -INFINITY;
        s[n][e] = x;
        mnew[e >> 1] = fmaxf(mnew[e >> 1], x);
      }
    }
    float corr[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mnew[r] = fmaxf(mnew[r], __shfl_xor_sync(0xffffffffu, mnew[r], 1));
      mnew[r] = fmaxf(mnew[r], __shfl_xor_sync(0xffffffffu, mnew[r], 2));
      corr[r] = (mnew[r] == -INFINITY) ? 1.f : fast_exp2(mrow[r] - mnew[r]);
      mrow[r] = mnew[r];
      lrow[r] *= corr[r];
    }
    float psum[2] = {0.f, 0.f};
#pragma unroll
    for (int n = 0; n < kBK / 8; ++n) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float m = mrow[e >> 1];
        const float p = (m == -INFINITY) ? 0.f : fast_exp2(s[n][e] - m);
        s[n][e] = p;
        psum[e >> 1] += p;
      }
    }
    lrow[0] += psum[0];
    lrow[1] += psum[1];
#pragma unroll
    for (int i = 0; i < HD / 8; ++i) {
      acc[i][0] *= corr[0]; acc[i][1] *= corr[0];
      acc[i][2] *= corr[1]; acc[i][3] *= corr[1];
    }
    // O += P V
#pragma unroll
    for (int j = 0; j < kBK / 16; ++j) {
      uint32_t a[4];
      a[0] = pack_half2(s[2 * j][0], s[2 * j][1]);
      a[1] = pack_half2(s[2 * j][2], s[2 * j][3]);
      a[2] = pack_half2(s[2 * j + 1][0], s[2 * j + 1][1]);
      a[3] = pack_half2(s[2 * j + 1][2], s[2 * j + 1][3]);
#pragma unroll
      for (int nd = 0; nd < HD / 8; nd += 2) {
        uint32_t b0, b1, b2, b3;
        ldb_kn<HD>(sV, nd, j, b0, b1, b2, b3);
        mma_16816(acc[nd], a, b0, b1);
        mma_16816(acc[nd + 1], a, b2, b3);
      }
    }
    __syncthreads();
  }
  cp_async_wait<0>();

  // finalise rows: the quad owns the row; full row sum by quad reduction
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    lrow[r] += __shfl_xor_sync(0xffffffffu, lrow[r], 1);
    lrow[r] += __shfl_xor_sync(0xffffffffu, lrow[r], 2);
  }
  const size_t obase = static_cast<size_t>(b) * S * ldo + h * HD;
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int qi = q_lo + r * 8;
    if (qi >= S) continue;
    const float inv = lrow[r] > 0.f ? 1.f / lrow[r] : 0.f;
    __half* orow = o + obase + static_cast<size_t>(qi) * ldo;
#pragma unroll
    for (int i = 0; i < HD / 8; ++i) {
      *reinterpret_cast<uint32_t*>(orow + i * 8 + 2 * t) = pack_half2(acc[i][2 * r] * inv, acc[i][2 * r + 1] * inv);
    }
    if (t == 0) lse[(static_cast<size_t>(b) * nh + h) * S + qi] = (mrow[r] + __log2f(lrow[r])) * 0.69314718055994531f;
  }
}

// delta[b, h, s] = sum_d dO * O  (fp32), one warp per (row, head)
template <int HD>
__global__ void attn_delta_kernel(const __half* __restrict__ o, const __half* __restrict__ dout,
                                  float* __restrict__ delta, int B, int S, int nh, int ld) {
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

// ---------------------------------------------------------------- dK / dV
// One CTA per (key block, KV head, batch); loops over the Q heads of the
// group and the query blocks at or after the key block.
template <int HD>
__global__ void __launch_bounds__(kAttnThreads)
    attn_bwd_dkdv_kernel(const __half* __restrict__ q, const __half* __restrict__ k, const __half* __restrict__ v,
                         const __half* __restrict__ dout, const float* __restrict__ lse,
                         const float* __restrict__ delta, float* __restrict__ dk, __half* __restrict__ dv, int S,
                         int nh, int nkv, int ldq, int ldk, int ldv, int ldo, int lddk, int lddv, float scale,
                         float scale_log2) {
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr int kTile = kBQ * HD * 2;
  const uint32_t sK = smem_u32(smem);
  const uint32_t sV = sK + kTile;
  const uint32_t sQ0 = sV + kTile;          // 2 buffers
  const uint32_t sO0 = sQ0 + 2 * kTile;     // 2 buffers (dO)
  float* sL = reinterpret_cast<float*>(smem + 6 * kTile);  // [2][kBQ] lse*log2e
  float* sD = sL + 2 * kBQ;                                 // [2][kBQ] delta

  const int kb = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int G = nh / nkv;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int nqb = (S + kBQ - 1) / kBQ;

  const __half* kg = k + static_cast<size_t>(b) * S * ldk + kvh * HD;
  const __half* vg = v + static_cast<size_t>(b) * S * ldv + kvh * HD;
  load_tile<HD, kBK>(sK, kg, ldk, kb * kBK, S);
  load_tile<HD, kBK>(sV, vg, ldv, kb * kBK, S);

  // iteration space: (head j in group, query block qb >= kb)
  const int per_head = nqb - kb;
  const int n_it = G * per_head;
  auto issue = [&](int it, int buf) {
    const int hq = kvh * G + it / per_head;
    const int qb = kb + it % per_head;
    const __half* qg = q + static_cast<size_t>(b) * S * ldq + hq * HD;
    const __half* og = dout + static_cast<size_t>(b) * S * ldo + hq * HD;
    load_tile<HD, kBQ>(sQ0 + buf * kTile, qg, ldq, qb * kBQ, S);
    load_tile<HD, kBQ>(sO0 + buf * kTile, og, ldo, qb * kBQ, S);
    const size_t rb = (static_cast<size_t>(b) * nh + hq) * S;
    for (int i = threadIdx.x; i < kBQ; i += kAttnThreads) {
      const int qi = qb * kBQ + i;
      sL[buf * kBQ + i] = qi < S ? lse[rb + qi] * kLog2e : INFINITY;
      sD[buf * kBQ + i] = qi < S ? delta[rb + qi] : 0.f;
    }
  };
  issue(0, 0);
  cp_async_commit();

  float dka[HD / 8][4], dva[HD / 8][4];
#pragma unroll
  for (int i = 0; i < HD / 8; ++i)
#pragma unroll
    for (int e = 0; e < 4; ++e) dka[i][e] = dva[i][e] = 0.f;

  const int k_lo = kb * kBK + warp * 16 + g;  // key rows k_lo, k_lo + 8
  for (int it = 0; it < n_it; ++it) {
    const int buf = it & 1;
    if (it + 1 < n_it) issue(it + 1, buf ^ 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    const int qb = kb + it % per_head;
    const uint32_t sQ = sQ0 + buf * kTile, sO = sO0 + buf * kTile;
    const float* L = sL + buf * kBQ;
    const float* Dl = sD + buf * kBQ;

#pragma unroll
    for (int half = 0; half < 2; ++half) {       // 32 query columns at a time
      const int nbase = half * 4;                 // n-tile offset (8 cols each)
      float st[4][4], dpt[4][4];
#pragma unroll
      for (int n = 0; n < 4; ++n)
#pragma unroll
        for (int e = 0; e < 4; ++e) st[n][e] = dpt[n][e] = 0.f;
      // S^T = K Q^T and dP^T = V dO^T for this warp's 16 key rows
#pragma unroll
      for (int kk = 0; kk < HD / 16; ++kk) {
        uint32_t ak[4], av[4];
        lda_frag<HD>(sK, warp * 16, kk, ak);
        lda_frag<HD>(sV, warp * 16, kk, av);
#pragma unroll
        for (int n = 0; n < 4; n += 2) {
          uint32_t b0, b1, b2, b3;
          ldb_nk<HD>(sQ, nbase + n, kk, b0, b1, b2, b3);
          mma_16816(st[n], ak, b0, b1);
          mma_16816(st[n + 1], ak, b2, b3);
          ldb_nk<HD>(sO, nbase + n, kk, b0, b1, b2, b3);
          mma_16816(dpt[n], av, b0, b1);
          mma_16816(dpt[n + 1], av, b2, b3);
        }
      }
      // P^T and dS^T
#pragma unroll
      for (int n = 0; n < 4; ++n) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int kr = k_lo + (e >> 1) * 8;
          const int qc_local = (nbase + n) * 8 + 2 * t + (e & 1);
          const int qc = qb * kBQ + qc_local;
          float p = fast_exp2(st[n][e] * scale_log2 - L[qc_local]);
          if (qc < kr || qc >= S || kr >= S) p = 0.f;
          st[n][e] = p;
          dpt[n][e] = p * (dpt[n][e] - Dl[qc_local]);
        }
      }
      // dV += P^T dO ; dK += dS^T Q   (k-dim = these 32 query rows)
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        uint32_t ap[4], as[4];
        ap[0] = pack_half2(st[2 * j][0], st[2 * j][1]);
        ap[1] = pack_half2(st[2 * j][2], st[2 * j][3]);
        ap[2] = pack_half2(st[2 * j + 1][0], st[2 * j + 1][1]);
        ap[3] = pack_half2(st[2 * j + 1][2], st[2 * j + 1][3]);
        as[0] = pack_half2(dpt[2 * j][0], dpt[2 * j][1]);
        as[1] = pack_half2(dpt[2 * j][2], dpt[2 * j][3]);
        as[2] = pack_half2(dpt[2 * j + 1][0], dpt[2 * j + 1][1]);
        as[3] = pack_half2(dpt[2 * j + 1][2], dpt[2 * j + 1][3]);
        const int jj = half * 2 + j;  // 16-row k-step within the 64-row query tile
#pragma unroll
        for (int nd = 0; nd < HD / 8; nd += 2) {
          uint32_t b0, b1, b2, b3;
          ldb_kn<HD>(sO, nd, jj, b0, b1, b2, b3);
          mma_16816(dva[nd], ap, b0, b1);
          mma_16816(dva[nd + 1], ap, b2, b3);
          ldb_kn<HD>(sQ, nd, jj, b0, b1, b2, b3);
          mma_16816(dka[nd], as, b0, b1);
          mma_16816(dka[nd + 1], as, b2, b3);
        }
      }
    }
    __syncthreads();
  }
  cp_async_wait<0>();

#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int kr = k_lo + r * 8;
    if (kr >= S) continue;
    float* dkrow = dk + (static_cast<size_t>(b) * S + kr) * lddk + kvh * HD;
    __half* dvrow = dv + (static_cast<size_t>(b) * S + kr) * lddv + kvh * HD;
#pragma unroll
    for (int i = 0; i < HD / 8; ++i) {
      *reinterpret_cast<float2*>(dkrow + i * 8 + 2 * t) = make_float2(dka[i][2 * r] * scale, dka[i][2 * r + 1] * scale);
      *reinterpret_cast<uint32_t*>(dvrow + i * 8 + 2 * t) = pack_half2(dva[i][2 * r], dva[i][2 * r + 1]);
    }
  }
}

// -------------------------------------------------------------------- dQ
template <int HD>
__global__ void __launch_bounds__(kAttnThreads)
    attn_bwd_dq_kernel(const __half* __restrict__ q, const __half* __restrict__ k, const __half* __restrict__ v,
                       const __half* __restrict__ dout, const float* __restrict__ lse,
                       const float* __restrict__ delta, float* __restrict__ dq, int S, int nh, int nkv, int ldq,
                       int ldk, int ldv, int ldo, int lddq, float scale, float scale_log2) {
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr int kTile = kBQ * HD * 2;
  const uint32_t sQ = smem_u32(smem);
  const uint32_t sO = sQ + kTile;
  const uint32_t sK0 = sO + kTile;       // 2 buffers
  const uint32_t sV0 = sK0 + 2 * kTile;  // 2 buffers

  const int qb = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int kvh = h / (nh / nkv);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;

  const __half* qg = q + static_cast<size_t>(b) * S * ldq + h * HD;
  const __half* og = dout + static_cast<size_t>(b) * S * ldo + h * HD;
  const __half* kg = k + static_cast<size_t>(b) * S * ldk + kvh * HD;
  const __half* vg = v + static_cast<size_t>(b) * S * ldv + kvh * HD;
  load_tile<HD, kBQ>(sQ, qg, ldq, qb * kBQ, S);
  load_tile<HD, kBQ>(sO, og, ldo, qb * kBQ, S);
  load_tile<HD, kBK>(sK0, kg, ldk, 0, S);
  load_tile<HD, kBK>(sV0, vg, ldv, 0, S);
  cp_async_commit();

  const int q_lo = qb * kBQ + warp * 16 + g;
  const size_t rb = (static_cast<size_t>(b) * nh + h) * S;
  float Lr[2], Dr[2];
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int qi = q_lo + r * 8;
    Lr[r] = qi < S ? lse[rb + qi] * kLog2e : INFINITY;
    Dr[r] = qi < S ? delta[rb + qi] : 0.f;
  }

  float dqa[HD / 8][4];
#pragma unroll
  for (int i = 0; i < HD / 8; ++i) dqa[i][0] = dqa[i][1] = dqa[i][2] = dqa[i][3] = 0.f;
  uint32_t qf[HD / 16][4], of[HD / 16][4];

  const int nkb = qb + 1;
  for (int kb = 0; kb < nkb; ++kb) {
    const int buf = kb & 1;
    if (kb + 1 < nkb) {
      load_tile<HD, kBK>(sK0 + (buf ^ 1) * kTile, kg, ldk, (kb + 1) * kBK, S);
      load_tile<HD, kBK>(sV0 + (buf ^ 1) * kTile, vg, ldv, (kb + 1) * kBK, S);
    }
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    if (kb == 0) {
#pragma unroll
      for (int kk = 0; kk < HD / 16; ++kk) {
        lda_frag<HD>(sQ, warp * 16, kk, qf[kk]);
        lda_frag<HD>(sO, warp * 16, kk, of[kk]);
      }
    }
    const uint32_t sK = sK0 + buf * kTile, sV = sV0 + buf * kTile;
#pragma unroll
    for (int half = 0; half < 2; ++half) {  // 32 key columns at a time
      const int nbase = half * 4;
      float s[4][4], dp[4][4];
#pragma unroll
      for (int n = 0; n < 4; ++n)
#pragma unroll
        for (int e = 0; e < 4; ++e) s[n][e] = dp[n][e] = 0.f;
#pragma unroll
      for (int kk = 0; kk < HD / 16; ++kk) {
#pragma unroll
        for (int n = 0; n < 4; n += 2) {
          uint32_t b0, b1, b2, b3;
          ldb_nk<HD>(sK, nbase + n, kk, b0, b1, b2, b3);
          mma_16816(s[n], qf[kk], b0, b1);
          mma_16816(s[n + 1], qf[kk], b2, b3);
          ldb_nk<HD>(sV, nbase + n, kk, b0, b1, b2, b3);
          mma_16816(dp[n], of[kk], b0, b1);
          mma_16816(dp[n + 1], of[kk], b2, b3);
        }
      }
#pragma unroll
      for (int n = 0; n < 4; ++n) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int qi = q_lo + (e >> 1) * 8;
          const int ki = kb * kBK + (nbase + n) * 8 + 2 * t + (e & 1);
          float p = fast_exp2(s[n][e] * scale_log2 - Lr[e >> 1]);
          if (ki > qi || ki >= S || qi >= S) p = 0.f;
          dp[n][e] = p * (dp[n][e] - Dr[e >> 1]);
        }
      }
      // dQ += dS K  (k-dim = these 32 key rows)
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        uint32_t as[4];
        as[0] = pack_half2(dp[2 * j][0], dp[2 * j][1]);
        as[1] = pack_half2(dp[2 * j][2], dp[2 * j][3]);
        as[2] = pack_half2(dp[2 * j + 1][0], dp[2 * j + 1][1]);
        as[3] = pack_half2(dp[2 * j + 1][2], dp[2 * j + 1][3]);
        const int jj = half * 2 + j;
#pragma unroll
        for (int nd = 0; nd < HD / 8; nd += 2) {
          uint32_t b0, b1, b2, b3;
          ldb_kn<HD>(sK, nd, jj, b0, b1, b2, b3);
          mma_16816(dqa[nd], as, b0, b1);
          mma_16816(dqa[nd + 1], as, b2, b3);
        }
      }
    }
    __syncthreads();
  }
  cp_async_wait<0>();

#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int qi = q_lo + r * 8;
    if (qi >= S) continue;
    float* row = dq + (static_cast<size_t>(b) * S + qi) * lddq + h * HD;
#pragma unroll
    for (int i = 0; i < HD / 8; ++i)
      *reinterpret_cast<float2*>(row + i * 8 + 2 * t) = make_float2(dqa[i][2 * r] * scale, dqa[i][2 * r + 1] * scale);
  }
}

template <int HD>
cudaError_t attn_fwd_launch(const __half* q, const __half* k, const __half* v, __half* o, float* lse, int B,
                            int S, int nh, int nkv, int ldq, int ldk, int ldv, int ldo, cudaStream_t st) {
  const size_t smem = 5 * kBQ * HD * 2;
  auto kern = attn_fwd_kernel<HD>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  dim3 grid((S + kBQ - 1) / kBQ, nh, B);
  const float scale = 1.0f / sqrtf(static_cast<float>(HD));
  kern<<<grid, kAttnThreads, smem, st>>>(q, k, v, o, lse, S, nh, nkv, ldq, ldk, ldv, ldo, scale * kLog2e);
  return cudaGetLastError();
}

template <int HD>
cudaError_t attn_bwd_launch(const __half* q, const __half* k, const __half* v, const __half* o, const __half* dout,
                            const float* lse, float* delta, float* dq, float* dk, __half* dv, int B, int S, int nh,
                            int nkv, int ldq, int ldk, int ldv, int ldo, int lddq, int lddk, int lddv,
                            cudaStream_t st) {
  const float scale = 1.0f / sqrtf(static_cast<float>(HD));
  {
    const int warps = B * S * nh;
    attn_delta_kernel<HD><<<(warps + 7) / 8, 256, 0, st>>>(o, dout, delta, B, S, nh, ldo);
  }
  {
    const size_t smem = 6 * kBQ * HD * 2 + 4 * kBQ * sizeof(float);
    auto kern = attn_bwd_dkdv_kernel<HD>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    dim3 grid((S + kBK - 1) / kBK, nkv, B);
    kern<<<grid, kAttnThreads, smem, st>>>(q, k, v, dout, lse, delta, dk, dv, S, nh, nkv, ldq, ldk, ldv, ldo, lddk,
                                           lddv, scale, scale * kLog2e);
  }
  {
    const size_t smem = 6 * kBQ * HD * 2;
    auto kern = attn_bwd_dq_kernel<HD>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    dim3 grid((S + kBQ - 1) / kBQ, nh, B);
    kern<<<grid, kAttnThreads, smem, st>>>(q, k, v, dout, lse, delta, dq, S, nh, nkv, ldq, ldk, ldv, ldo, lddq, scale,
                                           scale * kLog2e);
  }
  return cudaGetLastError();
}

}  // namespace

cudaError_t attention_forward(const __half* q, const __half* k, const __half* v, __half* o, float* lse, int B, int S,
                              int nh, int nkv, int hd, int ldq, int ldk, int ldv, int ldo, int* err, cudaStream_t st) {
  return attention_forward_tc(q, k, v, o, lse, B, S, nh, nkv, hd, ldq, ldk, ldv, ldo, err, st);
}

cudaError_t attention_backward(const __half* q, const __half* k, const __half* v, const __half* o,
                               const __half* dout, const float* lse, float* delta, float* dq, float* dk, __half* dv,
                               int B, int S, int nh, int nkv, int hd, int ldq, int ldk, int ldv, int ldo, int lddq,
                               int lddk, int lddv, cudaStream_t st) {
  if (hd == 128)
    return attn_bwd_launch<128>(q, k, v, o, dout, lse, delta, dq, dk, dv, B, S, nh, nkv, ldq, ldk, ldv, ldo, lddq,
                                lddk, lddv, st);
  if (hd == 64)
    return attn_bwd_launch<64>(q, k, v, o, dout, lse, delta, dq, dk, dv, B, S, nh, nkv, ldq, ldk, ldv, ldo, lddq,
                               lddk, lddv, st);
  return cudaErrorInvalidValue;
}

}  // namespace llmcu

namespace llmcu {

// ------------------------------------------- allocation-free backward variant
// File-scope scratch for the row-wise dO.O sums of llmcu_attention_bwd_noalloc.
// Every device that loads this library holds it (4 MiB) until the process
// exits.  In host code the name is only a stand-in; the device address comes
// from cudaGetSymbolAddress, looked up once per device with that device current.
namespace {
constexpr int64_t kNoAllocDeltaFloats = 1 << 20;  // batch * n_heads * seq <= 1,048,576
__device__ __align__(256) float g_noalloc_delta[kNoAllocDeltaFloats];
constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
float* g_noalloc_ptr[kMaxDevices] = {};

cudaError_t noalloc_scratch(float** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_delta);
    if (e != cudaSuccess) return e;
    g_noalloc_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_noalloc_ptr[dev];
  return cudaSuccess;
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
  if (noalloc_scratch(&delta) != cudaSuccess) return LLMCU_ERR_CUDA;
  const int ldo = n_heads * head_dim;
  const cudaError_t e = attention_backward(
      static_cast<const __half*>(q), static_cast<const __half*>(k), static_cast<const __half*>(v),
      static_cast<const __half*>(o), static_cast<const __half*>(dout), lse, delta, dq, dk, static_cast<__half*>(dv),
      batch, seq, n_heads, n_kv_heads, head_dim, ldq, ldk, ldv, ldo, ldo, n_kv_heads * head_dim, lddv,
      static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? LLMCU_OK : LLMCU_ERR_CUDA;
}
