// lora.cu -- LoRA operand preparation and the adapter-gradient kernel.
//
// Adapters live in one flat fp32 buffer (per layer: the enabled ones of
// Aq Bq Ak Bk Av Bv Ao Bo Agate Bgate Aup Bup Adown Bdown, A [r, d_in],
// B [d_out, r] as include/lora.h:13-20 of the reference), so AdamW and the
// data-parallel allreduce each touch one contiguous range.
//
// lora_merge builds, per layer and per step, the merged fp16 weights the
// tcgen05 GEMMs use in place of the reference's separate LoRA products
// (src/kernels/lora.cu:181-202: y += s (x A^T) B^T, s = alpha / r):
//   mqkv [QKV + 64, H + 64]  rows < QKV:   W_qkv + s B_p A_p (p = q, k, v by row)
//                            cols H + seg(p) + j:   s B_p[:, j]
//                            rows QKV + seg(p) + j: A_p[j, :]
//   mo   [H + 64, Q + 64]    rows < H: W_o + s B_o A_o; cols Q + j: s B_o[:, j];
//                            rows H + j: A_o[j, :]
//   mgu  [2I + 64, H + 64]   (MLP targets) the 128-row gate/up interleave of
//                            the base: gate rows W_g + s B_g A_g, cols H + j:
//                            s B_g; up rows likewise with seg 16; rows 2I +
//                            seg + j: A_g / A_u
//   md   [H + 64, I + 64]    (MLP targets) as mo for the down projection
// seg(q, k, v) = 0, 16, 32 (kSegK, kSegV), seg(gate, up) = 0, 16; everything
// else in the pads is 0, and so is the s B A of an adapter that is not
// trained (its rows are the base weight).
// The forward GEMM x . mqkv^T (K-major, N = QKV + 64) then yields q, k, v and,
// in its last 64 columns, h = x [Aq | Ak | Av]^T; the input-gradient GEMM
// dY . mqkv (MN-major, N = H + 64) yields dx and dh = dY [s Bq | s Bk | s Bv].
//
// lora_grad computes C[a, b] = scale * sum_m U[m, a] * W[m, b] (b < 16) for a
// batch of problems -- the reference's matmul_tn + scale_add
// (src/kernels/lora_backward.cu:50-90, src/kernels/matmul.cu:102-139):
//   dB = s * dY^T h     (a over d_out, b over r)
//   dA = dh^T x         (computed as (x^T dh)^T: a over d_in, b over r)
// on the tensor cores, split over m; the splits' fp32 partials are summed
// in split order by a second small kernel, so the gradients are the same bits
// from run to run.
#include "common.cuh"
#include "lora.cuh"

namespace llmcu {

namespace {

// Main block of one merged weight: `tiles` row tiles of 64 rows, columns
// [c0, c0 + 256) of W + s B A for one adapter (A [r, d_in], B [rows_p, r]).
// Base W is fp16 (w) or INT8 rows (q) times the per-row scale (s), as the
// reference's quantiser lays them out (src/kernels/quantize.cu:8-50).
using MergeSrc = MergeBase;

// Which adapter owns merged main-block row o, and its row in that adapter's
// B: which = 0 q/k/v (stacked), 1 o, 2 gate/up (128-row interleave, gate
// first), 3 down.
__device__ __forceinline__ void merge_row(const LoraDims& d, int which, int o, int& proj, int& arow) {
  if (which == 0) {
    if (o < d.Q) {
      proj = kPQ; arow = o;
    } else if (o < d.Q + d.KV) {
      proj = kPK; arow = o - d.Q;
    } else {
      proj = kPV; arow = o - d.Q - d.KV;
    }
  } else if (which == 1) {
    proj = kPO; arow = o;
  } else if (which == 2) {
    proj = ((o >> 7) & 1) ? kPUp : kPGate;
    arow = ((o >> 8) << 7) + (o & 127);
  } else {
    proj = kPDown; arow = o;
  }
}
constexpr int kMrgRows = 64;   // rows of one row tile
constexpr int kMrgCols = 256;  // columns of a block
constexpr int kMrgTiles = 4;   // row tiles per block (fewer when an adapter has fewer rows)

// Base weight row o, columns [c, c + 8): fp16 bits, or INT8 codes + row scale.
struct MergeRaw {
  uint4 bits;  // 8 fp16, or 8 int8 in the low 8 bytes
  float sc;
};
__device__ __forceinline__ MergeRaw merge_load(const MergeSrc& src, int l, int o, int d_in, int c) {
  MergeRaw m;
  const int64_t off = static_cast<int64_t>(l) * src.w_layer + static_cast<int64_t>(o) * d_in + c;
  if (src.q) {
    const int2 raw = *reinterpret_cast<const int2*>(src.q + off);
    m.bits = make_uint4(static_cast<uint32_t>(raw.x), static_cast<uint32_t>(raw.y), 0u, 0u);
    m.sc = src.s[static_cast<int64_t>(l) * src.s_layer + o];
  } else {
    m.bits = *reinterpret_cast<const uint4*>(src.w + off);
    m.sc = 1.f;
  }
  return m;
}
__device__ __forceinline__ void merge_unpack(const MergeRaw& m, bool int8, float (&v)[8]) {
  if (int8) {
    const int8_t* qb = reinterpret_cast<const int8_t*>(&m.bits);
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = static_cast<float>(qb[e]) * m.sc;
  } else {
    const __half2* h = reinterpret_cast<const __half2*>(&m.bits);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __half22float2(h[e]);
      v[2 * e] = f.x;
      v[2 * e + 1] = f.y;
    }
  }
}

// 256 threads; a block covers `tiles` row tiles of 64 rows (one adapter) and
// 256 columns.  Thread (rg = t / 32, cg = t % 32) owns rows rg*8.. and
// columns cg*8.. of each row tile: 64 accumulators start from W and take 16
// rank-1 updates from two 8-float smem vectors (A[j, cols] and s*B[rows, j]);
// a warp's global rows are 512 contiguous bytes.  The next tile's W rows are
// loaded while the current tile is computed.
__global__ void __launch_bounds__(256, 1)
    lora_merge_main_kernel(const float* __restrict__ flat, LoraDims d, MergeSrc src, int d_in, int which, int tiles,
                           __half* __restrict__ merged, int64_t merged_layer, int ldm) {
  pdl_trigger();
  pdl_wait();
  __shared__ __align__(16) float As[16][kMrgCols];
  __shared__ __align__(16) float Bs[kMrgTiles][16][kMrgRows];  // s * B, transposed: [tile][j][row]
  const int l = blockIdx.z;
  const int ob = blockIdx.y * kMrgRows * tiles, c0 = blockIdx.x * kMrgCols;
  const float* P = flat + static_cast<int64_t>(l) * d.per_layer;
  // adapter owning rows [ob, ob + 64 * tiles) (a block never straddles two)
  int proj, arow0;
  merge_row(d, which, ob, proj, arow0);
  const bool on = d.has(proj);  // off: the rows are the base weight
  const int rg = threadIdx.x >> 5, cg = threadIdx.x & 31;
  const int c = c0 + 8 * cg;
  const bool col_ok = c < d_in;
  const bool int8 = src.q != nullptr;
  MergeRaw raw[8];
  if (col_ok) {  // first tile's W rows, in flight while the adapters are staged
#pragma unroll
    for (int i = 0; i < 8; ++i) raw[i] = merge_load(src, l, ob + 8 * rg + i, d_in, c);
  }
  const float* A = P + (on ? d.offA(proj) : 0);
  const float* Bm = P + (on ? d.offB(proj) : 0);
  const int r = on ? d.r : 0;
  for (int i = threadIdx.x; i < 16 * kMrgCols; i += 256) {
    const int j = i / kMrgCols, cc = i % kMrgCols;
    As[j][cc] = (j < r && c0 + cc < d_in) ? A[static_cast<int64_t>(j) * d_in + c0 + cc] : 0.f;
  }
  for (int i = threadIdx.x; i < tiles * 16 * kMrgRows; i += 256) {
    const int t = i / (16 * kMrgRows), rr = (i / 16) % kMrgRows, j = i % 16;
    const int ar = arow0 + t * kMrgRows + rr;
    Bs[t][j][rr] = j < r ? d.scale * Bm[static_cast<int64_t>(ar) * r + j] : 0.f;
  }
  __syncthreads();
  if (!col_ok) return;
  __half* out = merged + static_cast<int64_t>(l) * merged_layer;
  for (int t = 0; t < tiles; ++t) {
    const int o0 = ob + t * kMrgRows + 8 * rg;
    float acc[8][8];
#pragma unroll
    for (int i = 0; i < 8; ++i) merge_unpack(raw[i], int8, acc[i]);
    if (t + 1 < tiles) {  // next tile's rows load during this tile's updates
#pragma unroll
      for (int i = 0; i < 8; ++i) raw[i] = merge_load(src, l, o0 + kMrgRows + i, d_in, c);
    }
#pragma unroll 4
    for (int j = 0; j < 16; ++j) {
      const float4 a0 = *reinterpret_cast<const float4*>(&As[j][8 * cg]);
      const float4 a1 = *reinterpret_cast<const float4*>(&As[j][8 * cg + 4]);
      const float4 b0 = *reinterpret_cast<const float4*>(&Bs[t][j][8 * rg]);
      const float4 b1 = *reinterpret_cast<const float4*>(&Bs[t][j][8 * rg + 4]);
      const float a[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      const float b[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[i][e] = fmaf(b[i], a[e], acc[i][e]);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      uint4 w;
      w.x = pack_half2(acc[i][0], acc[i][1]);
      w.y = pack_half2(acc[i][2], acc[i][3]);
      w.z = pack_half2(acc[i][4], acc[i][5]);
      w.w = pack_half2(acc[i][6], acc[i][7]);
      *reinterpret_cast<uint4*>(out + static_cast<int64_t>(o0 + i) * ldm + c) = w;
    }
  }
}

// Tensor-core form of the main block for fp16 base weights: a block merges
// 64 rows x 128 columns of one adapter.  The W tile is staged in shared
// memory (16-byte cp.async, issued before the wait on the previous kernel:
// the base weights are constant), s*B [64 x 16] and A [16 x 128] are
// rounded to fp16 there, and each warp adds s*B*A to its 16 rows with one
// m16n8k16 MMA per 8 columns, the accumulator starting from W.  The merged
// tile is written back in place and stored with 16-byte coalesced stores.
constexpr int kMtRows = 64;
constexpr int kMtCols = 128;
constexpr int kMtPad = 8;  // halves of row padding: conflict-free fragment access
// Q8: the base rows are INT8 codes with per-row scales (src/kernels/quantize.cu:
// 8-50); the accumulator starts from code * scale in fp32 and sW only holds
// the merged result.
template <bool Q8>
__global__ void __launch_bounds__(128)
    lora_merge_tc_kernel(const float* __restrict__ flat, LoraDims d, MergeBase src, int d_in, int which,
                         __half* __restrict__ merged, int64_t merged_layer, int ldm) {
  pdl_trigger();
  __shared__ __align__(16) __half sW[kMtRows][kMtCols + kMtPad];
  __shared__ __align__(16) __half sB[kMtRows][16 + kMtPad];
  __shared__ __align__(16) __half sA[16][kMtCols + kMtPad];
  __shared__ __align__(16) int8_t sQ[Q8 ? kMtRows : 1][Q8 ? kMtCols + 16 : 16];
  const int l = blockIdx.z, o0 = blockIdx.y * kMtRows, c0 = blockIdx.x * kMtCols;
  if constexpr (Q8) {
    const int8_t* ql = src.q + static_cast<int64_t>(l) * src.w_layer;
    for (int i = threadIdx.x; i < kMtRows * (kMtCols / 16); i += blockDim.x) {
      const int rr = i / (kMtCols / 16), ch = i % (kMtCols / 16);
      const int c = c0 + ch * 16;
      const bool ok = c < d_in;
      cp_async_16(smem_u32(&sQ[rr][ch * 16]), ql + static_cast<int64_t>(o0 + rr) * d_in + (ok ? c : 0), ok ? 16 : 0);
    }
  } else {
    const __half* wl = src.w + static_cast<int64_t>(l) * src.w_layer;
    for (int i = threadIdx.x; i < kMtRows * (kMtCols / 8); i += blockDim.x) {
      const int rr = i / (kMtCols / 8), ch = i % (kMtCols / 8);
      const int c = c0 + ch * 8;
      const bool ok = c < d_in;
      cp_async_16(smem_u32(&sW[rr][ch * 8]), wl + static_cast<int64_t>(o0 + rr) * d_in + (ok ? c : 0), ok ? 16 : 0);
    }
  }
  cp_async_commit();
  pdl_wait();  // the adapters are written by the previous step's optimizer
  const float* P = flat + static_cast<int64_t>(l) * d.per_layer;
  int proj, arow0;
  merge_row(d, which, o0, proj, arow0);
  const bool on = d.has(proj);  // off: the rows are the base weight (s B A = 0)
  const float* A = P + (on ? d.offA(proj) : 0);
  const float* Bm = P + (on ? d.offB(proj) : 0);
  const int r = on ? d.r : 0;
  if (r == 16 && d_in % 4 == 0) {
    // every adapter load of the thread in flight at once (16-byte loads):
    // A rows [16 x 128] are 512 float4, B rows [64 x 16] are 256
    static_assert(kMtCols == 128 && kMtRows == 64, "staging below assumes a 64 x 128 block of 128 threads");
    float4 av[4], bv[2];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int i = threadIdx.x + k * 128;
      const int j = i >> 5, c = (i & 31) * 4;
      av[k] = c0 + c < d_in ? *reinterpret_cast<const float4*>(A + static_cast<int64_t>(j) * d_in + c0 + c)
                            : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int i = threadIdx.x + k * 128;
      const int rr = i >> 2, j = (i & 3) * 4;
      bv[k] = *reinterpret_cast<const float4*>(Bm + static_cast<int64_t>(arow0 + rr) * 16 + j);
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int i = threadIdx.x + k * 128;
      const int j = i >> 5, c = (i & 31) * 4;
      *reinterpret_cast<__half2*>(&sA[j][c]) = __floats2half2_rn(av[k].x, av[k].y);
      *reinterpret_cast<__half2*>(&sA[j][c + 2]) = __floats2half2_rn(av[k].z, av[k].w);
    }
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int i = threadIdx.x + k * 128;
      const int rr = i >> 2, j = (i & 3) * 4;
      *reinterpret_cast<__half2*>(&sB[rr][j]) = __floats2half2_rn(d.scale * bv[k].x, d.scale * bv[k].y);
      *reinterpret_cast<__half2*>(&sB[rr][j + 2]) = __floats2half2_rn(d.scale * bv[k].z, d.scale * bv[k].w);
    }
  } else {
    for (int i = threadIdx.x; i < kMtRows * 16; i += blockDim.x) {
      const int rr = i / 16, j = i % 16;
      sB[rr][j] = __float2half_rn(j < r ? d.scale * Bm[static_cast<int64_t>(arow0 + rr) * r + j] : 0.f);
    }
    for (int i = threadIdx.x; i < 16 * kMtCols; i += blockDim.x) {
      const int j = i / kMtCols, c = i % kMtCols;
      sA[j][c] = __float2half_rn((j < r && c0 + c < d_in) ? A[static_cast<int64_t>(j) * d_in + c0 + c] : 0.f);
    }
  }
  cp_async_wait<0>();
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int wr = warp * 16;
  float sc0 = 1.f, sc1 = 1.f;  // Q8: the scales of this thread's two fragment rows
  if constexpr (Q8) {
    const float* sl = src.s + static_cast<int64_t>(l) * src.s_layer;
    sc0 = __ldg(sl + o0 + wr + g);
    sc1 = __ldg(sl + o0 + wr + g + 8);
  }
  uint32_t a[4];
  a[0] = *reinterpret_cast<const uint32_t*>(&sB[wr + g][2 * t]);
  a[1] = *reinterpret_cast<const uint32_t*>(&sB[wr + g + 8][2 * t]);
  a[2] = *reinterpret_cast<const uint32_t*>(&sB[wr + g][8 + 2 * t]);
  a[3] = *reinterpret_cast<const uint32_t*>(&sB[wr + g + 8][8 + 2 * t]);
  // B operand (k = rank, n = column) straight from the row-major A tile:
  // one transposed ldmatrix.x4 yields the fragments of two 8-column blocks
  const int lrow = (lane & 7) + ((lane >> 3) & 1) * 8;
#pragma unroll
  for (int nb = 0; nb < kMtCols / 8; nb += 2) {
    uint32_t bf[4];
    ldmatrix_x4_trans(smem_u32(&sA[lrow][nb * 8 + (lane >> 4) * 8]), bf[0], bf[1], bf[2], bf[3]);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      __half2* p0 = reinterpret_cast<__half2*>(&sW[wr + g][(nb + h) * 8 + 2 * t]);
      __half2* p1 = reinterpret_cast<__half2*>(&sW[wr + g + 8][(nb + h) * 8 + 2 * t]);
      float2 w0, w1;
      if constexpr (Q8) {
        const int cc = (nb + h) * 8 + 2 * t;
        w0 = make_float2(static_cast<float>(sQ[wr + g][cc]) * sc0, static_cast<float>(sQ[wr + g][cc + 1]) * sc0);
        w1 = make_float2(static_cast<float>(sQ[wr + g + 8][cc]) * sc1, static_cast<float>(sQ[wr + g + 8][cc + 1]) * sc1);
      } else {
        w0 = __half22float2(*p0);
        w1 = __half22float2(*p1);
      }
      float acc[4] = {w0.x, w0.y, w1.x, w1.y};
      mma_16816(acc, a, bf[2 * h], bf[2 * h + 1]);
      *p0 = __floats2half2_rn(acc[0], acc[1]);
      *p1 = __floats2half2_rn(acc[2], acc[3]);
    }
  }
  __syncwarp();
  __half* out = merged + static_cast<int64_t>(l) * merged_layer;
  for (int i = lane; i < 16 * (kMtCols / 8); i += 32) {
    const int rr = i / (kMtCols / 8), ch = i % (kMtCols / 8);
    const int c = c0 + ch * 8;
    if (c < d_in)
      *reinterpret_cast<uint4*>(out + static_cast<int64_t>(o0 + wr + rr) * ldm + c) =
          *reinterpret_cast<const uint4*>(&sW[wr + rr][ch * 8]);
  }
}

// s * B_p[n, j] and A_p[j, c] of an adapter, 0 when p is not trained or j >= r
__device__ __forceinline__ float pad_sb(const LoraDims& d, const float* P, int p, int n, int j) {
  return (d.has(p) && j >= 0 && j < d.r) ? d.scale * P[d.offB(p) + static_cast<int64_t>(n) * d.r + j] : 0.f;
}
__device__ __forceinline__ float pad_a(const LoraDims& d, const float* P, int p, int j, int c) {
  return (d.has(p) && j >= 0 && j < d.r) ? P[d.offA(p) + static_cast<int64_t>(j) * d.d_in(p) + c] : 0.f;
}

// The pads of the attention's merged weights: the 64 extra columns (s B) of
// the rows < out_rows and the 64 extra rows (A) of the columns < d_in.
__global__ void lora_merge_pad_kernel(const float* __restrict__ flat, LoraDims d, __half* __restrict__ mqkv,
                                      int64_t mqkv_layer, __half* __restrict__ mo, int64_t mo_layer) {
  pdl_trigger();
  pdl_wait();
  const int l = blockIdx.y;
  const float* P = flat + static_cast<int64_t>(l) * d.per_layer;
  const int H = d.H, Q = d.Q, KV = d.KV, QKV = Q + 2 * KV;
  const int n_cq = 64 * QKV, n_rq = 64 * H, n_co = 64 * H, n_ro = 64 * Q;
  const int total = n_cq + n_rq + n_co + n_ro;
  __half* Mq = mqkv + static_cast<int64_t>(l) * mqkv_layer;
  __half* Mo = mo + static_cast<int64_t>(l) * mo_layer;
  const int ldq = H + 64, ldo = Q + 64;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    int k = i;
    if (k < n_cq) {  // mqkv[n, H + j] = s * B_p[n', j - seg(p)]
      const int n = k >> 6, j = k & 63;
      const float v = n < Q         ? pad_sb(d, P, kPQ, n, j)
                      : n < Q + KV  ? pad_sb(d, P, kPK, n - Q, j - kSegK)
                                    : pad_sb(d, P, kPV, n - Q - KV, j - kSegV);
      Mq[static_cast<int64_t>(n) * ldq + H + j] = __float2half_rn(v);
      continue;
    }
    k -= n_cq;
    if (k < n_rq) {  // mqkv[QKV + j, c] = A_p[j - seg(p), c]
      const int j = k / H, c = k % H;
      const float v = j < kSegK ? pad_a(d, P, kPQ, j, c) : j < kSegV ? pad_a(d, P, kPK, j - kSegK, c)
                                                                     : pad_a(d, P, kPV, j - kSegV, c);
      Mq[static_cast<int64_t>(QKV + j) * ldq + c] = __float2half_rn(v);
      continue;
    }
    k -= n_rq;
    if (k < n_co) {  // mo[n, Q + j] = s * Bo[n, j]
      const int n = k >> 6, j = k & 63;
      Mo[static_cast<int64_t>(n) * ldo + Q + j] = __float2half_rn(pad_sb(d, P, kPO, n, j));
      continue;
    }
    k -= n_co;
    {  // mo[H + j, c] = Ao[j, c]
      const int j = k / Q, c = k % Q;
      Mo[static_cast<int64_t>(H + j) * ldo + c] = __float2half_rn(pad_a(d, P, kPO, j, c));
    }
  }
}

// The pads of the MLP's merged weights: mgu columns H + j (s B_gate at seg 0,
// s B_up at seg 16, by the row's place in the interleave) and rows 2I + j
// (A_gate, A_up); md columns I + j (s B_down) and rows H + j (A_down).
__global__ void lora_merge_pad_mlp_kernel(const float* __restrict__ flat, LoraDims d, __half* __restrict__ mgu,
                                          int64_t mgu_layer, __half* __restrict__ md, int64_t md_layer) {
  pdl_trigger();
  pdl_wait();
  const int l = blockIdx.y;
  const float* P = flat + static_cast<int64_t>(l) * d.per_layer;
  const int H = d.H, I = d.I;
  const int n_cg = 64 * 2 * I, n_rg = 64 * H, n_cd = 64 * H, n_rd = 64 * I;
  const int total = n_cg + n_rg + n_cd + n_rd;
  __half* Mg = mgu + static_cast<int64_t>(l) * mgu_layer;
  __half* Md = md + static_cast<int64_t>(l) * md_layer;
  const int ldg = H + 64, ldd = I + 64;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    int k = i;
    if (k < n_cg) {
      const int n = k >> 6, j = k & 63;
      const int ar = ((n >> 8) << 7) + (n & 127);
      const float v = ((n >> 7) & 1) ? pad_sb(d, P, kPUp, ar, j - 16) : pad_sb(d, P, kPGate, ar, j);
      Mg[static_cast<int64_t>(n) * ldg + H + j] = __float2half_rn(v);
      continue;
    }
    k -= n_cg;
    if (k < n_rg) {
      const int j = k / H, c = k % H;
      const float v = j < 16 ? pad_a(d, P, kPGate, j, c) : pad_a(d, P, kPUp, j - 16, c);
      Mg[static_cast<int64_t>(2 * I + j) * ldg + c] = __float2half_rn(v);
      continue;
    }
    k -= n_rg;
    if (k < n_cd) {
      const int n = k >> 6, j = k & 63;
      Md[static_cast<int64_t>(n) * ldd + I + j] = __float2half_rn(pad_sb(d, P, kPDown, n, j));
      continue;
    }
    k -= n_cd;
    {
      const int j = k / I, c = k % I;
      Md[static_cast<int64_t>(H + j) * ldd + c] = __float2half_rn(pad_a(d, P, kPDown, j, c));
    }
  }
}

constexpr int kLgThreads = 128;  // warp 0 lane 0: TMA, warp 1 lane 0: MMA; all four drain TMEM
constexpr int kLgA = 128;         // a-rows per CTA: the UMMA M
constexpr int kLgM = 64;          // m per stage: four K = 16 UMMA steps
constexpr int kLgStages = 4;
constexpr int kLgUBytes = kLgM * kLgA * 2;  // 16 KB: two [64 m][64 a] TMA boxes
constexpr int kLgWBytes = kLgM * 64 * 2;    // 8 KB: one [64 m][64 b] TMA box
constexpr int kLgSmem = kLgStages * (kLgUBytes + kLgWBytes) + 1024 + 256;

// Stores one a-tile's final sums into the problem's gradients: acc[16 g + b]
// of a-row ar (of the tile at a0) times the problem's scale.  [a][b]
// row-major gradients (dB: sa = 16, sb = 1) are staged through shared memory
// `stage` ([128][17] floats) so that the stores leave as contiguous runs; the
// [b][a] ones (dA: sa = 1) are already contiguous across the lanes.  The
// staged case synchronises the CTA (its condition is CTA-uniform).
__device__ __forceinline__ void lg_store(const LoraGradProb& pb, int a0, int sel, int ar, const float (&acc)[64],
                                         float* stage) {
  const int ng = pb.groups;
  const int a = a0 + ar;
  const bool staged = pb.sb == 1 && pb.sa == 16 && pb.Bn == 16 && (ng == 1 || pb.ilv) && a0 + 128 <= pb.A;
  if (staged) {  // group sel's 16 columns
#pragma unroll
    for (int j = 0; j < 16; ++j) stage[ar * 17 + j] = (sel ? acc[16 + j] : acc[j]) * pb.scale;
    __syncthreads();
    float* dst = pb.out[sel] + static_cast<size_t>(pb.ilv ? ((a0 >> 8) << 7) : a0) * 16;
    for (int i = threadIdx.x; i < 128 * 16; i += blockDim.x) dst[i] = stage[(i >> 4) * 17 + (i & 15)];
  } else if (a < pb.A) {
    // gradient row of this lane's a (the interleave maps a to its adapter row)
    const int orow = pb.ilv ? ((a0 >> 8) << 7) + ar : a;
#pragma unroll
    for (int bcol = 0; bcol < 64; ++bcol) {
      const int g = bcol >> 4, b = bcol & 15;
      if (g < ng && b < pb.Bn && pb.out[g] && (!pb.ilv || g == sel))
        pb.out[g][static_cast<size_t>(orow) * pb.sa + static_cast<size_t>(b) * pb.sb] = acc[bcol] * pb.scale;
    }
  }
}

// U and W of every problem as TMA tensors ([M, A] and [M, 16 * groups]),
// 64 x 64 boxes, 128-byte swizzle
struct LoraGradMaps {
  CUtensorMap u[kLoraMaxProbs];
  CUtensorMap w[kLoraMaxProbs];
};

// One CTA: a-rows [a0, a0 + 128) of one problem over its split's m range,
// D[a, b] = sum_m U[m, a] W[m, b] on the tensor cores: U^T is the A operand
// and W the B operand, both read MN-major (a and b are the contiguous
// dimensions of the [m, *] row-major inputs), D in 64 TMEM columns.  TMA
// keeps kLgStages stages in flight; the epilogue adds the scaled sums into
// the gradients.
__global__ void __launch_bounds__(kLgThreads, 2)
    lora_grad_kernel(const __grid_constant__ LoraGradMaps maps, const LoraGradBatch batch, int M, int splits) {
  pdl_trigger();
  extern __shared__ uint8_t lg_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(lg_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kLgStages * (kLgUBytes + kLgWBytes));
  uint64_t* empty = full + kLgStages;
  uint64_t* acc_full = empty + kLgStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const LoraGradProb& pb = batch.p[blockIdx.y];
  const int a0 = blockIdx.x * kLgA;
  if (a0 >= pb.A) return;  // whole CTA
  // interleaved U: the tile's 128 columns are all gate or all up
  const int sel = pb.ilv ? (a0 >> 7) & 1 : 0;
  if (!pb.out[sel] && (pb.ilv || pb.groups == 1)) return;  // that adapter is not trained
  const int split = blockIdx.z;
  const int m_per = ((M + splits - 1) / splits + kLgM - 1) / kLgM * kLgM;
  const int m_begin = split * m_per;
  const int m_end = min(M, m_begin + m_per);
  // splits end on 64-row boundaries or at M (where the boxes read zeros), so
  // no box reaches into the next split's rows
  const int nsteps = m_end > m_begin ? (m_end - m_begin + kLgM - 1) / kLgM : 0;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const CUtensorMap* umap = &maps.u[blockIdx.y];
  const CUtensorMap* wmap = &maps.w[blockIdx.y];
  if (threadIdx.x == 0) {
    for (int s = 0; s < kLgStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(umap);
    tma_prefetch_desc(wmap);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 64);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_wait();

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------------------ producer
    int issued = 0;
    bool ok = true;
    for (int s = 0; s < nsteps; ++s) {
      const int buf = s % kLgStages;
      if (!mbar_wait(&empty[buf], ((s / kLgStages) & 1) ^ 1, abort_flag, nullptr, 0)) {
        ok = false;
        break;
      }
      uint8_t* su = smem + buf * kLgUBytes;
      uint8_t* sw = smem + kLgStages * kLgUBytes + buf * kLgWBytes;
      const int m0 = m_begin + s * kLgM;
      mbar_arrive_expect_tx(&full[buf], kLgUBytes + kLgWBytes);
      tma_load_2d(su, umap, &full[buf], a0, m0);
      tma_load_2d(su + kLgUBytes / 2, umap, &full[buf], a0 + 64, m0);
      tma_load_2d(sw, wmap, &full[buf], 0, m0);
      ++issued;
    }
    if (!ok) {  // let the copies already issued land before the CTA can exit
      for (int j = max(0, issued - kLgStages); j < issued; ++j) {
        const uint32_t bar = smem_u32(&full[j % kLgStages]);
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(bar, (j / kLgStages) & 1) && globaltimer_ns() - t0 < 100000000ull) {
        }
      }
    }
  } else if (warp == 1 && lane == 0) {
    // ---------------------------------------------------------- MMA issuer
    constexpr uint32_t idesc = idesc_f16_f32(kLgA, 64) | (1u << 15) | (1u << 16);  // A, B MN-major
    bool ok = true;
    for (int s = 0; s < nsteps && ok; ++s) {
      const int buf = s % kLgStages;
      if (!mbar_wait(&full[buf], (s / kLgStages) & 1, abort_flag, nullptr, 0)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t su = smem_u32(smem + buf * kLgUBytes);
      const uint32_t sw = smem_u32(smem + kLgStages * kLgUBytes + buf * kLgWBytes);
      const uint64_t adesc = sw128_mn_desc(su, kLgUBytes / 2);
      const uint64_t bdesc = sw128_mn_desc(sw, kLgWBytes);
#pragma unroll
      for (int k = 0; k < kLgM / 16; ++k)  // +16 m rows of 128 bytes per K step
        umma_f16(tmem, adesc + (16 * 128 >> 4) * k, bdesc + (16 * 128 >> 4) * k, idesc, (s > 0 || k > 0) ? 1u : 0u);
      umma_commit(&empty[buf]);
    }
    if (ok && nsteps > 0) umma_commit(acc_full);
  }
  __syncwarp();

  // ------------------------------------------------------------ epilogue
  // warp w owns TMEM lanes 32w.. = a-rows a0 + 32w + lane; column b = 16 g + j
  const bool got = nsteps == 0 || mbar_wait(acc_full, 0, abort_flag, batch.err, kErrWaitAccum);
  if (__syncthreads_and(got)) {  // CTA-uniform: the staged store below synchronises
    tc_fence_after();
    const uint32_t taddr = tmem + (static_cast<uint32_t>(warp * 32) << 16);
    const int ar = warp * 32 + lane;  // a-row within the tile
    const int ncol = 16 * pb.groups;  // accumulator columns in use (<= 64)
    float acc[64];
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      if (nsteps > 0 && 32 * half < ncol) {  // warp-uniform
        uint32_t v[32];
        tmem_ld_32x32b_x32(taddr + 32 * half, v);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 32; ++j) acc[32 * half + j] = __uint_as_float(v[j]);
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) acc[32 * half + j] = 0.f;
      }
    }
    if (splits > 1) {
      // this split's partial [column][a-row] (each warp writes 128 contiguous
      // bytes per column); lora_grad_reduce_kernel sums the splits in order
      const int slot = blockIdx.y * gridDim.x + blockIdx.x;
      float* mine = batch.ws + (static_cast<size_t>(slot) * splits + split) * (64 * kLgA);
#pragma unroll
      for (int j = 0; j < 64; ++j)
        if (j < ncol) mine[j * kLgA + ar] = acc[j];
    } else {
      lg_store(pb, a0, sel, ar, acc, reinterpret_cast<float*>(smem));  // the stage buffers are idle now
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 64);
  }
}

// The m-splits' partials of lora_grad_kernel summed in split order (the same
// bits whatever order the splits finished in), scaled and stored where
// lg_store would put them.  One thread per (a-tile row, accumulator column):
// grid (a-tiles, problems, 32), 256 threads.
__global__ void __launch_bounds__(256) lora_grad_reduce_kernel(const LoraGradBatch batch, int splits) {
  pdl_trigger();
  pdl_wait();
  const LoraGradProb& pb = batch.p[blockIdx.y];
  const int a0 = blockIdx.x * kLgA;
  if (a0 >= pb.A) return;
  const int sel = pb.ilv ? (a0 >> 7) & 1 : 0;
  if (!pb.out[sel] && (pb.ilv || pb.groups == 1)) return;
  const int e = blockIdx.z * blockDim.x + threadIdx.x;
  const int j = e >> 7, ar = e & (kLgA - 1);  // column, a-row (a-rows fastest: coalesced partial reads)
  if (j >= 16 * pb.groups) return;
  const float* src = batch.ws + static_cast<size_t>(blockIdx.y * gridDim.x + blockIdx.x) * splits * (64 * kLgA) +
                     j * kLgA + ar;
  float t = 0.f;
#pragma unroll 4
  for (int s2 = 0; s2 < splits; ++s2) t += src[static_cast<size_t>(s2) * (64 * kLgA)];
  const int g = j >> 4, b = j & 15;
  const int a = a0 + ar;
  if (a < pb.A && b < pb.Bn && pb.out[g] && (!pb.ilv || g == sel)) {
    const int orow = pb.ilv ? ((a0 >> 8) << 7) + ar : a;  // the interleave maps a to its adapter row
    pb.out[g][static_cast<size_t>(orow) * pb.sa + static_cast<size_t>(b) * pb.sb] = t * pb.scale;
  }
}

}  // namespace

cudaError_t lora_merge(const float* flat, const LoraDims& d, int n_layers, const MergeWeights& base,
                       const MergedOut& out, cudaStream_t st) {
  const int H = d.H, Q = d.Q, KV = d.KV, I = d.I, QKV = Q + 2 * KV;
  const bool mlp = d.has_mlp();
  if (d.r > 16 || Q % kMrgRows || KV % kMrgRows || H % kMrgRows || H % 8 || Q % 8) return cudaErrorInvalidValue;
  if (64LL * (QKV + 2 * H + Q) >= (1LL << 31)) return cudaErrorInvalidValue;
  if (mlp && (I % 128 || !out.gu || !out.d || 64LL * (2 * I + 2 * H + I) >= (1LL << 31)))
    return cudaErrorInvalidValue;
  const int64_t mqkv_layer = merged_qkv_elems(d), mo_layer = merged_o_elems(d);
  const int64_t mgu_layer = merged_gu_elems(d), md_layer = merged_d_elems(d);
  // row tiles per block: a divisor of every adapter's row-tile count
  auto tiles_for = [](int a, int b) {
    int t = kMrgTiles;
    while (t > 1 && ((a / kMrgRows) % t || (b / kMrgRows) % t)) t /= 2;
    return t;
  };
  // one merged weight: rows [0, rows) of W (d_in columns) plus s B A
  auto main_block = [&](const MergeBase& src, int rows, int d_in, int which, int tiles, __half* dst, int64_t layer) {
    // tensor-core rank-r update over fp16 rows, or INT8 rows (16-column
    // multiples) starting from code * scale
    dim3 g((d_in + kMtCols - 1) / kMtCols, rows / kMtRows, n_layers);
    if (!src.q) {
      launch_pdl(lora_merge_tc_kernel<false>, g, 128, 0, st, flat, d, src, d_in, which, dst, layer, d_in + 64);
    } else if (d_in % 16 == 0) {
      launch_pdl(lora_merge_tc_kernel<true>, g, 128, 0, st, flat, d, src, d_in, which, dst, layer, d_in + 64);
    } else {
      dim3 gm((d_in + kMrgCols - 1) / kMrgCols, rows / (kMrgRows * tiles), n_layers);
      launch_pdl(lora_merge_main_kernel, gm, 256, 0, st, flat, d, src, d_in, which, tiles, dst, layer, d_in + 64);
    }
  };
  main_block(base.qkv, QKV, H, 0, tiles_for(Q, KV), out.qkv, mqkv_layer);
  main_block(base.o, H, Q, 1, tiles_for(H, H), out.o, mo_layer);
  if (mlp) {
    // gate/up: blocks of at most 128 rows stay inside one half of the interleave
    main_block(base.gu, 2 * I, H, 2, 2, out.gu, mgu_layer);
    main_block(base.d, H, I, 3, tiles_for(H, H), out.d, md_layer);
  }
  dim3 gp(128, n_layers);
  launch_pdl(lora_merge_pad_kernel, gp, 256, 0, st, flat, d, out.qkv, mqkv_layer, out.o, mo_layer);
  if (mlp) {
    dim3 gm(256, n_layers);
    launch_pdl(lora_merge_pad_mlp_kernel, gm, 256, 0, st, flat, d, out.gu, mgu_layer, out.d, md_layer);
  }
  return cudaGetLastError();
}

// CTAs per SM the m-splits aim for (two are resident at a time)
#ifndef LLMCU_LG_CTAS_PER_SM
#define LLMCU_LG_CTAS_PER_SM 2
#endif

int lora_grad_splits(int M, const LoraGradBatch& batch) {
  int tiles = 0;  // CTAs with work in one split
  for (int i = 0; i < batch.n; ++i) tiles += (batch.p[i].A + kLgA - 1) / kLgA;
  if (tiles < 1) tiles = 1;
  int s = (LLMCU_LG_CTAS_PER_SM * gemm_num_sms() + tiles - 1) / tiles;
  const int max_s = (M + 255) / 256;
  if (s > max_s) s = max_s;
  if (s > kLoraMaxSplits) s = kLoraMaxSplits;
  if (s < 1) s = 1;
  // the splits' partials must fit the workspace (fewer splits otherwise)
  const size_t per_split = static_cast<size_t>(batch.n) * ((batch.a_max + kLgA - 1) / kLgA) * 64 * kLgA;
  if (!batch.ws) s = 1;
  while (s > 1 && per_split * s > batch.ws_floats) --s;
  return s;
}

cudaError_t lora_grad(const LoraGradBatch& batch, int M, cudaStream_t st) {
  if (batch.n <= 0 || batch.n > kLoraMaxProbs) return cudaErrorInvalidValue;
  const int splits = lora_grad_splits(M, batch);
  const int tiles = (batch.a_max + kLgA - 1) / kLgA;
  static std::atomic<unsigned long long> attr_set{0};
  {
    cudaError_t e = once_per_device(attr_set, [] {
      return cudaFuncSetAttribute(lora_grad_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kLgSmem);
    });
    if (e != cudaSuccess) return e;
  }
  LoraGradMaps maps;
  for (int i = 0; i < batch.n; ++i) {
    const LoraGradProb& p = batch.p[i];
    if (p.groups < 1 || p.groups > 4) return cudaErrorInvalidValue;
    if (p.ilv && (p.groups != 2 || p.A % 256)) return cudaErrorInvalidValue;
    if (!encode_tma_2d_f16(&maps.u[i], p.U, M, p.A, p.ldu, kLgM) ||
        !encode_tma_2d_f16(&maps.w[i], p.W, M, 16 * p.groups, p.ldw, kLgM))
      return cudaErrorInvalidValue;
  }
  dim3 grid(tiles, batch.n, splits);
  launch_pdl(lora_grad_kernel, grid, kLgThreads, kLgSmem, st, maps, batch, M, splits);
  if (splits > 1) launch_pdl(lora_grad_reduce_kernel, dim3(tiles, batch.n, 64 * kLgA / 256), 256, 0, st, batch, splits);
  return cudaGetLastError();
}

}  // namespace llmcu
