// gemm.cuh -- persistent, warp-specialised tcgen05 GEMM for sm_100a.
//
//   C[M, N] = A[M, K] . B[N, K]^T
//
// fp16 operands, fp32 accumulation in TMEM, and a fused epilogue chosen at
// compile time.  A is K-major (rows contiguous along K).  B is K-major
// ([N, K] rows) or, with BMN, MN-major: the [K, N] matrix itself, read in
// 64 x 64 boxes, so a weight stored [out, in] serves both the forward
// (x W^T, K-major) and the input gradient (dY W, MN-major) without a
// transposed copy.  Columns at and past `n_main` are a side output: the
// LoRA projections h = x A^T / dh = dY B ride along as extra rows (columns)
// of the merged weight and leave through plain fp16 stores.
//
// Roles (64 + 32*EW threads, one CTA per SM):
//   warp 0        TMA producer -- fills a STAGES-deep ring of (A, B) smem tiles
//   warp 1        MMA issuer   -- tcgen05.mma into one of two TMEM accumulators
//                                (allocates / frees TMEM for the CTA)
//   warps 2..EW+1 epilogue     -- tcgen05.ld -> registers -> fused op; warp w
//                                reads TMEM lanes 32*(w%4).. (the lane quadrant
//                                it may access); with EW = 8 two warps share a
//                                quadrant and split the tile's columns.
// Epilogue I/O goes through a 4 KB shared-memory slab per warp (32 rows x
// 128 bytes, 128-byte swizzle): the warp writes its rows there and one lane
// issues a TMA store (or reduce-add) of the whole slab, so global writes leave
// the SM as full lines; inputs the epilogue needs (residual, SwiGLU
// pre-activations) arrive the same way through TMA loads.
// Tiles: BLOCK_M = 128 rows, BLOCK_N = BN (64/128/256), BLOCK_K = 64 (one
// 128-byte swizzle row of fp16).  Tile t -> (t % tiles_m, t / tiles_m), so
// CTAs that run together share the weight (B) tile and stream it once -- or,
// when A is the larger operand, the transposed order, so concurrent CTAs share
// A's rows instead.
#pragma once

#include <type_traits>

#include "common.cuh"
#include "sm100.cuh"

namespace llmcu {

struct GemmShape {
  int M, N;
  int K;
  int tiles_m, tiles_n, num_tiles;
  int splits;      // K splits (1 = none); split s writes rows [s * split_row_tiles * 128, ...)
  int kb_per_split;
  int split_row_tiles;  // tiles_m: one row block of partials per split; 0: splits reduce-add into the same rows
  int n_fastest;        // tile order: 1 = consecutive units walk N (share A rows), 0 = walk M (share B)
  int n_main;           // columns [n_main, N) go to the side output
  __half* side;         // [M, N - n_main] fp16, row stride ld_side
  int ld_side;
  // K splits with a fix-up (fixup != 0, splits > 1): every split of a tile
  // leaves its fp32 partial of each epilogue warp's slice in fx_ws; the last
  // split to arrive (counted in fx_cnt, one counter per slice, reset by that
  // split) sums all partials in split order into its TMEM accumulator and
  // runs the tile's epilogue as usual -- for GEMMs whose tiles fill under
  // half a wave
  int fixup;
  float* fx_ws;         // [tiles * CG * 4 * groups][splits][slice columns / 4][32] float4
  int* fx_cnt;          // [tiles * CG * 4 * groups], zero between launches
  // INT8 B, K-major (Q8 forward kernels): the weight's per-row fp32 scales,
  // one per output column, applied by the epilogue
  const float* b_scale;
};

constexpr int kBlockM = 128;
constexpr int kQ8Threads = 64;  // converter threads of the INT8-B kernels
constexpr int kBlockK = 64;
constexpr int kSlabBytes = 32 * 128;  // one 32-row x 128-byte box
constexpr int kMnBox = 64 * 128;      // MN-major B box: 64 K rows x 64 columns of fp16

// CG = 2: a CTA pair shares each 256 x BN tile; every CTA holds 128 rows
// of A and BN/2 rows of B per stage.
// Q8: B arrives as INT8 codes (kQBytes per stage) in the first half of the
// stage's B region; converter warps expand them in place into the fp16 tile.
template <int BN, int STAGES, int EW, int SLAB = kSlabBytes, int CG = 1, bool Q8 = false>
struct GemmSmem {
  static constexpr int kABytes = kBlockM * kBlockK * 2;       // 16 KB
  static constexpr int kBBytes = BN / CG * kBlockK * 2;       // 8/16/32 KB
  static constexpr int kQBytes = Q8 ? BN / CG * kBlockK : 0;  // INT8 codes of the B tile (inside B)
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kTmemCols = (2 * BN < 32) ? 32 : 2 * BN;  // two accumulators
  static constexpr int kSlabOffset = STAGES * kStageBytes;
  static constexpr int kBarOffset = kSlabOffset + EW * SLAB;
  static constexpr int kBytes = kBarOffset + 512 + 1024;       // + barriers + alignment slack
};

// ------------------------------------------------------ epilogue plumbing

// One epilogue warp's view: its 32-row slab of the tile and its staging slab.
struct EpiCtx {
  int lane;
  int row0;                 // first tile row of this warp (global row index)
  int row;                  // this thread's row = row0 + lane
  int M, N;
  uint32_t slab;            // shared address of the 4 KB staging slab
  uint64_t* bar;            // mbarrier for TMA loads into the slab
  uint32_t phase;           // its parity
  volatile int* abort_flag;
  int* err;
  const CUtensorMap* mapC;  // primary output
  const CUtensorMap* mapD;  // secondary input or output (epilogue specific)
  int n_main;               // first side-output column
  int fixup;                // K splits with a fix-up: a unit may end without its epilogue
  __half* side;
  int ld_side;
  const float* col_scale;   // INT8-B forward: the weight's row scale of each output column (null: none)
};

// Side-output columns [col0, col0 + n) of this thread's row as fp16 (plain
// 16-byte stores; the side output is a few columns wide).
__device__ __forceinline__ void side_store(const EpiCtx& c, int col0, const float* v, int n) {
  if (c.row >= c.M) return;
  __half* dst = c.side + static_cast<size_t>(c.row) * c.ld_side + (col0 - c.n_main);
  for (int j = 0; j < n / 8; ++j) {
    if (col0 + 8 * j >= c.N) break;
    uint4 w;
    w.x = pack_half2(v[8 * j], v[8 * j + 1]);
    w.y = pack_half2(v[8 * j + 2], v[8 * j + 3]);
    w.z = pack_half2(v[8 * j + 4], v[8 * j + 5]);
    w.w = pack_half2(v[8 * j + 6], v[8 * j + 7]);
    *reinterpret_cast<uint4*>(dst + 8 * j) = w;
  }
}

// byte offset of 16-byte chunk j (0..7) of the thread's 128-byte slab row,
// 128-byte swizzle (chunk ^ row % 8), as TMA lays the box out
// (box b of the slab: b * 4 KB; boxes are 1024-byte aligned)
__device__ __forceinline__ uint32_t slab_addr(const EpiCtx& c, int j, int b = 0) {
  return c.slab + static_cast<uint32_t>(b * kSlabBytes + c.lane * 128 + ((j ^ (c.lane & 7)) << 4));
}
__device__ __forceinline__ void slab_st(const EpiCtx& c, int j, uint4 v, int b = 0) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(slab_addr(c, j, b)), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w)
               : "memory");
}
__device__ __forceinline__ uint4 slab_ld(const EpiCtx& c, int j, int b = 0) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(slab_addr(c, j, b))
               : "memory");
  return v;
}
// Until the TMA engine has read the slab (previous store from this warp).
__device__ __forceinline__ void slab_wait_read(const EpiCtx& c) {
  if (c.lane == 0) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
  __syncwarp();
}
// Publish the slab to the async proxy and store box b of it to map at (x, y).
__device__ __forceinline__ void slab_store(const EpiCtx& c, const CUtensorMap* map, int x, int y, int b = 0) {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  __syncwarp();
  if (c.lane == 0) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(c.slab + b * kSlabBytes), "r"(x), "r"(y)
                 : "memory");
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
  }
}
// Same, adding the slab (fp32) into global memory.
__device__ __forceinline__ void slab_reduce_add(const EpiCtx& c, const CUtensorMap* map, int x, int y) {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  __syncwarp();
  if (c.lane == 0) {
    asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(c.slab), "r"(x), "r"(y)
                 : "memory");
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
  }
}
// TMA-load the box at (x, y) of map into the slab and wait for it.
__device__ __forceinline__ bool slab_load(EpiCtx& c, const CUtensorMap* map, int x, int y) {
  if (c.lane == 0) {
    mbar_arrive_expect_tx(c.bar, kSlabBytes);
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(c.slab),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(c.bar)), "r"(x), "r"(y)
        : "memory");
  }
  __syncwarp();
  const bool ok = mbar_wait(c.bar, c.phase, c.abort_flag, c.err, kErrWaitAccum);
  if (!ok) mbar_drain(c.bar, c.phase);
  c.phase ^= 1u;
  return ok;
}
__device__ __forceinline__ uint4 pack8(const float* v) {
  uint4 w;
  w.x = pack_half2(v[0], v[1]);
  w.y = pack_half2(v[2], v[3]);
  w.z = pack_half2(v[4], v[5]);
  w.w = pack_half2(v[6], v[7]);
  return w;
}
__device__ __forceinline__ void unpack8(uint4 w, float* v) {
  const __half2* h = reinterpret_cast<const __half2*>(&w);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}


// ----------------------------------------------------------------- epilogues
// Interface: kChunk accumulator columns per call (one 128-byte slab row per
// thread); chunk(col0) sees columns [col0, col0 + kChunk) of row c.row.
// Returning false aborts the epilogue (a bounded wait expired).

// C (fp16) = acc
struct EpiStoreF16 {
  struct Params {};
  struct State {};
  static constexpr int kChunk = 64;
  static constexpr int kSlab = kSlabBytes;
  static constexpr bool kPaired = false;
  static constexpr bool kStores = true;
  __device__ static void begin(State&, const Params&, const EpiCtx&, int) {}
  __device__ static bool chunk(State&, const Params&, EpiCtx& c, int col0, const float* v) {
    if (col0 >= c.N) return true;
    if (col0 >= c.n_main) {
      side_store(c, col0, v, kChunk);
      return true;
    }
    slab_wait_read(c);
#pragma unroll
    for (int j = 0; j < 8; ++j) slab_st(c, j, pack8(v + 8 * j));
    slab_store(c, c.mapC, col0, c.row0);
    return true;
  }
  __device__ static void end(State&, const Params&, const EpiCtx&, int) {}
};

// Output-projection dX with the attention backward's row sums fused:
// C (fp16) = dO = acc for the main columns, and per (row, head) of the slice
// delta = sum_d dO[row, d] * O[row, d] over the fp16-rounded dO (the value the
// attention backward reads) -- what FlashAttention's backward calls D
// (replaces a separate pass over dO and O).  O arrives by plain 16-byte
// loads one 32-column step ahead; the side columns (dh of the LoRA rows)
// leave as fp16 like EpiStoreF16's.
struct EpiStoreF16Delta {
  struct Params {
    const __half* o;  // attention output [M, n_main], row stride ldo
    int ldo;
    float* delta;     // [B, n_heads, S]
    int S, n_heads, head_dim;
  };
  struct State {
    uint4 f[4];  // O of the next 32 columns
  };
  static constexpr int kChunk = 128;
  static constexpr int kSlab = kSlabBytes;
  static constexpr bool kPaired = false;
  static constexpr bool kStores = true;
  static constexpr bool kTmemDirect = true;
  __device__ static void fetch(State& st, const Params& p, const EpiCtx& c, int col0, int q) {
    if (c.row < c.M && col0 < c.n_main) {
      const uint4* src = reinterpret_cast<const uint4*>(p.o + static_cast<size_t>(c.row) * p.ldo + col0 + 32 * q);
#pragma unroll
      for (int j = 0; j < 4; ++j) st.f[j] = __ldg(src + j);
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) st.f[j] = make_uint4(0u, 0u, 0u, 0u);
    }
  }
  __device__ static void begin(State& st, const Params& p, const EpiCtx& c, int, int col0) { fetch(st, p, c, col0, 0); }
  __device__ static bool tile(State& st, const Params& p, EpiCtx& c, int col0, uint32_t taddr, int) {
    if (col0 >= c.N) return true;
    if (col0 >= c.n_main) {
#pragma unroll 1
      for (int q = 0; q < 4; ++q) {
        float v[32];
        tmem_ld_32x32b_x32(taddr + 32 * q, *reinterpret_cast<uint32_t(*)[32]>(v));
        tmem_ld_wait();
        side_store(c, col0 + 32 * q, v, 32);
      }
      return true;
    }
    float dsum[2] = {0.f, 0.f};  // one or two heads per 128-column slice
#pragma unroll 1
    for (int q = 0; q < 4; ++q) {
      uint32_t of[16];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        of[4 * j] = st.f[j].x; of[4 * j + 1] = st.f[j].y; of[4 * j + 2] = st.f[j].z; of[4 * j + 3] = st.f[j].w;
      }
      if (q < 3) fetch(st, p, c, col0, q + 1);
      float v[32];
      tmem_ld_32x32b_x32(taddr + 32 * q, *reinterpret_cast<uint32_t(*)[32]>(v));
      tmem_ld_wait();
      uint32_t pk[16];
      float d = 0.f;
#pragma unroll
      for (int t = 0; t < 16; ++t) {
        pk[t] = pack_half2(v[2 * t], v[2 * t + 1]);
        const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&pk[t]));
        const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&of[t]));
        d = fmaf(a.x, b.x, fmaf(a.y, b.y, d));
      }
      if ((32 * q) / p.head_dim == 0)
        dsum[0] += d;
      else
        dsum[1] += d;
      const int h = (q & 1) * 4;
      if ((q & 1) == 0) slab_wait_read(c);
#pragma unroll
      for (int j = 0; j < 4; ++j) slab_st(c, h + j, make_uint4(pk[4 * j], pk[4 * j + 1], pk[4 * j + 2], pk[4 * j + 3]));
      if (q & 1) slab_store(c, c.mapC, col0 + 32 * (q - 1), c.row0);
    }
    if (c.row < c.M) {
      const int b = c.row / p.S, s = c.row % p.S;
      const int nh_slice = 128 / p.head_dim;
      for (int k = 0; k < nh_slice; ++k) {
        const int head = col0 / p.head_dim + k;
        p.delta[(static_cast<size_t>(b) * p.n_heads + head) * p.S + s] = dsum[k];
      }
    }
    return true;
  }
  __device__ static void end(State&, const Params&, const EpiCtx&, int) {}
};

// q/k/v projection with Qwen3's per-head q/k RMSNorm and the rotary
// embedding fused (head_dim 128: one warp's 128-column slice is one head of
// its 32 rows).  Every main column leaves as fp16 through mapC (the raw
// q/k/v the backward re-normalises); for q and k heads the warp then forms
// the head's sum of squares from the fp32 accumulator, and writes
// rot(x * rstd * gain) -- pairs (d, d + 64) rotated by the position's angle
// (src/kernels/rope.cu:26-35 after src/kernels/lora_forward.cu:233-237) --
// through mapD into the same columns of the rope output.  Side columns (h
// of the LoRA rows) leave as fp16 like EpiStoreF16's.  Replaces the
// separate QK-norm + RoPE pass over q and k.
struct EpiQKNormRope {
  struct Params {
    const float* qw;     // q_norm gain [128]
    const float* kw;     // k_norm gain [128]
    const float* cos_t;  // [S, 64]
    const float* sin_t;
    int S, n_q_cols, n_qk_cols;
    float eps;
  };
  struct State {};
  static constexpr int kChunk = 128;
  static constexpr int kSlab = 2 * kSlabBytes;  // both 64-column halves of the head at once
  static constexpr bool kPaired = false;
  static constexpr bool kStores = true;
  static constexpr bool kTmemDirect = true;
  __device__ static void begin(State&, const Params&, const EpiCtx&, int, int) {}
  __device__ static bool tile(State&, const Params& p, EpiCtx& c, int col0, uint32_t taddr, int) {
    if (col0 >= c.N) return true;
    if (col0 >= c.n_main) {
#pragma unroll 1
      for (int q = 0; q < 4; ++q) {
        float v[32];
        tmem_ld_32x32b_x32(taddr + 32 * q, *reinterpret_cast<uint32_t(*)[32]>(v));
        tmem_ld_wait();
        side_store(c, col0 + 32 * q, v, 32);
      }
      return true;
    }
    const bool qk = col0 < p.n_qk_cols;
    // raw fp16 values (box hb = columns [64 hb, 64 hb + 64)) and the head's sum of squares
    float ss = 0.f;
    slab_wait_read(c);
#pragma unroll 1
    for (int q = 0; q < 4; ++q) {
      float v[32];
      tmem_ld_32x32b_x32(taddr + 32 * q, *reinterpret_cast<uint32_t(*)[32]>(v));
      tmem_ld_wait();
#pragma unroll
      for (int i = 0; i < 32; ++i) ss = fmaf(v[i], v[i], ss);
#pragma unroll
      for (int j = 0; j < 4; ++j) slab_st(c, 4 * (q & 1) + j, pack8(v + 8 * j), q >> 1);
    }
    slab_store(c, c.mapC, col0, c.row0, 0);
    slab_store(c, c.mapC, col0 + 64, c.row0, 1);
    if (!qk) return true;
    const float* gw = col0 < p.n_q_cols ? p.qw : p.kw;
    const float r = rsqrtf(ss * (1.0f / 128.0f) + p.eps);
    const int pos = (c.row < c.M ? c.row : 0) % p.S;
    const float* cs = p.cos_t + static_cast<size_t>(pos) * 64;
    const float* sn = p.sin_t + static_cast<size_t>(pos) * 64;
    slab_wait_read(c);
#pragma unroll 1
    for (int d0 = 0; d0 < 64; d0 += 16) {
      // pairs (d, d + 64), d = d0 .. d0 + 15: y0 -> box 0, y1 -> box 1
      uint32_t a[16], b[16];
      tmem_ld_32x32b_x16(taddr + d0, a);
      tmem_ld_32x32b_x16(taddr + 64 + d0, b);
      float cv[16], sv[16], wa[16], wb[16];
#pragma unroll
      for (int i = 0; i < 16; i += 4) {
        *reinterpret_cast<float4*>(cv + i) = *reinterpret_cast<const float4*>(cs + d0 + i);
        *reinterpret_cast<float4*>(sv + i) = *reinterpret_cast<const float4*>(sn + d0 + i);
        *reinterpret_cast<float4*>(wa + i) = __ldg(reinterpret_cast<const float4*>(gw + d0 + i));
        *reinterpret_cast<float4*>(wb + i) = __ldg(reinterpret_cast<const float4*>(gw + 64 + d0 + i));
      }
      tmem_ld_wait();
      uint32_t p0[8], p1[8];
#pragma unroll
      for (int i = 0; i < 16; i += 2) {
        const float xa0 = __uint_as_float(a[i]) * r * wa[i], xb0 = __uint_as_float(b[i]) * r * wb[i];
        const float xa1 = __uint_as_float(a[i + 1]) * r * wa[i + 1], xb1 = __uint_as_float(b[i + 1]) * r * wb[i + 1];
        p0[i / 2] = pack_half2(xa0 * cv[i] - xb0 * sv[i], xa1 * cv[i + 1] - xb1 * sv[i + 1]);
        p1[i / 2] = pack_half2(xb0 * cv[i] + xa0 * sv[i], xb1 * cv[i + 1] + xa1 * sv[i + 1]);
      }
      slab_st(c, d0 / 8, make_uint4(p0[0], p0[1], p0[2], p0[3]), 0);
      slab_st(c, d0 / 8 + 1, make_uint4(p0[4], p0[5], p0[6], p0[7]), 0);
      slab_st(c, d0 / 8, make_uint4(p1[0], p1[1], p1[2], p1[3]), 1);
      slab_st(c, d0 / 8 + 1, make_uint4(p1[4], p1[5], p1[6], p1[7]), 1);
    }
    slab_store(c, c.mapD, col0, c.row0, 0);
    slab_store(c, c.mapD, col0 + 64, c.row0, 1);
    return true;
  }
  __device__ static void end(State&, const Params&, const EpiCtx&, int) {}
};

// C (fp32) = acc, or C += acc (TMA reduce-add) when accumulate != 0.
struct EpiStoreF32 {
  struct Params { int accumulate; };
  struct State {};
  static constexpr int kChunk = 32;
  static constexpr int kSlab = kSlabBytes;
  static constexpr bool kPaired = false;
  static constexpr bool kStores = true;
  __device__ static void begin(State&, const Params&, const EpiCtx&, int) {}
  __device__ static bool chunk(State&, const Params& p, EpiCtx& c, int col0, const float* v) {
    if (col0 >= c.N) return true;
    slab_wait_read(c);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      uint4 w;
      w.x = __float_as_uint(v[4 * j]);
      w.y = __float_as_uint(v[4 * j + 1]);
      w.z = __float_as_uint(v[4 * j + 2]);
      w.w = __float_as_uint(v[4 * j + 3]);
      slab_st(c, j, w);
    }
    if (p.accumulate)
      slab_reduce_add(c, c.mapC, col0, c.row0);
    else
      slab_store(c, c.mapC, col0, c.row0);
    return true;
  }
  __device__ static void end(State&, const Params&, const EpiCtx&, int) {}
};

// out (fp32) = acc + resid: the residual adds of the O and down projections
// (src/kernels/lora_forward.cu:265,297).  mapD = resid (input), mapC = out.
struct EpiResidF32 {
  struct Params {};
  struct State {};
  static constexpr int kChunk = 32;
  static constexpr int kSlab = kSlabBytes;
  static constexpr bool kPaired = false;
  static constexpr bool kStores = true;
  __device__ static void begin(State&, const Params&, const EpiCtx&, int) {}
  __device__ static bool chunk(State&, const Params&, EpiCtx& c, int col0, const float* v) {
    if (col0 >= c.N) return true;
    if (col0 >= c.n_main) {
      side_store(c, col0, v, kChunk);
      return true;
    }
    float f[kChunk];
#pragma unroll
    for (int j = 0; j < kChunk; ++j) f[j] = 1.f;
    if (c.col_scale) {
#pragma unroll
      for (int j = 0; j < kChunk; j += 4) *reinterpret_cast<float4*>(f + j) = __ldg(reinterpret_cast<const float4*>(c.col_scale + col0 + j));
    }
    slab_wait_read(c);
    if (!slab_load(c, c.mapD, col0, c.row0)) return false;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      uint4 r = slab_ld(c, j);
      r.x = __float_as_uint(__uint_as_float(r.x) + v[4 * j] * f[4 * j]);
      r.y = __float_as_uint(__uint_as_float(r.y) + v[4 * j + 1] * f[4 * j + 1]);
      r.z = __float_as_uint(__uint_as_float(r.z) + v[4 * j + 2] * f[4 * j + 2]);
      r.w = __float_as_uint(__uint_as_float(r.w) + v[4 * j + 3] * f[4 * j + 3]);
      slab_st(c, j, r);
    }
    slab_store(c, c.mapC, col0, c.row0);
    return true;
  }
  __device__ static void end(State&, const Params&, const EpiCtx&, int) {}
};

// Gate/up GEMM with SwiGLU (src/kernels/activation.cu:5-11).  The fused
// weight interleaves 128-row blocks of W_gate and W_up, so a 256-wide tile
// holds gate columns [0,128) and the matching up columns [128,256).  Writes
// act = silu(g) * u and, for the backward, the two factors it needs
// (src/kernels/activation.cu:26-38): at the gate slot  u * silu'(g)  =
// u * s * (1 + g * (1 - s)), at the up slot  silu(g) = g * s  (s = sigmoid(g)).
// mapC = stash [M, 2I] (fp16, interleaved like the weight), mapD = act [M, I].
struct EpiSwiGLU {
  struct Params {};
  struct State {};
  // one warp per TMEM lane quadrant (both 64-column chunks of its rows' gate
  // columns), so that two 4-KB slabs per warp -- the gate and up slots' factors
  // leave together -- still leave room for six pipeline stages
  static constexpr int kEpiGroups = 1;
  static constexpr int kChunk = 64;
  static constexpr int kSlab = 2 * kSlabBytes;
  static constexpr bool kPaired = true;  // requires BN == 256
  static constexpr bool kStores = true;
  __device__ static void begin(State&, const Params&, const EpiCtx&, int) {}
  // g: gate columns [cc, cc+64) of tile tn, u: the matching up columns.
  // A tile past n_main holds the side output (h of the gate/up adapters) in
  // its first 64 columns.
  __device__ static bool pair(State&, const Params&, EpiCtx& c, int tile_n, int cc, const float* g, const float* u) {
    if (tile_n * 256 >= c.n_main) {
      side_store(c, tile_n * 256 + cc, g, kChunk);
      return true;
    }
    uint32_t dgp[32], sp[32], ap[32];  // u silu'(g), silu(g), act as packed half2
    // INT8 weight: the row scales of these gate / up columns; lane L holds
    // columns 2L, 2L + 1 and hands them out by shuffle
    float2 my_g = make_float2(1.f, 1.f), my_u = make_float2(1.f, 1.f);
    if (c.col_scale) {
      my_g = __ldg(reinterpret_cast<const float2*>(c.col_scale + tile_n * 256 + cc) + c.lane);
      my_u = __ldg(reinterpret_cast<const float2*>(c.col_scale + tile_n * 256 + 128 + cc) + c.lane);
    }
    const bool scaled = c.col_scale != nullptr;  // warp-uniform
#pragma unroll
    for (int t = 0; t < 32; ++t) {
      float r0[3], r1[3];
      float2 sg2 = make_float2(1.f, 1.f), su2 = make_float2(1.f, 1.f);
      if (scaled) {
        sg2 = make_float2(__shfl_sync(0xffffffffu, my_g.x, t), __shfl_sync(0xffffffffu, my_g.y, t));
        su2 = make_float2(__shfl_sync(0xffffffffu, my_u.x, t), __shfl_sync(0xffffffffu, my_u.y, t));
      }
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const float gv = g[2 * t + e] * (e ? sg2.y : sg2.x), uv = u[2 * t + e] * (e ? su2.y : su2.x);
        // fast reciprocal (2 ulp; 0 once exp overflows): far below the fp16 rounding of the outputs
        const float sg = __fdividef(1.0f, 1.0f + __expf(-gv));
        const float si = gv * sg;
        float* r = e ? r1 : r0;
        r[0] = uv * sg * (1.0f + gv * (1.0f - sg));
        r[1] = si;
        r[2] = si * uv;
      }
      dgp[t] = pack_half2(r0[0], r1[0]);
      sp[t] = pack_half2(r0[1], r1[1]);
      ap[t] = pack_half2(r0[2], r1[2]);
    }
    slab_wait_read(c);
#pragma unroll
    for (int j = 0; j < 8; ++j) slab_st(c, j, make_uint4(dgp[4 * j], dgp[4 * j + 1], dgp[4 * j + 2], dgp[4 * j + 3]), 0);
#pragma unroll
    for (int j = 0; j < 8; ++j) slab_st(c, j, make_uint4(sp[4 * j], sp[4 * j + 1], sp[4 * j + 2], sp[4 * j + 3]), 1);
    slab_store(c, c.mapC, tile_n * 256 + cc, c.row0, 0);
    slab_store(c, c.mapC, tile_n * 256 + 128 + cc, c.row0, 1);
    // the first slab again, once its store (not the second's) has read it
    if (c.lane == 0) asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
    __syncwarp();
#pragma unroll
    for (int j = 0; j < 8; ++j) slab_st(c, j, make_uint4(ap[4 * j], ap[4 * j + 1], ap[4 * j + 2], ap[4 * j + 3]), 0);
    slab_store(c, c.mapD, tile_n * 128 + cc, c.row0, 0);
    return true;
  }
  __device__ static void end(State&, const Params&, const EpiCtx&, int) {}
};

// Down-projection dX with the SwiGLU backward fused (src/kernels/activation.cu:26-38):
// acc = d_act[row, i] for the tile's 128-column slice; with the factors the
// forward stashed, dg = d_act * u silu'(g) and du = d_act * silu(g), written
// into the interleaved dgu (mapC), the A operand of the gate/up dX GEMM.  The
// factors of each 32-column step arrive by TMA (mapD: [32 rows x 32 columns]
// boxes, 64-byte swizzle) into the warp's second 4-KB slab, one step ahead,
// the first issued before the accumulator is ready; outputs leave through
// the first slab.  (One row per thread would make the loads touch 32 lines
// per instruction; the boxes are read back from shared memory instead.)
// kScaled: the INT8 in-GEMM mode, whose dgu columns carry the gate/up row
// scales (out_scale) for the next GEMM; compiled out otherwise.
template <bool kScaled>
struct EpiSwiGLUBwdT {
  struct Params {
    const __half* gu_in;  // [M, 2N] interleaved stash (also behind mapD)
    int ld;
    const float* out_scale;  // per dgu column factors (an INT8 gate/up weight's row scales, folded into
                             // the next GEMM's A operand), null: none
  };
  struct State {
    bool pending;  // step 0's factor boxes were issued by begin()
  };
  // one warp per TMEM lane quadrant takes the whole 256-column tile (8 steps
  // of 32 columns): with 4 epilogue warps the two 4-KB slabs of each leave
  // room for a sixth pipeline stage, which the main loop needs more than the
  // epilogue needs a second warp
  static constexpr int kEpiGroups = 1;
  static constexpr int kChunk = 256;
  static constexpr int kSlab = 2 * kSlabBytes;  // [0, 4 KB) output staging, [4 KB, 8 KB) factor boxes
  static constexpr bool kPaired = false;
  static constexpr bool kStores = true;
  static constexpr bool kTmemDirect = true;
  static constexpr int kFacBox = 32 * 32 * 2;  // one [32 rows x 32 fp16] box
  // step q's boxes (gate-slot columns gcol + 32q, up-slot columns gcol + 128 + 32q)
  __device__ static void issue(const EpiCtx& c, int gcol, int q) {
    if (c.lane == 0) {
      mbar_arrive_expect_tx(c.bar, 2 * kFacBox);
      const uint32_t dst = c.slab + kSlabBytes;
#pragma unroll
      for (int h = 0; h < 2; ++h)
        asm volatile(
            "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
            " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst + h * kFacBox),
            "l"(reinterpret_cast<uint64_t>(c.mapD)), "r"(smem_u32(c.bar)), "r"(gcol + 128 * h + 32 * q), "r"(c.row0)
            : "memory");
    }
  }
  // this thread's row of box h: 16-byte chunk j sits at chunk j ^ ((row / 2) % 4) (64-byte swizzle)
  __device__ static uint4 box_ld(const EpiCtx& c, int h, int j) {
    uint4 v;
    const uint32_t a =
        c.slab + kSlabBytes + h * kFacBox + c.lane * 64 + ((j ^ ((c.lane >> 1) & 3)) << 4);
    asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a) : "memory");
    return v;
  }
  // the epilogue gave up before tile(): let step 0's boxes land first
  __device__ static void drain(State& st, const EpiCtx& c) {
    if (st.pending) mbar_drain(c.bar, c.phase);
  }
  // stash column of the gate slot of step t (0..7) of the tile at col0: each
  // 128-column half of the tile has its own 256-column block of factors
  __device__ static int gcol_of(int col0, int t) { return ((col0 + 128 * (t >> 2)) >> 7) * 256; }
  // before the accumulator is ready: the row's factors of this tile (2 x 512
  // contiguous bytes) into L2, and step 0's boxes (not for units that a K
  // split may finish elsewhere)
  __device__ static void begin(State& st, const Params& p, const EpiCtx& c, int, int col0) {
    st.pending = false;
    if (col0 >= c.n_main) return;
    if (c.row < c.M) {
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const char* f =
            reinterpret_cast<const char*>(p.gu_in + static_cast<size_t>(c.row) * p.ld + gcol_of(col0, 4 * hh));
#pragma unroll
        for (int j = 0; j < 4; ++j) prefetch_l2(f + 128 * j);
      }
    }
    if (!c.fixup) {
      issue(c, gcol_of(col0, 0), 0);
      st.pending = true;
    }
  }
  __device__ static bool tile(State& st, const Params& p, EpiCtx& c, int col0, uint32_t taddr, int) {
    if (col0 >= c.N) return true;
    if (col0 >= c.n_main) {  // dh of the down adapter (s B_down columns)
#pragma unroll 1
      for (int q = 0; q < kChunk / 32 && col0 + 32 * q < c.N; ++q) {
        float v[32];
        tmem_ld_32x32b_x32(taddr + 32 * q, *reinterpret_cast<uint32_t(*)[32]>(v));
        tmem_ld_wait();
        side_store(c, col0 + 32 * q, v, 32);
      }
      return true;
    }
    if (!st.pending) issue(c, gcol_of(col0, 0), 0);
    st.pending = false;
    uint32_t du_keep[16];
#pragma unroll 1
    for (int t = 0; t < kChunk / 32; ++t) {
      const int q = t & 3;  // step within the 128-column half
      const int gcol = gcol_of(col0, t);
      // step q's boxes landed: copy this row's 32 + 32 factors out, then
      // (reads ordered before the async proxy's next write) issue step q + 1
      if (!mbar_wait(c.bar, c.phase, c.abort_flag, c.err, kErrWaitAccum)) {
        mbar_drain(c.bar, c.phase);
        return false;
      }
      c.phase ^= 1u;
      uint32_t f0[16], f1[16];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint4 a = box_ld(c, 0, j), b = box_ld(c, 1, j);
        f0[4 * j] = a.x; f0[4 * j + 1] = a.y; f0[4 * j + 2] = a.z; f0[4 * j + 3] = a.w;
        f1[4 * j] = b.x; f1[4 * j + 1] = b.y; f1[4 * j + 2] = b.z; f1[4 * j + 3] = b.w;
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (t + 1 < kChunk / 32) issue(c, gcol_of(col0, t + 1), (t + 1) & 3);
      float v[32];
      tmem_ld_32x32b_x32(taddr + 32 * t, *reinterpret_cast<uint32_t(*)[32]>(v));
      tmem_ld_wait();
      uint32_t dg[16], du[16];
      // per dgu column factors of these 32 gate / up columns: lane L holds
      // gate column L and up column L (+128), handed out by shuffle
      float my_g = 1.f, my_u = 1.f;
      if (kScaled && p.out_scale) {
        my_g = __ldg(p.out_scale + gcol + 32 * q + c.lane);
        my_u = __ldg(p.out_scale + gcol + 128 + 32 * q + c.lane);
      }
      const bool scaled = kScaled && p.out_scale != nullptr;  // warp-uniform
#pragma unroll
      for (int t = 0; t < 16; ++t) {
        const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&f0[t]));
        const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&f1[t]));
        float sg0 = 1.f, sg1 = 1.f, su0 = 1.f, su1 = 1.f;
        if (scaled) {
          sg0 = __shfl_sync(0xffffffffu, my_g, 2 * t);
          sg1 = __shfl_sync(0xffffffffu, my_g, 2 * t + 1);
          su0 = __shfl_sync(0xffffffffu, my_u, 2 * t);
          su1 = __shfl_sync(0xffffffffu, my_u, 2 * t + 1);
        }
        dg[t] = pack_half2(v[2 * t] * a.x * sg0, v[2 * t + 1] * a.y * sg1);
        du[t] = pack_half2(v[2 * t] * b.x * su0, v[2 * t + 1] * b.y * su1);
      }
      // slab rows hold 64 columns: steps 0/2 fill chunks 0-3, steps 1/3 chunks 4-7
      const int h = (q & 1) * 4;
      if ((q & 1) == 0) slab_wait_read(c);
#pragma unroll
      for (int j = 0; j < 4; ++j) slab_st(c, h + j, make_uint4(dg[4 * j], dg[4 * j + 1], dg[4 * j + 2], dg[4 * j + 3]));
      if ((q & 1) == 0) {
#pragma unroll
        for (int t = 0; t < 16; ++t) du_keep[t] = du[t];
        continue;
      }
      const int gc = gcol + 32 * (q - 1);  // first column of these 64 gate columns
      slab_store(c, c.mapC, gc, c.row0);
      slab_wait_read(c);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        slab_st(c, j, make_uint4(du_keep[4 * j], du_keep[4 * j + 1], du_keep[4 * j + 2], du_keep[4 * j + 3]));
        slab_st(c, 4 + j, make_uint4(du[4 * j], du[4 * j + 1], du[4 * j + 2], du[4 * j + 3]));
      }
      slab_store(c, c.mapC, gc + 128, c.row0);
    }
    return true;
  }
  __device__ static void end(State&, const Params&, const EpiCtx&, int) {}
};
using EpiSwiGLUBwd = EpiSwiGLUBwdT<false>;
using EpiSwiGLUBwdScaled = EpiSwiGLUBwdT<true>;

// lm_head forward over one vocabulary chunk, for the streamed cross-entropy
// (src/kernels/loss.cu:24-61 without the [M, V] logits): per row and
// 128-column slot, exp(l - r) goes as fp16 into the chunk buffer (mapC,
// [M, chunk width]) that the chunk's input-gradient GEMM reads next, and
// (r, sum of exp(l - r)) into the slot's partials.  r is the row's running
// reference (ref, kept by ce_stream_rescale) unless the slot's max lies more
// than kCeSlotRange above it -- its values could leave fp16's range; always so
// in the first chunk, whose reference is -inf -- and then r is the slot's own
// max and ce_stream_rescale moves the row to a new reference before the
// chunk's values are read.  The target's column is stored as 0 (its
// (p - 1) E_t term is added in fp32 by ce_stream_finish) and its logit kept.
// Straight from TMEM: one pass for the max, one for exp / sum / store.
struct EpiCEStream {
  struct Params {
    const int* targets;   // [M]
    const float* ref;     // [M] running reference of each row
    float* part_ref;      // [M, slots]
    float* part_sum;      // [M, slots]
    float* tgt_logit;     // [M]
    int slots;            // 128-column slots of the whole vocabulary
    int vocab_off;        // vocabulary index of the chunk's column 0 (a multiple of 128)
  };
  struct State {};
  static constexpr int kChunk = 128;
  static constexpr int kSlab = kSlabBytes;
  static constexpr bool kPaired = false;
  static constexpr bool kStores = true;
  static constexpr bool kTmemDirect = true;
  __device__ static void begin(State&, const Params&, const EpiCtx&, int) {}
  // columns [col0, col0 + 128) of the chunk for row c.row; taddr = TMEM address of column col0
  __device__ static bool tile(State&, const Params& p, EpiCtx& c, int col0, uint32_t taddr, int) {
    if (col0 >= c.N) return true;
    const int nv = min(128, c.N - col0);
    const bool live = c.row < c.M;
    const int t = live ? __ldg(p.targets + c.row) - (p.vocab_off + col0) : -1;
    // the first chunk (column 0 of the vocabulary) starts every row at -inf
    const float r0 = (live && p.vocab_off > 0) ? p.ref[c.row] : -INFINITY;
    // a whole slot without any of the warp's targets (nearly every slot):
    // no per-column tests
    const bool plain = nv == 128 && !__any_sync(0xffffffffu, t >= 0 && t < 128);
    float m = -INFINITY;
#pragma unroll 1
    for (int q = 0; q < 4; ++q) {
      float v[32];
      tmem_ld_32x32b_x32(taddr + 32 * q, *reinterpret_cast<uint32_t(*)[32]>(v));
      tmem_ld_wait();
      if (plain) {
#pragma unroll
        for (int j = 0; j < 32; ++j) m = fmaxf(m, v[j]);
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          if (32 * q + j < nv) m = fmaxf(m, v[j]);
          if (32 * q + j == t) p.tgt_logit[c.row] = v[j];
        }
      }
    }
    const bool own = !(m <= r0 + kCeSlotRange);  // -inf reference: always
    const float r = own ? m : r0;
    const float r2 = r * kLog2e;
    float s = 0.f;
#pragma unroll 1
    for (int h = 0; h < 2; ++h) {  // 64 columns = one 128-byte slab row of fp16
      uint32_t pk[32];
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        float v[32];
        tmem_ld_32x32b_x32(taddr + 64 * h + 32 * q, *reinterpret_cast<uint32_t(*)[32]>(v));
        tmem_ld_wait();
        if (plain) {
#pragma unroll
          for (int j = 0; j < 32; j += 2) {
            const float e0 = fast_exp2(fmaf(v[j], kLog2e, -r2));
            const float e1 = fast_exp2(fmaf(v[j + 1], kLog2e, -r2));
            s += e0 + e1;
            pk[16 * q + j / 2] = pack_half2(e0, e1);
          }
        } else {
#pragma unroll
          for (int j = 0; j < 32; j += 2) {
            const int cj = 64 * h + 32 * q + j;
            const float e0 = cj < nv ? fast_exp2(fmaf(v[j], kLog2e, -r2)) : 0.f;
            const float e1 = cj + 1 < nv ? fast_exp2(fmaf(v[j + 1], kLog2e, -r2)) : 0.f;
            s += e0 + e1;
            pk[16 * q + j / 2] = pack_half2(cj == t ? 0.f : e0, cj + 1 == t ? 0.f : e1);
          }
        }
      }
      if (64 * h < nv) {
        slab_wait_read(c);
#pragma unroll
        for (int j = 0; j < 8; ++j) slab_st(c, j, make_uint4(pk[4 * j], pk[4 * j + 1], pk[4 * j + 2], pk[4 * j + 3]));
        slab_store(c, c.mapC, col0 + 64 * h, c.row0);
      }
    }
    if (live) {
      const size_t o = static_cast<size_t>(c.row) * p.slots + ((p.vocab_off + col0) >> 7);
      p.part_ref[o] = r;
      p.part_sum[o] = s;
    }
    return true;
  }
  __device__ static void end(State&, const Params&, const EpiCtx&, int) {}
};

// begin(st, p, c, slot, col0): the epilogue takes its slice's first column
template <class E, class = void>
struct epi_begin_col : std::false_type {};
template <class E>
struct epi_begin_col<E, std::void_t<decltype(E::begin(std::declval<typename E::State&>(), std::declval<const typename E::Params&>(),
                                                      std::declval<const EpiCtx&>(), 0, 0))>> : std::true_type {};

template <class E, class = void>
struct epi_drain : std::false_type {};
template <class E>
struct epi_drain<E, std::void_t<decltype(E::drain(std::declval<typename E::State&>(), std::declval<const EpiCtx&>()))>>
    : std::true_type {};

template <class E, class = void>
struct epi_tmem_direct : std::false_type {};
template <class E>
struct epi_tmem_direct<E, std::void_t<decltype(E::kTmemDirect)>> : std::bool_constant<E::kTmemDirect> {};

// ---------------------------------------------------------------- the kernel

// CG = 2: launched as clusters of two CTAs.  The even CTA's MMA warp issues
// tcgen05.mma.cta_group::2 (M = 256) for both; both CTAs' TMA loads count
// on the even CTA's `full` barriers, its commits arrive on both CTAs'
// `empty` / `acc_full` barriers, and both CTAs' epilogues drain their own
// TMEM rows and arrive on the even CTA's `acc_empty`.
// Q8: B is INT8 codes.  The producer's TMA brings them (plain row-major
// boxes) into the stage's Q region; the converter warps (kQ8Threads, after
// the epilogue warps) write the codes as exact fp16 values into the stage's
// B tile in the 128-byte-swizzled layout the MMA reads, and each CTA's
// converters arrive once on the (even CTA's) full barrier.  The weight's
// per-row scales act outside the MMA, as in the reference's INT8 GEMM
// (src/kernels/quantize.cu:55-78 multiplies the sum by scale[n]): K-major
// (forward) by the epilogue on each output column (sh.b_scale); MN-major
// (input gradient, the scales run along K) by the caller, folded into A.
template <int BN, int STAGES, int EW, class Epi, bool BMN, int CG, bool Q8 = false>
__global__ void __launch_bounds__(64 + 32 * EW + (Q8 ? kQ8Threads : 0), 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmD,
                   const GemmShape sh, const typename Epi::Params ep, int* err) {
  static_assert(CG == 1 || (CG == 2 && BN == 256), "CTA pairs use 256-wide tiles");
  static_assert(!Q8 || BN == 256, "INT8 B only with 256-wide tiles");
  using L = GemmSmem<BN, STAGES, EW, Epi::kSlab, CG, Q8>;
  constexpr int kRowsPerTile = kBlockM * CG;  // tile rows (both CTAs of a pair)
  constexpr int kBRows = BN / CG;             // B rows (N) this CTA loads
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBarOffset);
  uint64_t* full = bars;                    // [STAGES]
  uint64_t* empty = bars + STAGES;          // [STAGES]
  uint64_t* acc_full = bars + 2 * STAGES;   // [2]
  uint64_t* acc_empty = acc_full + 2;       // [2]
  uint64_t* slab_bar = acc_empty + 2;       // [EW]
  uint64_t* qfull = slab_bar + EW;          // [STAGES] (Q8): the stage's INT8 codes landed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(qfull + (Q8 ? STAGES : 0));
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* conv_ok = reinterpret_cast<volatile int*>(tmem_slot + 2);  // Q8 converters' shared verdict

  pdl_trigger();
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = CG == 2 ? cluster_ctarank() : 0u;
  const int unit0 = CG == 2 ? static_cast<int>(blockIdx.x) / 2 : static_cast<int>(blockIdx.x);
  const int ustep = CG == 2 ? static_cast<int>(gridDim.x) / 2 : static_cast<int>(gridDim.x);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], Q8 ? 1 + CG : 1);  // Q8: + one converter arrival per CTA
      mbar_init(&empty[s], 1);
      if constexpr (Q8) mbar_init(&qfull[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 32 * EW * CG);
    }
    for (int w = 0; w < EW; ++w) mbar_init(&slab_bar[w], 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    if constexpr (CG == 2) {
      tmem_alloc_pair(tmem_slot, L::kTmemCols);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, L::kTmemCols);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  if constexpr (CG == 2)
    cluster_sync_all();  // barriers initialised in both CTAs before any remote arrive
  else
    __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int nk = (sh.K + kBlockK - 1) / kBlockK;
  const int num_units = sh.num_tiles * sh.splits;  // (tile, K split) work units
  if (warp == 0 && lane == 0 && unit0 < num_units) {
    // while the previous kernel finishes: the first unit's first stages of A
    // and B into L2.  A prefetch only fills L2, which stays coherent with that
    // kernel's writes; the loads into shared memory wait for it below.
    const int tile = unit0 % sh.num_tiles;
    const int sp = unit0 / sh.num_tiles;
    const int tm = sh.n_fastest ? tile / sh.tiles_n : tile % sh.tiles_m;
    const int tn = sh.n_fastest ? tile % sh.tiles_n : tile / sh.tiles_m;
    const int arow = tm * kRowsPerTile + static_cast<int>(rank) * kBlockM;
    const int brow = tn * BN + static_cast<int>(rank) * kBRows;
    const int kb0 = sp * sh.kb_per_split;
    const int kb1 = min(min(nk, kb0 + sh.kb_per_split), kb0 + STAGES);
    for (int kb = kb0; kb < kb1; ++kb) {
      tma_prefetch_l2_2d(&tmA, kb * kBlockK, arow);
      if constexpr (!BMN) {
        tma_prefetch_l2_2d(&tmB, kb * kBlockK, brow);
      } else {
#pragma unroll
        for (int j = 0; j < kBRows / 64; ++j) tma_prefetch_l2_2d(&tmB, brow + 64 * j, kb * kBlockK);
      }
    }
  }
  pdl_wait();  // the prologue above overlapped the previous kernel's tail

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ producer
      int it = 0;
      bool ok = true;
      for (int u = unit0; u < num_units && ok; u += ustep) {
        const int tile = u % sh.num_tiles;
        const int sp = u / sh.num_tiles;
        const int tm = sh.n_fastest ? tile / sh.tiles_n : tile % sh.tiles_m;
        const int tn = sh.n_fastest ? tile % sh.tiles_n : tile / sh.tiles_m;
        const int kb_end = min(nk, (sp + 1) * sh.kb_per_split);
        const int arow = tm * kRowsPerTile + static_cast<int>(rank) * kBlockM;
        const int brow = tn * BN + static_cast<int>(rank) * kBRows;
        for (int kb = sp * sh.kb_per_split; kb < kb_end; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t par = ((it / STAGES) & 1) ^ 1;
          if (!mbar_wait(&empty[s], par, abort_flag, err, kErrWaitConsumer)) { ok = false; break; }
          uint8_t* sa = smem + s * L::kStageBytes;
          uint8_t* sb = sa + L::kABytes;
          if constexpr (Q8) {
            // the INT8 codes of this CTA's B rows into the B region's first half (local barrier)
            uint8_t* sq = sb;
            mbar_arrive_expect_tx(&qfull[s], L::kQBytes);
            if constexpr (!BMN) {
              tma_load_2d(sq, &tmB, &qfull[s], kb * kBlockK, brow);
            } else {
#pragma unroll
              for (int j = 0; j < kBRows / 64; ++j) tma_load_2d(sq + j * 4096, &tmB, &qfull[s], brow + 64 * j, kb * kBlockK);
            }
          }
          if constexpr (CG == 2) {
            // both CTAs' bytes count on the even CTA's barrier
            const uint32_t fb = mapa_shared(smem_u32(&full[s]), 0);
            if (rank == 0) mbar_arrive_expect_tx(&full[s], Q8 ? 2 * L::kABytes : 2 * (L::kABytes + L::kBBytes));
            tma_load_2d_pair(sa, &tmA, fb, kb * kBlockK, arow);
            if constexpr (Q8) {
              // B comes from the converters
            } else if constexpr (!BMN) {
              tma_load_2d_pair(sb, &tmB, fb, kb * kBlockK, brow);
            } else {
#pragma unroll
              for (int j = 0; j < kBRows / 64; ++j) tma_load_2d_pair(sb + j * kMnBox, &tmB, fb, brow + 64 * j, kb * kBlockK);
            }
          } else {
            mbar_arrive_expect_tx(&full[s], Q8 ? L::kABytes : L::kABytes + L::kBBytes);
            tma_load_2d(sa, &tmA, &full[s], kb * kBlockK, arow);
            if constexpr (Q8) {
              // B comes from the converters
            } else if constexpr (!BMN) {
              tma_load_2d(sb, &tmB, &full[s], kb * kBlockK, brow);
            } else {
              // [64 K rows x 64 N columns] boxes side by side along N
#pragma unroll
              for (int j = 0; j < BN / 64; ++j)
                tma_load_2d(sb + j * kMnBox, &tmB, &full[s], brow + 64 * j, kb * kBlockK);
            }
          }
        }
      }
      if (!ok && CG == 1) {
        // Let the copies already issued land before the CTA can exit (a CTA
        // pair waits for the peer at the final cluster barrier instead).
        for (int j = 0; j < STAGES; ++j) {
          const int i2 = it - 1 - j;
          if (i2 < 0) break;
          uint32_t a = smem_u32(&full[i2 % STAGES]);
          const uint64_t t0 = globaltimer_ns();
          while (!mbar_try_wait(a, (i2 / STAGES) & 1) && globaltimer_ns() - t0 < 100000000ull) {
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      // ---------------------------------------------------------- MMA issuer
      constexpr uint32_t idesc = idesc_f16_f32(kRowsPerTile, BN) | (BMN ? (1u << 16) : 0u);
      int it = 0;
      int i = 0;
      bool ok = true;
      for (int u = unit0; u < num_units && ok; u += ustep, ++i) {
        const int acc = i & 1;
        if (!mbar_wait(&acc_empty[acc], ((i >> 1) & 1) ^ 1, abort_flag, err, kErrWaitEpilogue)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        const int sp = u / sh.num_tiles;
        const int kb_begin = sp * sh.kb_per_split;
        const int kb_end = min(nk, kb_begin + sh.kb_per_split);
        for (int kb = kb_begin; kb < kb_end; ++kb, ++it) {
          const int s = it % STAGES;
          if (!mbar_wait(&full[s], (it / STAGES) & 1, abort_flag, err, kErrWaitProducer)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + s * L::kStageBytes);
          const uint32_t sb = sa + L::kABytes;
          const uint64_t adesc = sw128_kmajor_desc(sa);
          const uint64_t bdesc = BMN ? sw128_mn_desc(sb, kMnBox) : sw128_kmajor_desc(sb);
#pragma unroll
          for (int k = 0; k < kBlockK / 16; ++k) {
            // K-major: +32 bytes per 16-element K step inside the 128-byte
            // swizzle row; MN-major: +16 rows of 128 bytes
            const uint64_t bk = BMN ? bdesc + (16 * 128 >> 4) * k : bdesc + 2 * k;
            if constexpr (CG == 2)
              umma_f16_pair(d_tmem, adesc + 2 * k, bk, idesc, (kb != kb_begin || k != 0) ? 1u : 0u);
            else
              umma_f16(d_tmem, adesc + 2 * k, bk, idesc, (kb != kb_begin || k != 0) ? 1u : 0u);
          }
          if constexpr (CG == 2) {
            umma_commit_pair(smem_u32(&empty[s]));
            umma_commit_pair(mapa_shared(smem_u32(&empty[s]), 1));
          } else {
            umma_commit(&empty[s]);
          }
        }
        if (ok) {
          if constexpr (CG == 2) {
            umma_commit_pair(smem_u32(&acc_full[acc]));
            umma_commit_pair(mapa_shared(smem_u32(&acc_full[acc]), 1));
          } else {
            umma_commit(&acc_full[acc]);
          }
        }
      }
    }
  } else if (Q8 && warp >= 2 + EW) {
    // ------------------------------------------------------------ converters
    // per stage: this CTA's kBRows B rows x 64 K of INT8 codes -> fp16 in
    // the MMA's 128-byte-swizzled layout.  K-major (forward): row r = output
    // feature brow + r, 64 codes of K.  MN-major (input gradient): box j of
    // 64 K rows (the weight's output features, scale per row) x 64 N columns.
    const int ct = threadIdx.x - (64 + 32 * EW);  // 0 .. kQ8Threads - 1
    int it = 0;
    bool ok = true;
    for (int u = unit0; u < num_units && ok; u += ustep) {
      const int sp = u / sh.num_tiles;
      const int kb_end = min(nk, (sp + 1) * sh.kb_per_split);
      for (int kb = sp * sh.kb_per_split; kb < kb_end; ++kb, ++it) {
        const int s = it % STAGES;
        // one thread waits for the codes and publishes the outcome, so that
        // every converter thread leaves together when a wait gives up
        if (ct == 0) *conv_ok = mbar_wait(&qfull[s], (it / STAGES) & 1, abort_flag, err, kErrWaitProducer) ? 1 : 0;
        asm volatile("bar.sync 1, %0;" ::"n"(kQ8Threads) : "memory");
        if (!*conv_ok) {
          ok = false;
          break;
        }
        const uint32_t sb32 = smem_u32(smem + s * L::kStageBytes + L::kABytes);  // shared-space addresses
        // kBRows x 64 codes = kBRows * 4 groups of 16: every group is read
        // before any fp16 is written over the codes (they share the region)
        constexpr int kPer = kBRows * 4 / kQ8Threads;
        int4 raw[kPer];
#pragma unroll
        for (int i = 0; i < kPer; ++i) {
          const int g = ct + i * kQ8Threads;
          const int box = BMN ? g / 256 : 0;
          const int srow = BMN ? (g >> 2) & 63 : g >> 2;
          asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                       : "=r"(raw[i].x), "=r"(raw[i].y), "=r"(raw[i].z), "=r"(raw[i].w)
                       : "r"(sb32 + box * 4096 + srow * 64 + (g & 3) * 16));
        }
        asm volatile("bar.sync 1, %0;" ::"n"(kQ8Threads) : "memory");
#pragma unroll
        for (int i = 0; i < kPer; ++i) {
          const int g = ct + i * kQ8Threads;
          // K-major: row = output feature; MN-major: box of 64 N columns, row = K
          const int box = BMN ? g / 256 : 0;
          const int srow = BMN ? (g >> 2) & 63 : g >> 2;
          const int part = g & 3;  // codes [16 part, 16 part + 16) of the row
          // exact int8 -> fp16: bias each code to 0..255, place it in the low
          // byte of fp16 1024 (0x6400 | u = 1024 + u) and subtract 1152
          const uint32_t w4[4] = {static_cast<uint32_t>(raw[i].x) ^ 0x80808080u,
                                  static_cast<uint32_t>(raw[i].y) ^ 0x80808080u,
                                  static_cast<uint32_t>(raw[i].z) ^ 0x80808080u,
                                  static_cast<uint32_t>(raw[i].w) ^ 0x80808080u};
          const __half2 bias = __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480));  // 1152
          uint32_t h[8];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const uint32_t lo = __byte_perm(w4[e], 0x64646464u, 0x4140);
            const uint32_t hi = __byte_perm(w4[e], 0x64646464u, 0x4342);
            const __half2 a0 = __hsub2(*reinterpret_cast<const __half2*>(&lo), bias);
            const __half2 a1 = __hsub2(*reinterpret_cast<const __half2*>(&hi), bias);
            h[2 * e] = *reinterpret_cast<const uint32_t*>(&a0);
            h[2 * e + 1] = *reinterpret_cast<const uint32_t*>(&a1);
          }
          // 16-byte chunks 2 part, 2 part + 1 of the 128-byte row, swizzled by row % 8
          const uint32_t rowp = sb32 + (BMN ? box * kMnBox : 0) + srow * 128;
          const int c0 = 2 * part, c1 = 2 * part + 1;
          asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(rowp + ((c0 ^ (srow & 7)) << 4)), "r"(h[0]),
                       "r"(h[1]), "r"(h[2]), "r"(h[3])
                       : "memory");
          asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(rowp + ((c1 ^ (srow & 7)) << 4)), "r"(h[4]),
                       "r"(h[5]), "r"(h[6]), "r"(h[7])
                       : "memory");
        }
        // generic-proxy writes -> visible to the tensor cores, then one arrival per CTA
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        asm volatile("bar.sync 1, %0;" ::"n"(kQ8Threads) : "memory");
        if (ct == 0) {
          if constexpr (CG == 2)
            mbar_arrive_cluster(mapa_shared(smem_u32(&full[s]), 0));
          else
            mbar_arrive(&full[s]);
        }
      }
    }
  } else {
    // -------------------------------------------------------------- epilogue
    static_assert(EW == 4 || EW == 8, "4 or 8 epilogue warps");
    constexpr int kGroups = EW / 4;           // warps sharing one lane quadrant
    constexpr int kCols = BN / kGroups;       // accumulator columns per warp
    constexpr int kChunk = Epi::kChunk;
    static_assert(kCols % kChunk == 0 || Epi::kPaired, "column slice must hold whole chunks");
    static_assert(!epi_tmem_direct<Epi>::value || kCols == Epi::kChunk, "direct epilogues take whole slices");
    const int ew = warp & 3;                  // TMEM lane quadrant this warp may access
    const int cgrp = (warp - 2) / 4;          // which column slice of the tile
    const uint32_t lane_off = static_cast<uint32_t>(ew * 32) << 16;
    EpiCtx c;
    c.lane = lane;
    c.M = sh.M;
    c.N = sh.N;
    c.slab = smem_u32(smem + L::kSlabOffset + (warp - 2) * Epi::kSlab);
    c.bar = &slab_bar[warp - 2];
    c.phase = 0;
    c.abort_flag = abort_flag;
    c.err = err;
    c.mapC = &tmC;
    c.mapD = &tmD;
    c.n_main = sh.n_main;
    c.fixup = sh.fixup;
    c.side = sh.side;
    c.ld_side = sh.ld_side;
    c.col_scale = (Q8 && !BMN) ? sh.b_scale : nullptr;
    int i = 0;
    bool ok = true;
    for (int u = unit0; u < num_units && ok; u += ustep, ++i) {
      const int acc = i & 1;
      const int tile = u % sh.num_tiles;
      const int sp = u / sh.num_tiles;
      const int tm = sh.n_fastest ? tile / sh.tiles_n : tile % sh.tiles_m;
      const int tn = sh.n_fastest ? tile % sh.tiles_n : tile / sh.tiles_m;
      // split s -> its row block of partials; the odd CTA of a pair owns rows 128..255
      c.row0 = (sp * sh.split_row_tiles + tm) * kRowsPerTile + static_cast<int>(rank) * kBlockM + ew * 32;
      c.row = c.row0 + lane;
      const uint32_t tbase = tmem_base + lane_off + acc * BN;
      typename Epi::State st;
      const int slot = tn * kGroups + cgrp;  // per-(tile, column slice) id for row-state epilogues
      // begin() runs before the accumulator is ready: epilogues that read
      // global inputs start fetching them here
      if constexpr (epi_begin_col<Epi>::value)
        Epi::begin(st, ep, c, slot, tn * BN + cgrp * kCols);
      else
        Epi::begin(st, ep, c, slot);
      if (!mbar_wait(&acc_full[acc], (i >> 1) & 1, abort_flag, err, kErrWaitAccum)) {
        if constexpr (epi_drain<Epi>::value) Epi::drain(st, c);  // copies begin() issued
        break;
      }
      tc_fence_after();
      bool run = true;  // false: another K split of this tile finishes it
      if (sh.fixup) {
        // this warp's slice of the tile: kSliceCols accumulator columns, in
        // 32-column chunks (the paired epilogue reads gate columns and the
        // matching up columns 128 further)
        constexpr int kSliceCols = BN / kGroups;
        auto col_of = [&](int q) -> int {
          if constexpr (Epi::kPaired) {
            constexpr int kPairChunks = 128 / kGroups / 32;
            return q < kPairChunks ? cgrp * (128 / kGroups) + 32 * q : 128 + cgrp * (128 / kGroups) + 32 * (q - kPairChunks);
          } else {
            return cgrp * kSliceCols + 32 * q;
          }
        };
        const int wslot = ((tile * CG + static_cast<int>(rank)) * 4 + ew) * kGroups + cgrp;
        // a split's partial: [chunk q][column quad][lane] float4, so that
        // each warp access moves 512 contiguous bytes
        float4* wsb = reinterpret_cast<float4*>(sh.fx_ws) + static_cast<size_t>(wslot) * sh.splits * (8 * kSliceCols);
        float4* mine = wsb + static_cast<size_t>(sp) * (8 * kSliceCols);
#pragma unroll 1
        for (int q = 0; q < kSliceCols / 32; ++q) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(tbase + col_of(q), v);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 8; ++j)
            __stcg(mine + (8 * q + j) * 32 + lane, make_float4(__uint_as_float(v[4 * j]), __uint_as_float(v[4 * j + 1]),
                                                              __uint_as_float(v[4 * j + 2]), __uint_as_float(v[4 * j + 3])));
        }
        __threadfence();
        __syncwarp();
        int prev = 0;
        if (lane == 0) prev = atomicAdd(sh.fx_cnt + wslot, 1);
        prev = __shfl_sync(0xffffffffu, prev, 0);
        run = prev == sh.splits - 1;
        if (run) {
          __threadfence();
          // every split's partial (this one's included), summed in split
          // order into the accumulator: the same bits whichever split is last
#pragma unroll 1
          for (int q = 0; q < kSliceCols / 32; ++q) {
            float4 a[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) a[j] = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int s2 = 0; s2 < sh.splits; ++s2) {
              const float4* o = wsb + static_cast<size_t>(s2) * (8 * kSliceCols) + 8 * q * 32 + lane;
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                const float4 t = __ldcg(o + 32 * j);
                a[j].x += t.x;
                a[j].y += t.y;
                a[j].z += t.z;
                a[j].w += t.w;
              }
            }
            uint32_t v[32];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              v[4 * j] = __float_as_uint(a[j].x);
              v[4 * j + 1] = __float_as_uint(a[j].y);
              v[4 * j + 2] = __float_as_uint(a[j].z);
              v[4 * j + 3] = __float_as_uint(a[j].w);
            }
            tmem_st_32x32b_x32(tbase + col_of(q), v);
          }
          tmem_st_wait();
          if (lane == 0) sh.fx_cnt[wslot] = 0;  // ready for the next launch
        }
      }
      if (!run) {
        // nothing to store for this unit
      } else if constexpr (epi_tmem_direct<Epi>::value) {
        ok = Epi::tile(st, ep, c, tn * BN + cgrp * kCols, tbase + cgrp * kCols, slot);
      } else if constexpr (!Epi::kPaired) {
#pragma unroll 1
        for (int cc = cgrp * kCols; cc < (cgrp + 1) * kCols && ok; cc += kChunk) {
          float v[kChunk];
#pragma unroll
          for (int q = 0; q < kChunk / 32; ++q)
            tmem_ld_32x32b_x32(tbase + cc + 32 * q, *reinterpret_cast<uint32_t(*)[32]>(v + 32 * q));
          tmem_ld_wait();
          ok = Epi::chunk(st, ep, c, tn * BN + cc, v);
        }
      } else {
        static_assert(BN == 256, "paired epilogue needs 256-wide tiles");
        constexpr int kPairCols = 128 / kGroups;
#pragma unroll 1
        for (int cc = cgrp * kPairCols; cc < (cgrp + 1) * kPairCols && ok; cc += kChunk) {
          float g[kChunk], u[kChunk];
#pragma unroll
          for (int q = 0; q < kChunk / 32; ++q) {
            tmem_ld_32x32b_x32(tbase + cc + 32 * q, *reinterpret_cast<uint32_t(*)[32]>(g + 32 * q));
            tmem_ld_32x32b_x32(tbase + 128 + cc + 32 * q, *reinterpret_cast<uint32_t(*)[32]>(u + 32 * q));
          }
          tmem_ld_wait();
          ok = Epi::pair(st, ep, c, tn, cc, g, u);
        }
      }
      if (run) Epi::end(st, ep, c, slot);
      tc_fence_before();
      if constexpr (CG == 2)
        mbar_arrive_cluster(mapa_shared(smem_u32(&acc_empty[acc]), 0));
      else
        mbar_arrive(&acc_empty[acc]);
    }
    if (Epi::kStores && lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
    __syncwarp();
  }

  tc_fence_before();
  if constexpr (CG == 2)
    cluster_sync_all();  // the peer's MMAs, barriers and TMEM stay live until both CTAs are done
  else
    __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    if constexpr (CG == 2)
      tmem_dealloc_pair(tmem_base, L::kTmemCols);
    else
      tmem_dealloc(tmem_base, L::kTmemCols);
  }
}

}  // namespace llmcu
