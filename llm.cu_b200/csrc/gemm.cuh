// gemm.cuh -- persistent, warp-specialised tcgen05 GEMM for sm_100a.
//
//   C[M, N] = A0[M, K0] . B0[N, K0]^T  (+ A1[M, K1] . B1[N, K1]^T)
//
// fp16 operands, both K-major (rows contiguous along K), fp32 accumulation in
// TMEM, and a fused epilogue chosen at compile time.  The optional second
// K-segment (A1, B1) carries the LoRA term: appending [h | 2B] to [x | W] turns
// y = xW^T + 2(xA^T)B^T into one accumulation, so the adapter update costs one
// extra 64-wide K block instead of a separate GEMM and an add pass.
//
// Roles (192 threads, one CTA per SM):
//   warp 0      TMA producer  -- fills a STAGES-deep ring of (A, B) smem tiles
//   warp 1      MMA issuer    -- tcgen05.mma into one of two TMEM accumulators
//                               (allocates / frees TMEM for the CTA)
//   warps 2..5  epilogue      -- tcgen05.ld -> registers -> fused op -> global
// Tiles: BLOCK_M = 128 rows, BLOCK_N = BN (64/128/256), BLOCK_K = 64 (one
// 128-byte swizzle row of fp16).  Tile t -> (t % tiles_m, t / tiles_m), so
// CTAs that run together share the weight (B) tile and stream it once.
#pragma once

#include "sm100.cuh"

namespace llmcu {

struct GemmShape {
  int M, N;
  int K0, K1;      // K of segment 0 and of the optional segment 1 (0 = none)
  int tiles_m, tiles_n, num_tiles;
};

constexpr int kGemmThreads = 192;
constexpr int kBlockM = 128;
constexpr int kBlockK = 64;

template <int BN, int STAGES>
struct GemmSmem {
  static constexpr int kABytes = kBlockM * kBlockK * 2;       // 16 KB
  static constexpr int kBBytes = BN * kBlockK * 2;            // 8/16/32 KB
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kTmemCols = (2 * BN < 32) ? 32 : 2 * BN;  // two accumulators
  static constexpr int kBarOffset = STAGES * kStageBytes;
  static constexpr int kBytes = kBarOffset + 256 + 1024;       // + barriers + alignment slack
};

// ----------------------------------------------------------------- epilogues
// An epilogue sees one row (`row`, < M guaranteed only via the check below)
// and 32 consecutive accumulator columns starting at `col0`.

struct EpiStoreF16 {
  struct Params { __half* C; int ldc; };
  struct State {};
  static constexpr bool kPaired = false;
  __device__ static void begin(State&, const Params&, int, int) {}
  __device__ static void chunk(State&, const Params& p, int row, int col0, int M, int N, const float* v) {
    if (row >= M) return;
    __half* dst = p.C + static_cast<size_t>(row) * p.ldc + col0;
    if (col0 + 32 <= N) {
#pragma unroll
      for (int j = 0; j < 32; j += 8) {
        uint4 w;
        w.x = pack_half2(v[j + 0], v[j + 1]);
        w.y = pack_half2(v[j + 2], v[j + 3]);
        w.z = pack_half2(v[j + 4], v[j + 5]);
        w.w = pack_half2(v[j + 6], v[j + 7]);
        *reinterpret_cast<uint4*>(dst + j) = w;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (col0 + j < N) dst[j] = __float2half_rn(v[j]);
    }
  }
  __device__ static void end(State&, const Params&, int, int, int) {}
};

// C = acc (fp32), or C += acc when accumulate != 0.
struct EpiStoreF32 {
  struct Params { float* C; int ldc; int accumulate; };
  struct State {};
  static constexpr bool kPaired = false;
  __device__ static void begin(State&, const Params&, int, int) {}
  __device__ static void chunk(State&, const Params& p, int row, int col0, int M, int N, const float* v) {
    if (row >= M) return;
    float* dst = p.C + static_cast<size_t>(row) * p.ldc + col0;
    if (col0 + 32 <= N) {
#pragma unroll
      for (int j = 0; j < 32; j += 4) {
        float4 w = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
        if (p.accumulate) {
          float4 o = *reinterpret_cast<const float4*>(dst + j);
          w.x += o.x; w.y += o.y; w.z += o.z; w.w += o.w;
        }
        *reinterpret_cast<float4*>(dst + j) = w;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (col0 + j < N) dst[j] = p.accumulate ? dst[j] + v[j] : v[j];
    }
  }
  __device__ static void end(State&, const Params&, int, int, int) {}
};

// out = acc + resid (fp32): the residual adds of the O and down projections
// (src/kernels/lora_forward.cu:265,297).
struct EpiResidF32 {
  struct Params { float* out; const float* resid; int ld; };
  struct State {};
  static constexpr bool kPaired = false;
  __device__ static void begin(State&, const Params&, int, int) {}
  __device__ static void chunk(State&, const Params& p, int row, int col0, int M, int N, const float* v) {
    if (row >= M) return;
    const size_t base = static_cast<size_t>(row) * p.ld + col0;
    if (col0 + 32 <= N) {
#pragma unroll
      for (int j = 0; j < 32; j += 4) {
        float4 r = *reinterpret_cast<const float4*>(p.resid + base + j);
        *reinterpret_cast<float4*>(p.out + base + j) =
            make_float4(v[j] + r.x, v[j + 1] + r.y, v[j + 2] + r.z, v[j + 3] + r.w);
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (col0 + j < N) p.out[base + j] = v[j] + p.resid[base + j];
    }
  }
  __device__ static void end(State&, const Params&, int, int, int) {}
};

__device__ __forceinline__ float silu_f(float g) { return g / (1.0f + __expf(-g)); }

// Gate/up GEMM with SwiGLU (src/kernels/activation.cu:5-11).  The fused
// weight interleaves 128-row blocks of W_gate and W_up, so a 256-wide tile
// holds gate columns [0,128) and the matching up columns [128,256).  Writes
// the pre-activations (kept for the backward) and act = silu(g) * u.
struct EpiSwiGLU {
  struct Params { __half* gu; int ld_gu; __half* act; int ld_act; };
  struct State {};
  static constexpr bool kPaired = true;  // requires BN == 256
  __device__ static void begin(State&, const Params&, int, int) {}
  // g: columns [col0, col0+32) of the gate half, u: the matching up columns.
  __device__ static void pair(State&, const Params& p, int row, int tile_n, int c, int M, const float* g,
                              const float* u) {
    if (row >= M) return;
    __half* gdst = p.gu + static_cast<size_t>(row) * p.ld_gu + tile_n * 256 + c;
    __half* udst = gdst + 128;
    __half* adst = p.act + static_cast<size_t>(row) * p.ld_act + tile_n * 128 + c;
#pragma unroll
    for (int j = 0; j < 32; j += 8) {
      uint4 wg, wu, wa;
      wg.x = pack_half2(g[j], g[j + 1]); wg.y = pack_half2(g[j + 2], g[j + 3]);
      wg.z = pack_half2(g[j + 4], g[j + 5]); wg.w = pack_half2(g[j + 6], g[j + 7]);
      wu.x = pack_half2(u[j], u[j + 1]); wu.y = pack_half2(u[j + 2], u[j + 3]);
      wu.z = pack_half2(u[j + 4], u[j + 5]); wu.w = pack_half2(u[j + 6], u[j + 7]);
      float a[8];
#pragma unroll
      for (int t = 0; t < 8; ++t) a[t] = silu_f(g[j + t]) * u[j + t];
      wa.x = pack_half2(a[0], a[1]); wa.y = pack_half2(a[2], a[3]);
      wa.z = pack_half2(a[4], a[5]); wa.w = pack_half2(a[6], a[7]);
      *reinterpret_cast<uint4*>(gdst + j) = wg;
      *reinterpret_cast<uint4*>(udst + j) = wu;
      *reinterpret_cast<uint4*>(adst + j) = wa;
    }
  }
  __device__ static void end(State&, const Params&, int, int, int) {}
};

// Down-projection dX with the SwiGLU backward fused (src/kernels/activation.cu:26-38):
// acc = d_act[row, i]; reads g, u from the interleaved stash and writes
// dg, du into the same interleaved layout (the A operand of the gate/up dX GEMM).
struct EpiSwiGLUBwd {
  struct Params { const __half* gu; __half* dgu; int ld; };
  struct State {};
  static constexpr bool kPaired = false;
  __device__ static void begin(State&, const Params&, int, int) {}
  __device__ static void chunk(State&, const Params& p, int row, int col0, int M, int N, const float* v) {
    if (row >= M || col0 >= N) return;
    // col0 is a multiple of 32, so the 32 columns share one 128-block.
    const int gcol = (col0 >> 7) * 256 + (col0 & 127);
    const size_t base = static_cast<size_t>(row) * p.ld + gcol;
#pragma unroll
    for (int j = 0; j < 32; j += 8) {
      uint4 gr = *reinterpret_cast<const uint4*>(p.gu + base + j);
      uint4 ur = *reinterpret_cast<const uint4*>(p.gu + base + 128 + j);
      const __half* gh = reinterpret_cast<const __half*>(&gr);
      const __half* uh = reinterpret_cast<const __half*>(&ur);
      float dg[8], du[8];
#pragma unroll
      for (int t = 0; t < 8; ++t) {
        const float g = __half2float(gh[t]);
        const float u = __half2float(uh[t]);
        const float sig = 1.0f / (1.0f + __expf(-g));
        const float dy = v[j + t];
        dg[t] = dy * u * sig * (1.0f + g * (1.0f - sig));
        du[t] = dy * g * sig;
      }
      uint4 wg, wu;
      wg.x = pack_half2(dg[0], dg[1]); wg.y = pack_half2(dg[2], dg[3]);
      wg.z = pack_half2(dg[4], dg[5]); wg.w = pack_half2(dg[6], dg[7]);
      wu.x = pack_half2(du[0], du[1]); wu.y = pack_half2(du[2], du[3]);
      wu.z = pack_half2(du[4], du[5]); wu.w = pack_half2(du[6], du[7]);
      *reinterpret_cast<uint4*>(p.dgu + base + j) = wg;
      *reinterpret_cast<uint4*>(p.dgu + base + 128 + j) = wu;
    }
  }
  __device__ static void end(State&, const Params&, int, int, int) {}
};

// lm_head pass 1 (src/kernels/loss.cu:24-61 without the [M,V] logits tensor):
// per row and vocab tile, the running max and sum of exp of the logits, plus
// the target logit when the target falls in this tile.
struct EpiCEStats {
  struct Params {
    const int* targets;   // [M]
    float* part_max;      // [M, tiles_n]
    float* part_sum;      // [M, tiles_n]
    float* tgt_logit;     // [M]
    int tiles_n;
  };
  struct State { float m, s; int t; };
  static constexpr bool kPaired = false;
  __device__ static void begin(State& st, const Params& p, int row, int) {
    st.m = -INFINITY;
    st.s = 0.0f;
    st.t = -1;
    (void)p;
    (void)row;
  }
  __device__ static void chunk(State& st, const Params& p, int row, int col0, int M, int N, const float* v) {
    if (row >= M || col0 >= N) return;
    if (st.t < 0) st.t = __ldg(p.targets + row);
    const int nv = min(32, N - col0);
    float cm = -INFINITY;
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (j < nv) cm = fmaxf(cm, v[j]);
    const float mn = fmaxf(st.m, cm);
    float s = st.s * fast_exp2((st.m - mn) * kLog2e);
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (j < nv) s += fast_exp2((v[j] - mn) * kLog2e);
    st.m = mn;
    st.s = s;
    const int tj = st.t - col0;
    if (tj >= 0 && tj < nv) {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (j == tj) p.tgt_logit[row] = v[j];
    }
  }
  __device__ static void end(State& st, const Params& p, int row, int tile_n, int M) {
    if (row >= M) return;
    p.part_max[static_cast<size_t>(row) * p.tiles_n + tile_n] = st.m;
    p.part_sum[static_cast<size_t>(row) * p.tiles_n + tile_n] = st.s;
  }
};

// lm_head pass 2: dlogits tile = gscale * (softmax - onehot) for rows that
// count in the loss, 0 for the others; written fp16 into a vocab chunk buffer
// (columns relative to the chunk start).
struct EpiCEGrad {
  struct Params {
    const int* targets;    // [M]
    const float* lse;      // [M] natural-log LSE
    const uint8_t* valid;  // [M] 1 if the row counts in the loss
    __half* dl;            // [M, ld] chunk buffer, columns relative to the chunk
    int ld;
    int col_base;          // vocab id of the chunk's first column
    float gscale;
  };
  struct State { float lse2; int t; int ok; };
  static constexpr bool kPaired = false;
  __device__ static void begin(State& st, const Params& p, int row, int) {
    st.ok = 0;
    (void)p;
    (void)row;
  }
  __device__ static void chunk(State& st, const Params& p, int row, int col0, int M, int N, const float* v) {
    if (row >= M || col0 >= N) return;
    if (!st.ok) {
      st.ok = p.valid[row] ? 1 : 2;
      st.t = __ldg(p.targets + row);
      st.lse2 = p.lse[row] * kLog2e;
    }
    __half* dst = p.dl + static_cast<size_t>(row) * p.ld + col0;
    const int nv = min(32, N - col0);
    const int tl = st.t - p.col_base - col0;  // target column relative to this chunk of 32
    float d[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      float pr = fast_exp2(v[j] * kLog2e - st.lse2);
      if (j == tl) pr -= 1.0f;
      d[j] = (st.ok == 1) ? pr * p.gscale : 0.0f;
    }
    if (nv == 32) {
#pragma unroll
      for (int j = 0; j < 32; j += 8) {
        uint4 w;
        w.x = pack_half2(d[j], d[j + 1]); w.y = pack_half2(d[j + 2], d[j + 3]);
        w.z = pack_half2(d[j + 4], d[j + 5]); w.w = pack_half2(d[j + 6], d[j + 7]);
        *reinterpret_cast<uint4*>(dst + j) = w;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (j < nv) dst[j] = __float2half_rn(d[j]);
    }
  }
  __device__ static void end(State&, const Params&, int, int, int) {}
};

// ---------------------------------------------------------------- the kernel

template <int BN, int STAGES, class Epi>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA0, const __grid_constant__ CUtensorMap tmB0,
                   const __grid_constant__ CUtensorMap tmA1, const __grid_constant__ CUtensorMap tmB1,
                   const GemmShape sh, const typename Epi::Params ep, int* err) {
  using L = GemmSmem<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBarOffset);
  uint64_t* full = bars;                    // [STAGES]
  uint64_t* empty = bars + STAGES;          // [STAGES]
  uint64_t* acc_full = bars + 2 * STAGES;   // [2]
  uint64_t* acc_empty = acc_full + 2;       // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 128);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA0);
    tma_prefetch_desc(&tmB0);
    if (sh.K1 > 0) {
      tma_prefetch_desc(&tmA1);
      tma_prefetch_desc(&tmB1);
    }
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, L::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int nk0 = (sh.K0 + kBlockK - 1) / kBlockK;
  const int nk1 = (sh.K1 + kBlockK - 1) / kBlockK;
  const int nk = nk0 + nk1;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ producer
      int it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < sh.num_tiles && ok; tile += gridDim.x) {
        const int tm = tile % sh.tiles_m;
        const int tn = tile / sh.tiles_m;
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t par = ((it / STAGES) & 1) ^ 1;
          if (!mbar_wait(&empty[s], par, abort_flag, err, kErrWaitConsumer)) { ok = false; break; }
          uint8_t* sa = smem + s * L::kStageBytes;
          uint8_t* sb = sa + L::kABytes;
          mbar_arrive_expect_tx(&full[s], L::kStageBytes);
          if (kb < nk0) {
            tma_load_2d(sa, &tmA0, &full[s], kb * kBlockK, tm * kBlockM);
            tma_load_2d(sb, &tmB0, &full[s], kb * kBlockK, tn * BN);
          } else {
            const int k = (kb - nk0) * kBlockK;
            tma_load_2d(sa, &tmA1, &full[s], k, tm * kBlockM);
            tma_load_2d(sb, &tmB1, &full[s], k, tn * BN);
          }
        }
      }
      if (!ok) {
        // Let the copies already issued land before the CTA can exit.
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
    if (lane == 0) {
      // ---------------------------------------------------------- MMA issuer
      constexpr uint32_t idesc = idesc_f16_f32(kBlockM, BN);
      int it = 0;
      int i = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < sh.num_tiles && ok; tile += gridDim.x, ++i) {
        const int acc = i & 1;
        if (!mbar_wait(&acc_empty[acc], ((i >> 1) & 1) ^ 1, abort_flag, err, kErrWaitEpilogue)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int s = it % STAGES;
          if (!mbar_wait(&full[s], (it / STAGES) & 1, abort_flag, err, kErrWaitProducer)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + s * L::kStageBytes);
          const uint32_t sb = sa + L::kABytes;
          const uint64_t adesc = sw128_kmajor_desc(sa);
          const uint64_t bdesc = sw128_kmajor_desc(sb);
#pragma unroll
          for (int k = 0; k < kBlockK / 16; ++k) {
            // +32 bytes per 16-element K step inside the 128-byte swizzle row
            umma_f16(d_tmem, adesc + 2 * k, bdesc + 2 * k, idesc, (kb | k) != 0 ? 1u : 0u);
          }
          umma_commit(&empty[s]);
        }
        if (ok) umma_commit(&acc_full[acc]);
      }
    }
  } else {
    // -------------------------------------------------------------- epilogue
    const int ew = warp & 3;  // TMEM lane quadrant this warp may access
    const uint32_t lane_off = static_cast<uint32_t>(ew * 32) << 16;
    int i = 0;
    for (int tile = blockIdx.x; tile < sh.num_tiles; tile += gridDim.x, ++i) {
      const int acc = i & 1;
      if (!mbar_wait(&acc_full[acc], (i >> 1) & 1, abort_flag, err, kErrWaitAccum)) break;
      tc_fence_after();
      const int tm = tile % sh.tiles_m;
      const int tn = tile / sh.tiles_m;
      const int row = tm * kBlockM + ew * 32 + lane;
      const uint32_t tbase = tmem_base + lane_off + acc * BN;
      typename Epi::State st;
      Epi::begin(st, ep, row, tn);
      if constexpr (!Epi::kPaired) {
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(tbase + c, r);
          tmem_ld_wait();
          Epi::chunk(st, ep, row, tn * BN + c, sh.M, sh.N, reinterpret_cast<const float*>(r));
        }
      } else {
        static_assert(BN == 256, "paired epilogue needs 256-wide tiles");
#pragma unroll 1
        for (int c = 0; c < 128; c += 32) {
          uint32_t rg[32], ru[32];
          tmem_ld_32x32b_x32(tbase + c, rg);
          tmem_ld_32x32b_x32(tbase + 128 + c, ru);
          tmem_ld_wait();
          Epi::pair(st, ep, row, tn, c, sh.M, reinterpret_cast<const float*>(rg),
                    reinterpret_cast<const float*>(ru));
        }
      }
      Epi::end(st, ep, row, tn, sh.M);
      tc_fence_before();
      mbar_arrive(&acc_empty[acc]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, L::kTmemCols);
  }
}

}  // namespace llmcu
