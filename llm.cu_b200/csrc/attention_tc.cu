// attention_tc.cu -- causal GQA flash attention on tcgen05 / TMEM (forward and backward).
//
// Forward: one CTA per (128-row query tile, query head, sequence), 192
// threads, two CTAs per SM (96 KB of shared memory and 256 TMEM columns
// each), so one CTA's softmax overlaps the other's MMAs:
//   warp 0     TMA producer: Q once, then K_j and V_j, each single-buffered
//              and refilled as soon as the MMA that reads it completes
//   warp 1     MMA issuer:   S_j = Q K_j^T (SS form), then O += P_j V_j with P
//                            read from tensor memory (TS form)
//   warps 2-5  softmax:      thread r owns query row r: one pass over S_j in
//                            TMEM for the row max, one for exp / sum, writing
//                            P_j (fp16 pairs) back over the consumed S columns;
//                            keeps the running max / sum in registers and
//                            rescales its O row in TMEM only when the max grew
//                            by more than 2^8 (P stays < 256, exact in fp16)
// TMEM: S_j / P_j [0,128), O [128, 128+hd).  P V uses V as an MN-major
// operand (head_dim contiguous), so no transposed copy of V is made.
// Writes O (fp16) and the per-row log-sum-exp; P never leaves the SM.
// Replaces naive_attn_kernel (src/kernels/lora_forward.cu:48-135).
#include <cudaTypedefs.h>

#include "common.cuh"

namespace llmcu {

namespace {

constexpr int kTq = 128;  // query rows per CTA
constexpr int kTk = 128;  // key rows per tile
constexpr int kBox = 128 * 64 * 2;  // one [128 rows x 64 fp16] TMA box, 16 KB

template <int HD>
struct FwdLayout {
  static constexpr int kQ = kTq * HD * 2;
  static constexpr int kKV = kTk * HD * 2;
  static constexpr int kQOff = 0;
  static constexpr int kKOff = kQOff + kQ;
  static constexpr int kVOff = kKOff + kKV;
  static constexpr int kBarOff = kVOff + kKV;
  static constexpr int kBytes = kBarOff + 128 + 1024;
  static constexpr int kTmemCols = 256;  // S / P 128 + O hd
};

// MN-major (column-contiguous) 128-byte-swizzled operand: 64-element rows of
// 128 B, 8-row atoms of 1 KB stacked along K (stride byte offset 1 KB), the
// next 64 columns one 16 KB box further (leading byte offset).
__device__ __forceinline__ uint64_t sw128_mnmajor_desc(uint32_t smem_addr) { return sw128_mn_desc(smem_addr, kBox); }

template <int HD>
__global__ void __launch_bounds__(192, 2)
    attn_fwd_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV, __half* __restrict__ o, float* __restrict__ lse,
                       int S, int nh, int nkv, int ldo, float scale_log2, int* err) {
  using L = FwdLayout<HD>;
  constexpr int kDBoxes = HD / 64;  // 64-wide boxes along head_dim
  pdl_trigger();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* k_empty = bars + 2;
  uint64_t* v_full = bars + 3;
  uint64_t* v_empty = bars + 4;
  uint64_t* s_full = bars + 5;
  uint64_t* p_full = bars + 6;
  uint64_t* pv_done = bars + 7;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // blocks start in linear order (x fastest): every (head, sequence) of the
  // longest causal query tile first, so short tiles fill the last wave
  const int qt = gridDim.z - 1 - blockIdx.z;
  const int h = blockIdx.x, b = blockIdx.y;
  const int kvh = h / (nh / nkv);
  const int n_kv = qt + 1;
  const int row_base = b * S;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(k_full, 1);
    mbar_init(k_empty, 1);
    mbar_init(v_full, 1);
    mbar_init(v_empty, 1);
    mbar_init(s_full, 1);
    mbar_init(p_full, 128);
    mbar_init(pv_done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, L::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_wait();  // the prologue above overlapped the previous kernel's tail
  const uint32_t t_s = tmem, t_o = tmem + 128;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ producer
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      mbar_arrive_expect_tx(q_full, L::kQ);
      for (int i = 0; i < kDBoxes; ++i)
        tma_load_2d(smem + L::kQOff + i * kBox, &tmQ, q_full, h * HD + 64 * i, row_base + qt * kTq);
      bool ok = true;
      int jk = -1, jv = -1;  // last K / V tile issued
      for (int j = 0; j < n_kv && ok; ++j) {
        // K_j once S_{j-1} has read K_{j-1}; V_j once P_{j-1} V_{j-1} has read V_{j-1}
        if (j >= 1 && !mbar_wait(k_empty, (j - 1) & 1, abort_flag, err, kErrWaitConsumer)) { ok = false; break; }
        mbar_arrive_expect_tx(k_full, L::kKV);
        for (int i = 0; i < kDBoxes; ++i)
          tma_load_2d(smem + L::kKOff + i * kBox, &tmK, k_full, kvh * HD + 64 * i, row_base + j * kTk);
        jk = j;
        if (j >= 1 && !mbar_wait(v_empty, (j - 1) & 1, abort_flag, err, kErrWaitConsumer)) { ok = false; break; }
        mbar_arrive_expect_tx(v_full, L::kKV);
        for (int i = 0; i < kDBoxes; ++i)
          tma_load_2d(smem + L::kVOff + i * kBox, &tmV, v_full, kvh * HD + 64 * i, row_base + j * kTk);
        jv = j;
      }
      if (!ok) {  // let the copies already issued land before the CTA can exit
        mbar_drain(q_full, 0);
        if (jk >= 0) mbar_drain(k_full, jk & 1);
        if (jv >= 0) mbar_drain(v_full, jv & 1);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------------------------------------------------- MMA issuer
      constexpr uint32_t idesc_s = idesc_f16_f32(kTq, kTk);
      constexpr uint32_t idesc_pv = idesc_f16_f32(kTq, HD) | (1u << 16);  // B (V) MN-major
      const uint32_t sq = smem_u32(smem + L::kQOff);
      const uint32_t sk = smem_u32(smem + L::kKOff);
      const uint32_t sv = smem_u32(smem + L::kVOff);
      bool ok = mbar_wait(q_full, 0, abort_flag, err, kErrWaitProducer);
      for (int j = 0; j < n_kv && ok; ++j) {
        // S_j overwrites P_{j-1}, which the P V MMA issued before it has read (in order)
        if (!mbar_wait(k_full, j & 1, abort_flag, err, kErrWaitProducer)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < HD / 16; ++k) {
          const uint64_t adesc = sw128_kmajor_desc(sq + (k >> 2) * kBox + (k & 3) * 32);
          const uint64_t bdesc = sw128_kmajor_desc(sk + (k >> 2) * kBox + (k & 3) * 32);
          umma_f16(t_s, adesc, bdesc, idesc_s, k > 0 ? 1u : 0u);
        }
        umma_commit(s_full);
        umma_commit(k_empty);
        if (!mbar_wait(p_full, j & 1, abort_flag, err, kErrWaitAccum)) { ok = false; break; }
        if (!mbar_wait(v_full, j & 1, abort_flag, err, kErrWaitProducer)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < kTk / 16; ++k) {
          // P columns [16k, 16k + 16) are 32-bit TMEM columns [8k, 8k + 8)
          const uint64_t bdesc = sw128_mnmajor_desc(sv + k * 16 * 128);
          umma_f16_ts(t_o, t_s + 8 * k, bdesc, idesc_pv, (j > 0 || k > 0) ? 1u : 0u);
        }
        umma_commit(pv_done);
        umma_commit(v_empty);
      }
    }
  } else {
    // ------------------------------------------------------------- softmax
    const int qd = warp & 3;                 // TMEM lane quadrant
    const int r = qd * 32 + lane;            // query row within the tile
    const int q = qt * kTq + r;              // query position in the sequence
    const uint32_t lane_off = static_cast<uint32_t>(qd * 32) << 16;
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < n_kv && ok; ++j) {
      if (!mbar_wait(s_full, j & 1, abort_flag, err, kErrWaitAccum)) { ok = false; break; }
      tc_fence_after();
      const int kv0 = j * kTk;
      // every key of the tile before every query of this CTA, all inside the
      // sequence: no masking (and a finite row max)
      const bool interior = j < qt && kv0 + kTk <= S;
      // masked tiles: key kv0 + i is visible to row q iff i <= lim (causal and
      // inside the sequence); one compare and a select per score, no branch
      const int lim = min(q, S - 1) - kv0;
      // pass 1: row max of the scaled, masked scores
      float mx = -INFINITY;
#pragma unroll 1
      for (int c = 0; c < kTk / 32; ++c) {
        float sv[32];
        tmem_ld_32x32b_x32(t_s + lane_off + 32 * c, *reinterpret_cast<uint32_t(*)[32]>(sv));
        tmem_ld_wait();
        if (interior) {
#pragma unroll
          for (int i = 0; i < 32; ++i) mx = fmaxf(mx, sv[i] * scale_log2);
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) mx = fmaxf(mx, 32 * c + i <= lim ? sv[i] * scale_log2 : -INFINITY);
        }
      }
      const float m_new = fmaxf(m_used, mx);
      const bool resc = (j > 0) && (m_new > m_used + 8.0f);
      const float m_next = (j == 0 || resc) ? m_new : m_used;
      const float corr = resc ? fast_exp2(m_used - m_next) : 1.0f;
      // pass 2: P = exp2(s - m) as fp16 pairs over the S columns already read
      // (chunk c of 32 scores -> P columns [16c, 16c + 16), below 32c)
      float rs = 0.f;
#pragma unroll 1
      for (int c = 0; c < kTk / 32; ++c) {
        float sv[32];
        tmem_ld_32x32b_x32(t_s + lane_off + 32 * c, *reinterpret_cast<uint32_t(*)[32]>(sv));
        tmem_ld_wait();
        uint32_t pk[16];
        if (interior) {
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float p0 = fast_exp2(fmaf(sv[2 * i], scale_log2, -m_next));
            const float p1 = fast_exp2(fmaf(sv[2 * i + 1], scale_log2, -m_next));
            rs += p0 + p1;
            pk[i] = pack_half2(p0, p1);
          }
        } else {
          // no visible key yet (m_next = -inf): every P of the row is zero
          const int lim_c = (m_next == -INFINITY ? -1 : lim) - 32 * c;
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            float p0 = fast_exp2(fmaf(sv[2 * i], scale_log2, -m_next));
            float p1 = fast_exp2(fmaf(sv[2 * i + 1], scale_log2, -m_next));
            p0 = 2 * i <= lim_c ? p0 : 0.f;
            p1 = 2 * i + 1 <= lim_c ? p1 : 0.f;
            rs += p0 + p1;
            pk[i] = pack_half2(p0, p1);
          }
        }
        tmem_st_32x32b_x16(t_s + lane_off + 16 * c, pk);
      }
      l = l * corr + rs;
      m_used = m_next;
      if (j >= 1) {
        if (!mbar_wait(pv_done, (j - 1) & 1, abort_flag, err, kErrWaitAccum)) { ok = false; break; }
        tc_fence_after();
      }
      if (__any_sync(0xffffffffu, resc)) {
#pragma unroll 1
        for (int c = 0; c < HD / 32; ++c) {
          uint32_t ov[32];
          tmem_ld_32x32b_x32(t_o + lane_off + 32 * c, ov);
          tmem_ld_wait();
#pragma unroll
          for (int t = 0; t < 32; ++t) ov[t] = __float_as_uint(__uint_as_float(ov[t]) * corr);
          tmem_st_32x32b_x32(t_o + lane_off + 32 * c, ov);
        }
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(p_full);
    }
    if (ok && mbar_wait(pv_done, (n_kv - 1) & 1, abort_flag, err, kErrWaitAccum)) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.0f / l : 0.f;
      __half* orow = o + static_cast<size_t>(row_base + q) * ldo + h * HD;
#pragma unroll 1
      for (int c = 0; c < HD / 32; ++c) {
        uint32_t ov[32];
        tmem_ld_32x32b_x32(t_o + lane_off + 32 * c, ov);
        tmem_ld_wait();
        if (q < S) {
#pragma unroll
          for (int t = 0; t < 32; t += 8) {
            uint4 w;
            w.x = pack_half2(__uint_as_float(ov[t]) * inv, __uint_as_float(ov[t + 1]) * inv);
            w.y = pack_half2(__uint_as_float(ov[t + 2]) * inv, __uint_as_float(ov[t + 3]) * inv);
            w.z = pack_half2(__uint_as_float(ov[t + 4]) * inv, __uint_as_float(ov[t + 5]) * inv);
            w.w = pack_half2(__uint_as_float(ov[t + 6]) * inv, __uint_as_float(ov[t + 7]) * inv);
            *reinterpret_cast<uint4*>(orow + 32 * c + t) = w;
          }
        }
      }
      if (q < S) lse[(static_cast<size_t>(b) * nh + h) * S + q] = (m_used + __log2f(l)) * 0.69314718055994531f;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, L::kTmemCols);
  }
}

// ------------------------------------------------------------- backward
// One CTA per (128-row key tile, KV head, sequence), 320 threads:
//   warp 0     TMA producer: K, V once; then per iteration one (Q, dO) tile
//   warp 1     MMA issuer:   S^T = K Q^T and dP^T = V dO^T; then dV += P^T dO,
//                            dK += dS^T Q and dQ_part = dS K (dS read from the
//                            dS^T tile as an MN-major operand)
//   warps 2-9  softmax:      two warps per TMEM lane quadrant, each taking
//                            half of the columns (one CTA per SM: a single
//                            warp per scheduler would leave every latency of
//                            the exp / multiply chain exposed).  Thread r of
//                            a half owns key row r: P^T = exp(S^T - LSE),
//                            dS^T = P^T (dP^T - delta) into shared memory;
//                            then, as query row r, drains its half of
//                            dQ_part's columns into the global fp32 dQ with
//                            TMA reduce-add
// Iterations run over the query heads of the KV group and the query tiles at
// or after the key tile (causal).  TMEM: S^T [0,128), dP^T / dQ_part
// [128,256), dV [256, 256+hd), dK [256+hd, 256+2hd); the next S^T is issued
// while the softmax warps drain dQ_part.
template <int HD>
struct BwdLayout {
  static constexpr int kT = 128 * HD * 2;       // K, V, Q or dO tile
  static constexpr int kP = 128 * 128 * 2;      // P^T or dS^T tile
  static constexpr int kKOff = 0;
  static constexpr int kVOff = kKOff + kT;
  static constexpr int kQOff = kVOff + kT;
  static constexpr int kOOff = kQOff + kT;      // dO
  static constexpr int kPOff = kOOff + kT;      // P^T (later the dQ drain slabs)
  static constexpr int kSOff = kPOff + kP;      // dS^T
  static constexpr int kLOff = kSOff + kP;      // 2 x (lse*log2e [128], delta [128])
  static constexpr int kBarOff = kLOff + 4 * 128 * 4;
  static constexpr int kBytes = kBarOff + 256 + 1024;
};

constexpr int kBwdSoftmaxThreads = 256;

// P^T = exp(S^T - LSE) and dS^T = P^T (dP^T - delta) for one 32-column chunk
// (query columns 32c ..) of key row kr, packed to fp16 pairs.  kMasked: the
// causal diagonal tile or a ragged edge, where entries past the row's last
// query or the sequence are zero; interior tiles skip those tests.
template <bool kMasked>
__device__ __forceinline__ void bwd_softmax_chunk(const uint32_t (&sv)[32], const uint32_t (&dv)[32], const float* sLb,
                                                  const float* sDb, int c, float scale_log2, int q0, int kr, int S,
                                                  uint32_t (&pp)[16], uint32_t (&dsp)[16]) {
#pragma unroll
  for (int t = 0; t < 32; t += 4) {
    // the column statistics four at a time (16-byte aligned: 32c + t)
    const float4 l4 = *reinterpret_cast<const float4*>(sLb + 32 * c + t);
    const float4 d4 = *reinterpret_cast<const float4*>(sDb + 32 * c + t);
    const float lq[4] = {l4.x, l4.y, l4.z, l4.w};
    const float dq[4] = {d4.x, d4.y, d4.z, d4.w};
    float pv[4], dsv[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int qc = 32 * c + t + e;
      float p = fast_exp2(__uint_as_float(sv[t + e]) * scale_log2 - lq[e]);
      if (kMasked) {
        const int qq = q0 + qc;
        if (qq < kr || qq >= S || kr >= S) p = 0.f;
      }
      pv[e] = p;
      dsv[e] = p * (__uint_as_float(dv[t + e]) - dq[e]);
    }
    pp[t / 2] = pack_half2(pv[0], pv[1]);
    pp[t / 2 + 1] = pack_half2(pv[2], pv[3]);
    dsp[t / 2] = pack_half2(dsv[0], dsv[1]);
    dsp[t / 2 + 1] = pack_half2(dsv[2], dsv[3]);
  }
}
__device__ __forceinline__ void named_sync_softmax() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

template <int HD>
__global__ void __launch_bounds__(64 + kBwdSoftmaxThreads, 1)
    attn_bwd_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO,
                       const __grid_constant__ CUtensorMap tmDQ, const float* __restrict__ lse,
                       const float* __restrict__ delta, float* __restrict__ dk, __half* __restrict__ dv, int S,
                       int nh, int nkv, int lddk, int lddv, float scale, float scale_log2, int dq_slab_rows,
                       int* err) {
  using L = BwdLayout<HD>;
  constexpr int kDBoxes = HD / 64;
  pdl_trigger();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* kv_full = bars;
  uint64_t* q_full = bars + 1;
  uint64_t* q_free = bars + 2;
  uint64_t* s_full = bars + 3;
  uint64_t* p_full = bars + 4;
  uint64_t* dq_full = bars + 5;
  uint64_t* dq_free = bars + 6;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 7);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* sL = reinterpret_cast<float*>(smem + L::kLOff);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nkt = gridDim.z;
  // blocks start in linear order (x fastest): key tile 0 (the most query
  // tiles after it) of every (KV head, sequence) first
  const int kt = blockIdx.z;
  const int kvh = blockIdx.x, b = blockIdx.y;
  const int G = nh / nkv;
  const int nqt = (S + 127) / 128;
  const int per_head = nqt - kt;
  const int n_it = G * per_head;
  const int row_base = b * S;
  (void)nkt;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    mbar_init(q_full, 1);
    mbar_init(q_free, 1);
    mbar_init(s_full, 1);
    mbar_init(p_full, kBwdSoftmaxThreads);
    mbar_init(dq_full, 1);
    mbar_init(dq_free, kBwdSoftmaxThreads);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_wait();  // the prologue above overlapped the previous kernel's tail
  const uint32_t t_s = tmem, t_dp = tmem + 128, t_dv = tmem + 256, t_dk = tmem + 256 + HD;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ producer
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      tma_prefetch_desc(&tmO);
      mbar_arrive_expect_tx(kv_full, 2 * L::kT);
      for (int i = 0; i < kDBoxes; ++i) {
        tma_load_2d(smem + L::kKOff + i * kBox, &tmK, kv_full, kvh * HD + 64 * i, row_base + kt * 128);
        tma_load_2d(smem + L::kVOff + i * kBox, &tmV, kv_full, kvh * HD + 64 * i, row_base + kt * 128);
      }
      for (int it = 0; it < n_it; ++it) {
        const int hq = kvh * G + it / per_head;
        const int qt = kt + it % per_head;
        if (it >= 1 && !mbar_wait(q_free, (it - 1) & 1, abort_flag, err, kErrWaitConsumer)) {
          // let the copies already issued land before the CTA can exit
          mbar_drain(kv_full, 0);
          mbar_drain(q_full, (it - 1) & 1);
          break;
        }
        mbar_arrive_expect_tx(q_full, 2 * L::kT);
        for (int i = 0; i < kDBoxes; ++i) {
          tma_load_2d(smem + L::kQOff + i * kBox, &tmQ, q_full, hq * HD + 64 * i, row_base + qt * 128);
          tma_load_2d(smem + L::kOOff + i * kBox, &tmO, q_full, hq * HD + 64 * i, row_base + qt * 128);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------------------------------------------------- MMA issuer
      constexpr uint32_t idesc_s = idesc_f16_f32(128, 128);                       // K-major x K-major
      constexpr uint32_t idesc_acc = idesc_f16_f32(128, HD) | (1u << 16);          // B MN-major
      constexpr uint32_t idesc_dq = idesc_f16_f32(128, HD) | (1u << 15) | (1u << 16);  // A, B MN-major
      const uint32_t sk = smem_u32(smem + L::kKOff), sv = smem_u32(smem + L::kVOff);
      const uint32_t sq = smem_u32(smem + L::kQOff), so = smem_u32(smem + L::kOOff);
      const uint32_t sp = smem_u32(smem + L::kPOff), ss = smem_u32(smem + L::kSOff);
      // S^T of the next iteration goes out as soon as its Q tile has landed
      // (the softmax has read the previous S^T; P^T lives in shared memory),
      // overlapping the drain of the previous dQ_part, which occupies the dP^T
      // columns until dq_free
      auto issue_st = [&]() {
#pragma unroll
        for (int k = 0; k < HD / 16; ++k) {
          const uint32_t off = (k >> 2) * kBox + (k & 3) * 32;
          umma_f16(t_s, sw128_kmajor_desc(sk + off), sw128_kmajor_desc(sq + off), idesc_s, k > 0 ? 1u : 0u);
        }
      };
      bool ok = mbar_wait(kv_full, 0, abort_flag, err, kErrWaitProducer);
      if (ok && n_it > 0) {
        ok = mbar_wait(q_full, 0, abort_flag, err, kErrWaitProducer);
        if (ok) {
          tc_fence_after();
          issue_st();
        }
      }
      for (int it = 0; it < n_it && ok; ++it) {
        if (it >= 1 && !mbar_wait(dq_free, (it - 1) & 1, abort_flag, err, kErrWaitEpilogue)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < HD / 16; ++k) {
          const uint32_t off = (k >> 2) * kBox + (k & 3) * 32;
          umma_f16(t_dp, sw128_kmajor_desc(sv + off), sw128_kmajor_desc(so + off), idesc_s, k > 0 ? 1u : 0u);
        }
        umma_commit(s_full);
        if (!mbar_wait(p_full, it & 1, abort_flag, err, kErrWaitProducer)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < 128 / 16; ++k) {
          const uint32_t offp = (k >> 2) * kBox + (k & 3) * 32;  // K-major over the 128 query columns
          umma_f16(t_dv, sw128_kmajor_desc(sp + offp), sw128_mnmajor_desc(so + k * 2048), idesc_acc,
                   (it > 0 || k > 0) ? 1u : 0u);
          umma_f16(t_dk, sw128_kmajor_desc(ss + offp), sw128_mnmajor_desc(sq + k * 2048), idesc_acc,
                   (it > 0 || k > 0) ? 1u : 0u);
        }
        umma_commit(q_free);
        // dQ_part into the dP^T columns (read by the softmax before p_full)
#pragma unroll
        for (int k = 0; k < 128 / 16; ++k)
          umma_f16(t_dp, sw128_mnmajor_desc(ss + k * 2048), sw128_mnmajor_desc(sk + k * 2048), idesc_dq,
                   k > 0 ? 1u : 0u);
        umma_commit(dq_full);
        if (it + 1 < n_it) {
          if (!mbar_wait(q_full, (it + 1) & 1, abort_flag, err, kErrWaitProducer)) { ok = false; break; }
          tc_fence_after();
          issue_st();
        }
      }
    }
  } else {
    // ------------------------------------------------------------- softmax
    const int qd = warp & 3;
    const int hf = (warp - 2) >> 2;           // which half of the columns
    const int r = qd * 32 + lane;             // key row (phase 1) / query row (drain)
    const int kr = kt * 128 + r;              // key position
    const uint32_t lane_off = static_cast<uint32_t>(qd * 32) << 16;
    uint8_t* sP = smem + L::kPOff;
    uint8_t* sS = smem + L::kSOff;
    // this warp's rows of box hf of P^T and of dS^T -- the only bytes of those
    // tiles it writes -- double as the staging slabs of its dQ drain, so
    // waiting for its own reduce-adds' reads is enough before rewriting them
    const uint32_t slab0 = smem_u32(sP + (hf * 4 + qd) * 4096);
    const uint32_t slab1 = smem_u32(sS + (hf * 4 + qd) * 4096);
    bool ok = true;
    // lse * log2(e) and delta of query row r of iteration `it`, loaded one
    // iteration ahead into registers and published through a double buffer
    auto stats = [&](int it, float& l2, float& dl) {
      const int hq = kvh * G + it / per_head;
      const int qq = (kt + it % per_head) * 128 + r;
      const size_t idx = (static_cast<size_t>(b) * nh + hq) * S + qq;
      l2 = qq < S ? lse[idx] * kLog2e : INFINITY;
      dl = qq < S ? delta[idx] : 0.f;
    };
    float l_next = 0.f, d_next = 0.f;
    if (n_it > 0) stats(0, l_next, d_next);
    for (int it = 0; it < n_it && ok; ++it) {
      const int hq = kvh * G + it / per_head;
      const int qt = kt + it % per_head;
      const int q0 = qt * 128;
      // every query of the tile after every key, all inside the sequence: no masking
      const bool interior = qt > kt && q0 + 128 <= S && kt * 128 + 128 <= S;
      float* sLb = sL + (it & 1) * 256;  // lse of this tile's query columns
      float* sDb = sLb + 128;            // delta
      if (hf == 0) {
        sLb[r] = l_next;
        sDb[r] = d_next;
      }
      // one barrier per iteration: rows of sL[it & 1] were last read in
      // iteration it - 2, which every thread finished before arriving here
      named_sync_softmax();
      if (it + 1 < n_it) stats(it + 1, l_next, d_next);
      if (!mbar_wait(s_full, it & 1, abort_flag, err, kErrWaitAccum)) { ok = false; break; }
      tc_fence_after();
      // the previous drain's TMA reduce must have read the slabs before P^T is rewritten
      if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
      __syncwarp();
#pragma unroll 1
      for (int c = 2 * hf; c < 2 * hf + 2; ++c) {  // 32 query columns at a time
        uint32_t sv[32], dv32[32];
        tmem_ld_32x32b_x32(t_s + lane_off + 32 * c, sv);
        tmem_ld_32x32b_x32(t_dp + lane_off + 32 * c, dv32);
        tmem_ld_wait();
        uint32_t pp[16], dsp[16];
        if (interior)
          bwd_softmax_chunk<false>(sv, dv32, sLb, sDb, c, scale_log2, q0, kr, S, pp, dsp);
        else
          bwd_softmax_chunk<true>(sv, dv32, sLb, sDb, c, scale_log2, q0, kr, S, pp, dsp);
        // row r of P^T / dS^T: query columns 32c.. -> box c/2, 16-byte chunks 4(c%2)..
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int ch = 4 * (c & 1) + u;
          const uint32_t off = (c >> 1) * kBox + r * 128 + ((ch ^ (r & 7)) << 4);
          asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(smem_u32(sP + off)), "r"(pp[4 * u]),
                       "r"(pp[4 * u + 1]), "r"(pp[4 * u + 2]), "r"(pp[4 * u + 3])
                       : "memory");
          asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(smem_u32(sS + off)), "r"(dsp[4 * u]),
                       "r"(dsp[4 * u + 1]), "r"(dsp[4 * u + 2]), "r"(dsp[4 * u + 3])
                       : "memory");
        }
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      tc_fence_before();
      mbar_arrive(p_full);
      // ---- drain dQ_part (query row r of this tile) into the global dQ
      if (!mbar_wait(dq_full, it & 1, abort_flag, err, kErrWaitAccum)) { ok = false; break; }
      tc_fence_after();
      const bool valid = q0 + r < S;
      constexpr int kHalfChunks = HD / 64;  // 32-column chunks of dQ_part per half
      // this warp's chunks of dQ_part, loaded from TMEM together
      uint32_t dq2[kHalfChunks][32];
#pragma unroll
      for (int i = 0; i < kHalfChunks; ++i) tmem_ld_32x32b_x32(t_dp + lane_off + 32 * (hf * kHalfChunks + i), dq2[i]);
      tmem_ld_wait();
#pragma unroll
      for (int i = 0; i < kHalfChunks; ++i) {
        // chunk c of this warp's 32 rows -> its own 4 KB slab inside the P^T /
        // dS^T tiles (free once dQ_part is committed), so the reduce-adds of
        // its chunks are in flight together
        const int c = hf * kHalfChunks + i;
        const uint32_t slab = i == 0 ? slab0 : slab1;
        const uint32_t* dqv = dq2[i];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float f0 = valid ? __uint_as_float(dqv[4 * j]) * scale : 0.f;
          const float f1 = valid ? __uint_as_float(dqv[4 * j + 1]) * scale : 0.f;
          const float f2 = valid ? __uint_as_float(dqv[4 * j + 2]) * scale : 0.f;
          const float f3 = valid ? __uint_as_float(dqv[4 * j + 3]) * scale : 0.f;
          const uint32_t a = slab + lane * 128 + ((j ^ (lane & 7)) << 4);
          asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(a), "f"(f0), "f"(f1), "f"(f2), "f"(f3)
                       : "memory");
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) {
          if (dq_slab_rows == 0) {
            asm volatile(
                "cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                    reinterpret_cast<uint64_t>(&tmDQ)),
                "r"(slab), "r"(hq * HD + 32 * c), "r"(row_base + q0 + qd * 32)
                : "memory");
          } else {
            // deterministic mode: this key tile's partial into its own slab
            // (rows padded to whole 128-row tiles per sequence), summed in key
            // tile order by the QK-norm / RoPE backward
            const int prow = kt * dq_slab_rows + (b * nqt + qt) * 128 + qd * 32;
            asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                             reinterpret_cast<uint64_t>(&tmDQ)),
                         "r"(slab), "r"(hq * HD + 32 * c), "r"(prow)
                         : "memory");
          }
          asm volatile("cp.async.bulk.commit_group;" ::: "memory");
        }
      }
      tc_fence_before();
      mbar_arrive(dq_free);
    }
    if (lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
    __syncwarp();
    // ---- dK (scaled) and dV of key row r
    if (ok && n_it > 0) {
      tc_fence_after();
      const bool valid = kr < S;
      float* dkrow = dk + static_cast<size_t>(row_base + kr) * lddk + kvh * HD;
      __half* dvrow = dv + static_cast<size_t>(row_base + kr) * lddv + kvh * HD;
#pragma unroll 1
      for (int c = hf * (HD / 64); c < (hf + 1) * (HD / 64); ++c) {
        uint32_t a[32], bvv[32];
        tmem_ld_32x32b_x32(t_dk + lane_off + 32 * c, a);
        tmem_ld_32x32b_x32(t_dv + lane_off + 32 * c, bvv);
        tmem_ld_wait();
        if (valid) {
#pragma unroll
          for (int t = 0; t < 32; t += 4)
            *reinterpret_cast<float4*>(dkrow + 32 * c + t) =
                make_float4(__uint_as_float(a[t]) * scale, __uint_as_float(a[t + 1]) * scale,
                            __uint_as_float(a[t + 2]) * scale, __uint_as_float(a[t + 3]) * scale);
#pragma unroll
          for (int t = 0; t < 32; t += 8) {
            uint4 w;
            w.x = pack_half2(__uint_as_float(bvv[t]), __uint_as_float(bvv[t + 1]));
            w.y = pack_half2(__uint_as_float(bvv[t + 2]), __uint_as_float(bvv[t + 3]));
            w.z = pack_half2(__uint_as_float(bvv[t + 4]), __uint_as_float(bvv[t + 5]));
            w.w = pack_half2(__uint_as_float(bvv[t + 6]), __uint_as_float(bvv[t + 7]));
            *reinterpret_cast<uint4*>(dvrow + 32 * c + t) = w;
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

PFN_cuTensorMapEncodeTiled_v12000 encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// [rows, cols] fp16 with row stride ld (elements); box 64 columns x 128 rows, 128-B swizzle.
bool tile_map(CUtensorMap* m, const __half* p, int rows, int cols, int ld) {
  auto enc = encoder();
  if (!enc || reinterpret_cast<uintptr_t>(p) % 16 || (ld * 2) % 16) return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 2};
  cuuint32_t box[2] = {64u, 128u};
  cuuint32_t es[2] = {1u, 1u};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half*>(p), dims, strides, box, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// [rows, cols] fp32, box 32 columns x 32 rows (one drain slab), 128-B swizzle.
bool f32_slab_map(CUtensorMap* m, const float* p, int rows, int cols, int ld) {
  auto enc = encoder();
  if (!enc || reinterpret_cast<uintptr_t>(p) % 16 || (ld * 4) % 16) return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 4};
  cuuint32_t box[2] = {32u, 32u};
  cuuint32_t es[2] = {1u, 1u};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(p), dims, strides, box, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int HD>
cudaError_t bwd_tc_launch(const __half* q, const __half* k, const __half* v, const __half* dout, const float* lse,
                          const float* delta, float* dq, float* dk, __half* dv, int B, int S, int nh, int nkv,
                          int ldq, int ldk, int ldv, int ldo, int lddq, int lddk, int lddv, int* err,
                          cudaStream_t st, bool dq_zeroed, float* dq_slabs) {
  using L = BwdLayout<HD>;
  CUtensorMap mq, mk, mv, mo, mdq;
  const int nqt = (S + 127) / 128;
  const int slab_rows = dq_slabs ? B * nqt * 128 : 0;  // rows of one key tile's slab
  if (!tile_map(&mq, q, B * S, nh * HD, ldq) || !tile_map(&mk, k, B * S, nkv * HD, ldk) ||
      !tile_map(&mv, v, B * S, nkv * HD, ldv) || !tile_map(&mo, dout, B * S, nh * HD, ldo) ||
      !(dq_slabs ? f32_slab_map(&mdq, dq_slabs, nqt * slab_rows, nh * HD, nh * HD)
                 : f32_slab_map(&mdq, dq, B * S, nh * HD, lddq)))
    return cudaErrorInvalidValue;
  auto kern = attn_bwd_tc_kernel<HD>;
  static std::atomic<unsigned long long> attr_set{0};
  {
    cudaError_t e = once_per_device(attr_set, [&] {
      return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kBytes);
    });
    if (e != cudaSuccess) return e;
  }
  // dQ accumulates partial products of every key tile (into zeros), unless
  // each key tile stores its own slab
  if (!dq_zeroed && !dq_slabs) {
    cudaError_t e = fill_f32_2d(dq, lddq, B * S, nh * HD, 0.f, st);
    if (e != cudaSuccess) return e;
  }
  dim3 grid(nkv, B, (S + 127) / 128);
  const float scale = 1.0f / sqrtf(static_cast<float>(HD));
  launch_pdl(kern, grid, 64 + kBwdSoftmaxThreads, L::kBytes, st, mq, mk, mv, mo, mdq, lse, delta, dk, dv, S, nh, nkv,
             lddk, lddv, scale,
             scale * kLog2e, slab_rows, err);
  return cudaGetLastError();
}

template <int HD>
cudaError_t fwd_tc_launch(const __half* q, const __half* k, const __half* v, __half* o, float* lse, int B, int S,
                          int nh, int nkv, int ldq, int ldk, int ldv, int ldo, int* err, cudaStream_t st) {
  using L = FwdLayout<HD>;
  CUtensorMap mq, mk, mv;
  if (!tile_map(&mq, q, B * S, nh * HD, ldq) || !tile_map(&mk, k, B * S, nkv * HD, ldk) ||
      !tile_map(&mv, v, B * S, nkv * HD, ldv))
    return cudaErrorInvalidValue;
  auto kern = attn_fwd_tc_kernel<HD>;
  static std::atomic<unsigned long long> attr_set{0};
  {
    cudaError_t e = once_per_device(attr_set, [&] {
      cudaError_t r = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kBytes);
      // two CTAs per SM need the whole shared-memory carveout
      if (r == cudaSuccess) r = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
      return r;
    });
    if (e != cudaSuccess) return e;
  }
  dim3 grid(nh, B, (S + kTq - 1) / kTq);
  const float scale = 1.0f / sqrtf(static_cast<float>(HD));
  launch_pdl(kern, grid, 192, L::kBytes, st, mq, mk, mv, o, lse, S, nh, nkv, ldo, scale * kLog2e, err);
  return cudaGetLastError();
}

}  // namespace

cudaError_t attention_backward_tc(const __half* q, const __half* k, const __half* v, const __half* dout,
                                  const float* lse, const float* delta, float* dq, float* dk, __half* dv, int B, int S,
                                  int nh, int nkv, int hd, int ldq, int ldk, int ldv, int ldo, int lddq, int lddk,
                                  int lddv, int* err, cudaStream_t st, bool dq_zeroed, float* dq_slabs) {
  if (hd == 128)
    return bwd_tc_launch<128>(q, k, v, dout, lse, delta, dq, dk, dv, B, S, nh, nkv, ldq, ldk, ldv, ldo, lddq, lddk,
                              lddv, err, st, dq_zeroed, dq_slabs);
  if (hd == 64)
    return bwd_tc_launch<64>(q, k, v, dout, lse, delta, dq, dk, dv, B, S, nh, nkv, ldq, ldk, ldv, ldo, lddq, lddk,
                             lddv, err, st, dq_zeroed, dq_slabs);
  return cudaErrorInvalidValue;
}

cudaError_t attention_forward_tc(const __half* q, const __half* k, const __half* v, __half* o, float* lse, int B,
                                 int S, int nh, int nkv, int hd, int ldq, int ldk, int ldv, int ldo, int* err,
                                 cudaStream_t st) {
  if (hd == 128) return fwd_tc_launch<128>(q, k, v, o, lse, B, S, nh, nkv, ldq, ldk, ldv, ldo, err, st);
  if (hd == 64) return fwd_tc_launch<64>(q, k, v, o, lse, B, S, nh, nkv, ldq, ldk, ldv, ldo, err, st);
  return cudaErrorInvalidValue;
}

}  // namespace llmcu
