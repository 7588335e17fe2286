// attention_tc.cu -- causal GQA flash attention forward on tcgen05 / TMEM.
//
// One CTA per (128-row query tile, query head, sequence), 192 threads:
//   warp 0     TMA producer: Q once, then (K_j, V_j) 128-row tiles in a 2-deep ring
//   warp 1     MMA issuer:   S_j = Q K_j^T into one of two TMEM buffers, then
//                            O += P_{j-1} V_{j-1} (O accumulates in TMEM)
//   warps 2-5  softmax:      thread r owns query row r: reads S_j from TMEM,
//                            masks, keeps the running max / sum in registers,
//                            writes P_j (fp16) to shared memory, and rescales
//                            its O row in TMEM only when the max grew by more
//                            than 2^8 (P stays < 256, exact in fp16)
// Shared memory (hd 128): Q 32 KB, K 2x32 KB, V 2x32 KB, P 32 KB.  TMEM:
// S0 [0,128), S1 [128,256), O [256, 256+hd).  P V uses V as an MN-major
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
  static constexpr int kP = kTq * kTk * 2;
  static constexpr int kQOff = 0;
  static constexpr int kKOff = kQOff + kQ;        // 2 stages
  static constexpr int kVOff = kKOff + 2 * kKV;   // 2 stages
  static constexpr int kPOff = kVOff + 2 * kKV;
  static constexpr int kBarOff = kPOff + kP;
  static constexpr int kBytes = kBarOff + 256 + 1024;
};

// MN-major (column-contiguous) 128-byte-swizzled operand: 64-element rows of
// 128 B, 8-row atoms of 1 KB stacked along K (stride byte offset 1 KB), the
// next 64 columns one 16 KB box further (leading byte offset).
__device__ __forceinline__ uint64_t sw128_mnmajor_desc(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>(kBox >> 4) << 16;      // leading byte offset: next 64 columns
  d |= static_cast<uint64_t>(1024 >> 4) << 32;      // stride byte offset: next 8 K rows
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;
  return d;
}

__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
      "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
      "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

template <int HD>
__global__ void __launch_bounds__(192, 1)
    attn_fwd_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV, __half* __restrict__ o, float* __restrict__ lse,
                       int S, int nh, int nkv, int ldo, float scale_log2, int* err) {
  using L = FwdLayout<HD>;
  constexpr int kDBoxes = HD / 64;  // 64-wide boxes along head_dim
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;   // [2]
  uint64_t* kv_empty = bars + 3;  // [2]
  uint64_t* s_full = bars + 5;    // [2]
  uint64_t* s_free = bars + 7;    // [2]
  uint64_t* p_full = bars + 9;
  uint64_t* pv_done = bars + 10;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 11);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qt = gridDim.x - 1 - blockIdx.x;  // longest (causal) tiles first
  const int h = blockIdx.y, b = blockIdx.z;
  const int kvh = h / (nh / nkv);
  const int n_kv = qt + 1;
  const int row_base = b * S;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 128);
    }
    mbar_init(p_full, 128);
    mbar_init(pv_done, 1);
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
  const uint32_t t_s0 = tmem, t_o = tmem + 256;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ producer
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      mbar_arrive_expect_tx(q_full, L::kQ);
      for (int i = 0; i < kDBoxes; ++i)
        tma_load_2d(smem + L::kQOff + i * kBox, &tmQ, q_full, h * HD + 64 * i, row_base + qt * kTq);
      for (int j = 0; j < n_kv; ++j) {
        const int s = j & 1;
        if (j >= 2 && !mbar_wait(&kv_empty[s], ((j >> 1) - 1) & 1, abort_flag, err, kErrWaitConsumer)) break;
        mbar_arrive_expect_tx(&kv_full[s], 2 * L::kKV);
        for (int i = 0; i < kDBoxes; ++i) {
          tma_load_2d(smem + L::kKOff + s * L::kKV + i * kBox, &tmK, &kv_full[s], kvh * HD + 64 * i,
                      row_base + j * kTk);
          tma_load_2d(smem + L::kVOff + s * L::kKV + i * kBox, &tmV, &kv_full[s], kvh * HD + 64 * i,
                      row_base + j * kTk);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------------------------------------------------- MMA issuer
      constexpr uint32_t idesc_s = idesc_f16_f32(kTq, kTk);
      constexpr uint32_t idesc_pv = idesc_f16_f32(kTq, HD) | (1u << 16);  // B (V) MN-major
      const uint32_t sq = smem_u32(smem + L::kQOff);
      const uint32_t sp = smem_u32(smem + L::kPOff);
      auto issue_pv = [&](int j) -> bool {
        if (!mbar_wait(p_full, j & 1, abort_flag, err, kErrWaitProducer)) return false;
        tc_fence_after();
        const uint32_t sv = smem_u32(smem + L::kVOff + (j & 1) * L::kKV);
#pragma unroll
        for (int k = 0; k < kTk / 16; ++k) {
          const uint64_t adesc = sw128_kmajor_desc(sp + (k >> 2) * kBox + (k & 3) * 32);
          const uint64_t bdesc = sw128_mnmajor_desc(sv + k * 16 * 128);
          umma_f16(t_o, adesc, bdesc, idesc_pv, (j > 0 || k > 0) ? 1u : 0u);
        }
        umma_commit(pv_done);
        umma_commit(&kv_empty[j & 1]);
        return true;
      };
      bool ok = mbar_wait(q_full, 0, abort_flag, err, kErrWaitProducer);
      for (int j = 0; j < n_kv && ok; ++j) {
        const int s = j & 1;
        if (!mbar_wait(&kv_full[s], (j >> 1) & 1, abort_flag, err, kErrWaitProducer)) { ok = false; break; }
        if (j >= 2 && !mbar_wait(&s_free[s], ((j >> 1) - 1) & 1, abort_flag, err, kErrWaitEpilogue)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t sk = smem_u32(smem + L::kKOff + s * L::kKV);
#pragma unroll
        for (int k = 0; k < HD / 16; ++k) {
          const uint64_t adesc = sw128_kmajor_desc(sq + (k >> 2) * kBox + (k & 3) * 32);
          const uint64_t bdesc = sw128_kmajor_desc(sk + (k >> 2) * kBox + (k & 3) * 32);
          umma_f16(t_s0 + s * kTk, adesc, bdesc, idesc_s, k > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[s]);
        if (j >= 1 && !issue_pv(j - 1)) { ok = false; break; }
      }
      if (ok) issue_pv(n_kv - 1);
    }
  } else {
    // ------------------------------------------------------------- softmax
    const int qd = warp & 3;                 // TMEM lane quadrant
    const int r = qd * 32 + lane;            // query row within the tile
    const int q = qt * kTq + r;              // query position in the sequence
    const uint32_t lane_off = static_cast<uint32_t>(qd * 32) << 16;
    uint8_t* sP = smem + L::kPOff;
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < n_kv && ok; ++j) {
      const int s = j & 1;
      if (!mbar_wait(&s_full[s], (j >> 1) & 1, abort_flag, err, kErrWaitAccum)) { ok = false; break; }
      tc_fence_after();
      float sv[kTk];
#pragma unroll
      for (int c = 0; c < kTk / 32; ++c)
        tmem_ld_32x32b_x32(t_s0 + s * kTk + lane_off + 32 * c, *reinterpret_cast<uint32_t(*)[32]>(sv + 32 * c));
      tmem_ld_wait();
      tc_fence_before();
      mbar_arrive(&s_free[s]);
      float mx = -INFINITY;
#pragma unroll
      for (int i = 0; i < kTk; ++i) {
        const int kv = j * kTk + i;
        float x = sv[i] * scale_log2;
        if (kv > q || kv >= S) x = -INFINITY;
        sv[i] = x;
        mx = fmaxf(mx, x);
      }
      const float m_new = fmaxf(m_used, mx);
      const bool resc = (j > 0) && (m_new > m_used + 8.0f);
      const float m_next = (j == 0 || resc) ? m_new : m_used;
      const float corr = resc ? fast_exp2(m_used - m_next) : 1.0f;
      uint32_t pk[kTk / 2];
      float rs = 0.f;
#pragma unroll
      for (int i = 0; i < kTk / 2; ++i) {
        float p0 = fast_exp2(sv[2 * i] - m_next);
        float p1 = fast_exp2(sv[2 * i + 1] - m_next);
        if (m_next == -INFINITY) p0 = p1 = 0.f;
        rs += p0 + p1;
        pk[i] = pack_half2(p0, p1);
      }
      l = l * corr + rs;
      m_used = m_next;
      if (j >= 1) {
        if (!mbar_wait(pv_done, (j - 1) & 1, abort_flag, err, kErrWaitAccum)) { ok = false; break; }
        tc_fence_after();
      }
      if (__any_sync(0xffffffffu, resc)) {
#pragma unroll
        for (int c = 0; c < HD / 32; ++c) {
          uint32_t ov[32];
          tmem_ld_32x32b_x32(t_o + lane_off + 32 * c, ov);
          tmem_ld_wait();
#pragma unroll
          for (int t = 0; t < 32; ++t) ov[t] = __float_as_uint(__uint_as_float(ov[t]) * corr);
          tmem_st_32x32b_x32(t_o + lane_off + 32 * c, ov);
        }
        tmem_st_wait();
      }
      // P row r: columns [64*bx, 64*bx + 64) in box bx, 16-byte chunk c swizzled by r % 8
#pragma unroll
      for (int c = 0; c < kTk / 8; ++c) {
        const int bx = c >> 3, cc = c & 7;
        const uint32_t addr = smem_u32(sP + bx * kBox + r * 128 + ((cc ^ (r & 7)) << 4));
        asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(pk[4 * c]), "r"(pk[4 * c + 1]),
                     "r"(pk[4 * c + 2]), "r"(pk[4 * c + 3])
                     : "memory");
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      tc_fence_before();
      mbar_arrive(p_full);
    }
    if (ok && mbar_wait(pv_done, (n_kv - 1) & 1, abort_flag, err, kErrWaitAccum)) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.0f / l : 0.f;
      __half* orow = o + static_cast<size_t>(row_base + q) * ldo + h * HD;
#pragma unroll
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

template <int HD>
cudaError_t fwd_tc_launch(const __half* q, const __half* k, const __half* v, __half* o, float* lse, int B, int S,
                          int nh, int nkv, int ldq, int ldk, int ldv, int ldo, int* err, cudaStream_t st) {
  using L = FwdLayout<HD>;
  CUtensorMap mq, mk, mv;
  if (!tile_map(&mq, q, B * S, nh * HD, ldq) || !tile_map(&mk, k, B * S, nkv * HD, ldk) ||
      !tile_map(&mv, v, B * S, nkv * HD, ldv))
    return cudaErrorInvalidValue;
  auto kern = attn_fwd_tc_kernel<HD>;
  static bool attr = false;
  if (!attr) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kBytes);
    if (e != cudaSuccess) return e;
    attr = true;
  }
  dim3 grid((S + kTq - 1) / kTq, nh, B);
  const float scale = 1.0f / sqrtf(static_cast<float>(HD));
  kern<<<grid, 192, L::kBytes, st>>>(mq, mk, mv, o, lse, S, nh, nkv, ldo, scale * kLog2e, err);
  return cudaGetLastError();
}

}  // namespace

cudaError_t attention_forward_tc(const __half* q, const __half* k, const __half* v, __half* o, float* lse, int B,
                                 int S, int nh, int nkv, int hd, int ldq, int ldk, int ldv, int ldo, int* err,
                                 cudaStream_t st) {
  if (hd == 128) return fwd_tc_launch<128>(q, k, v, o, lse, B, S, nh, nkv, ldq, ldk, ldv, ldo, err, st);
  if (hd == 64) return fwd_tc_launch<64>(q, k, v, o, lse, B, S, nh, nkv, ldq, ldk, ldv, ldo, err, st);
  return cudaErrorInvalidValue;
}

}  // namespace llmcu
