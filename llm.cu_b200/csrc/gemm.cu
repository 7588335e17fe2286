// gemm.cu -- host side of the tcgen05 GEMM: TMA descriptor encoding, tile
// shape choice and the launch of the instantiated kernels.
#include <cudaTypedefs.h>

#include <algorithm>
#include <cmath>
#include <mutex>

#include "common.cuh"
#include "gemm.cuh"

namespace llmcu {

namespace {

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
int g_num_sms = 0;
std::once_flag g_once;

void init_once() {
  cudaDriverEntryPointQueryResult q;
  void* fn = nullptr;
  if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
      q == cudaDriverEntryPointSuccess)
    g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  int dev = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
  if (g_num_sms <= 0) g_num_sms = 148;
}

// 2-D fp16 operand map, 128-B swizzle.  K-major: rows x k (k contiguous), box
// 64 (k) x box_rows.  MN-major: k x rows (rows contiguous), box 64 x 64.
bool make_map(CUtensorMap* map, const Operand& op, int box_rows) {
  if (!g_encode) return false;
  if (reinterpret_cast<uintptr_t>(op.ptr) % 16 != 0 || (op.ld * 2) % 16 != 0) return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(op.mn ? op.rows : op.k),
                        static_cast<cuuint64_t>(op.mn ? op.k : op.rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(op.ld) * 2};
  cuuint32_t box[2] = {64u, static_cast<cuuint32_t>(op.mn ? 64 : box_rows)};
  cuuint32_t estr[2] = {1u, 1u};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half*>(op.ptr), dims, strides, box,
                        estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// INT8 B operand: the same dimensions as make_map's, unswizzled boxes of 64
// codes x box rows (the converter warps read them with 16-byte loads).
bool make_map_q8(CUtensorMap* map, const Operand& op, int box_rows) {
  if (!g_encode || !op.q8) return false;
  if (reinterpret_cast<uintptr_t>(op.q8) % 16 != 0 || op.ld % 16 != 0) return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(op.mn ? op.rows : op.k),
                        static_cast<cuuint64_t>(op.mn ? op.k : op.rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(op.ld)};
  cuuint32_t box[2] = {64u, static_cast<cuuint32_t>(op.mn ? 64 : box_rows)};
  cuuint32_t estr[2] = {1u, 1u};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<int8_t*>(op.q8), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// Output / epilogue-input map: rows x cols of fp16 or fp32, box = 128 bytes of
// columns x 32 rows (one epilogue warp's slab), 128-byte swizzle.
bool make_io_map(CUtensorMap* map, const void* ptr, int rows, int cols, int ld, bool f32) {
  if (!g_encode || !ptr) return false;
  const int es = f32 ? 4 : 2;
  if (reinterpret_cast<uintptr_t>(ptr) % 16 != 0 || (static_cast<int64_t>(ld) * es) % 16 != 0) return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * es};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(128 / es), 32u};
  cuuint32_t estr[2] = {1u, 1u};
  CUresult r = g_encode(map, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                        const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// fp16 [rows, cols] with row stride ld read in [32 rows x 32 columns] boxes,
// 64-byte swizzle (the SwiGLU backward's factor boxes).
bool make_box32_map(CUtensorMap* map, const void* ptr, int rows, int cols, int ld) {
  if (!g_encode || !ptr) return false;
  if (reinterpret_cast<uintptr_t>(ptr) % 16 != 0 || (static_cast<int64_t>(ld) * 2) % 16 != 0) return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 2};
  cuuint32_t box[2] = {32u, 32u};
  cuuint32_t estr[2] = {1u, 1u};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// As many pipeline stages as fit beside the epilogue slabs (at most 8).
template <int BN, int EW, int SLAB, int CG, bool Q8 = false>
constexpr int stages_for() {
  constexpr int stage = kBlockM * kBlockK * 2 + BN / CG * kBlockK * 2;  // INT8 codes land inside B
  constexpr int s = (232448 - 1536 - EW * SLAB) / stage;
  return s > 8 ? 8 : s;
}

template <class E, class = void>
struct epi_groups : std::integral_constant<int, kGemmEpiGroups> {};
template <class E>
struct epi_groups<E, std::void_t<decltype(E::kEpiGroups)>> : std::integral_constant<int, E::kEpiGroups> {};

// 8 epilogue warps (two per TMEM lane quadrant) for 128/256-wide tiles, 4 for
// 64 -- or as many groups of 4 as the epilogue asks for
template <int BN, class E>
constexpr int epi_warps() {
  return BN >= 128 ? 4 * epi_groups<E>::value : 4;
}

template <int BN, class E, bool BMN, int CG, bool Q8 = false>
cudaError_t launch(const CUtensorMap* maps, const GemmShape& sh, const typename E::Params& p, int* err,
                   cudaStream_t st) {
  constexpr int kEpiWarps = epi_warps<BN, E>();
  constexpr int S = stages_for<BN, kEpiWarps, E::kSlab, CG, Q8>();
  using L = GemmSmem<BN, S, kEpiWarps, E::kSlab, CG, Q8>;
  static_assert(L::kBytes <= 232448, "shared memory budget");
  constexpr int kThreads = 64 + 32 * kEpiWarps + (Q8 ? kQ8Threads : 0);
  auto kern = gemm_tc_kernel<BN, S, kEpiWarps, E, BMN, CG, Q8>;
  static std::atomic<unsigned long long> attr_set{0};  // per instantiation, one bit per device
  {
    cudaError_t e = once_per_device(attr_set, [&] {
      return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kBytes);
    });
    if (e != cudaSuccess) return e;
  }
  const int units = sh.num_tiles * sh.splits;
  if constexpr (CG == 1) {
    const int grid = units < g_num_sms ? units : g_num_sms;
    cudaError_t e = launch_pdl(kern, grid, kThreads, L::kBytes, st, maps[0], maps[1], maps[2], maps[3], sh, p, err);
    if (e != cudaSuccess) return e;
  } else {
    // one CTA pair per unit, at most one CTA per SM
    const int pairs = std::min(units, g_num_sms / 2);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * pairs);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = L::kBytes;
    cfg.stream = st;
    cudaLaunchAttribute at[2];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = 2;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = pdl_enabled() ? 2 : 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, maps[0], maps[1], maps[2], maps[3], sh, p, err);
    if (e != cudaSuccess) return e;
  }
  return cudaGetLastError();
}

template <int BN, bool BMN, int CG>
cudaError_t dispatch(Epi epi, const EpiArgs& ea, const CUtensorMap* maps, const GemmShape& sh, int* err,
                     cudaStream_t st) {
  switch (epi) {
    case Epi::kStoreF16:
      return launch<BN, EpiStoreF16, BMN, CG>(maps, sh, EpiStoreF16::Params{}, err, st);
    case Epi::kStoreF32:
      return launch<BN, EpiStoreF32, BMN, CG>(maps, sh, EpiStoreF32::Params{ea.accumulate}, err, st);
    case Epi::kResidF32:
      return launch<BN, EpiResidF32, BMN, CG>(maps, sh, EpiResidF32::Params{}, err, st);
    case Epi::kSwiGLUBwd:
      if constexpr (BN == 256) {
        return launch<BN, EpiSwiGLUBwd, BMN, CG>(maps, sh, EpiSwiGLUBwd::Params{ea.gu_in, ea.ld_gu, ea.gu_out_scale}, err, st);
      } else {
        return cudaErrorInvalidValue;
      }
    case Epi::kStoreF16Delta:
      if constexpr (BN == 256) {
        EpiStoreF16Delta::Params p{ea.attn_o, ea.ld_o, ea.delta, ea.seq, ea.n_heads, ea.head_dim};
        return launch<BN, EpiStoreF16Delta, BMN, CG>(maps, sh, p, err, st);
      } else {
        return cudaErrorInvalidValue;
      }
    case Epi::kQKNormRope:
      if constexpr (BN == 256 && !BMN) {
        EpiQKNormRope::Params p{ea.q_norm_w, ea.k_norm_w, ea.rope_cos, ea.rope_sin, ea.seq, ea.n_q_cols,
                                ea.n_qk_cols, ea.eps};
        return launch<BN, EpiQKNormRope, BMN, CG>(maps, sh, p, err, st);
      } else {
        return cudaErrorInvalidValue;
      }
    case Epi::kSwiGLU:
      if constexpr (BN == 256 && !BMN) {
        return launch<BN, EpiSwiGLU, BMN, CG>(maps, sh, EpiSwiGLU::Params{}, err, st);
      } else {
        return cudaErrorInvalidValue;
      }
    case Epi::kCEStream:
      if constexpr (BN == 256 && !BMN) {
        EpiCEStream::Params p{ea.targets, ea.ce_ref, ea.part_max, ea.part_sum, ea.tgt_logit, ea.ce_slots,
                              ea.vocab_off};
        return launch<BN, EpiCEStream, BMN, CG>(maps, sh, p, err, st);
      } else {
        return cudaErrorInvalidValue;
      }
  }
  return cudaErrorInvalidValue;
}

// INT8 B: the MLP GEMMs of an INT8 base -- gate/up + SwiGLU and down +
// residual (B K-major), down dX + SwiGLU backward and gate/up dX (B MN-major)
template <int CG>
cudaError_t dispatch_q8(Epi epi, bool bmn, const EpiArgs& ea, const CUtensorMap* maps, const GemmShape& sh, int* err,
                        cudaStream_t st) {
  if (!bmn && epi == Epi::kSwiGLU) return launch<256, EpiSwiGLU, false, CG, true>(maps, sh, EpiSwiGLU::Params{}, err, st);
  if (!bmn && epi == Epi::kResidF32) return launch<256, EpiResidF32, false, CG, true>(maps, sh, EpiResidF32::Params{}, err, st);
  if (bmn && epi == Epi::kSwiGLUBwd)
    return launch<256, EpiSwiGLUBwdScaled, true, CG, true>(
        maps, sh, EpiSwiGLUBwdScaled::Params{ea.gu_in, ea.ld_gu, ea.gu_out_scale}, err, st);
  if (bmn && epi == Epi::kStoreF16) return launch<256, EpiStoreF16, true, CG, true>(maps, sh, EpiStoreF16::Params{}, err, st);
  return cudaErrorInvalidValue;
}

}  // namespace

int gemm_num_sms() {
  std::call_once(g_once, init_once);
  return g_num_sms;
}

bool encode_tma_2d_f16(CUtensorMap* map, const void* ptr, int rows, int cols, int ld, int box_rows) {
  std::call_once(g_once, init_once);
  Operand op{static_cast<const __half*>(ptr), rows, cols, ld, false};
  return make_map(map, op, box_rows);
}

namespace {
// split-K fix-up workspace of the calling host thread (set_gemm_workspace)
thread_local float* t_fx_ws = nullptr;
thread_local size_t t_fx_ws_floats = 0;
thread_local int* t_fx_cnt = nullptr;
thread_local int t_fx_cnt_n = 0;
}  // namespace

void set_gemm_workspace(float* ws, size_t ws_floats, int* cnt, int cnt_n) {
  t_fx_ws = ws;
  t_fx_ws_floats = ws_floats;
  t_fx_cnt = cnt;
  t_fx_cnt_n = cnt_n;
}

cudaError_t gemm(const Operand& A, const Operand& B, int M, int N, Epi epi, const EpiArgs& ea, int* err,
                 cudaStream_t st, int bn_hint) {
  std::call_once(g_once, init_once);
  if (!g_encode) return cudaErrorNotSupported;
  if (M <= 0 || N <= 0 || A.k <= 0 || A.k != B.k || A.mn) return cudaErrorInvalidValue;
  int BN = bn_hint;
  if (BN == 0) BN = (epi == Epi::kSwiGLU || epi == Epi::kSwiGLUBwd) ? 256 : (N <= 64 ? 64 : (N <= 128 ? 128 : 256));
  if (epi == Epi::kQKNormRope) {
    BN = 256;
    // 128-wide heads that start on slice boundaries; tables [seq, 64]
    if (!ea.rope_out || !ea.q_norm_w || !ea.k_norm_w || !ea.rope_cos || !ea.rope_sin || ea.seq <= 0 ||
        ea.n_q_cols % 128 || ea.n_qk_cols % 128 || ea.n_qk_cols < ea.n_q_cols || ea.ld_rope % 8 ||
        reinterpret_cast<uintptr_t>(ea.q_norm_w) % 16 || reinterpret_cast<uintptr_t>(ea.k_norm_w) % 16 ||
        reinterpret_cast<uintptr_t>(ea.rope_cos) % 16 || reinterpret_cast<uintptr_t>(ea.rope_sin) % 16)
      return cudaErrorInvalidValue;
  }
  if (epi == Epi::kStoreF16Delta) {
    BN = 256;
    if (!ea.attn_o || !ea.delta || ea.seq <= 0 || (ea.head_dim != 64 && ea.head_dim != 128) || ea.ld_o % 8 ||
        reinterpret_cast<uintptr_t>(ea.attn_o) % 16)
      return cudaErrorInvalidValue;
  }
  if ((epi == Epi::kSwiGLU || epi == Epi::kSwiGLUBwd || epi == Epi::kCEStream) && BN != 256)
    return cudaErrorInvalidValue;  // paired columns / partial slots assume 256-wide tiles
  if (epi == Epi::kCEStream && (!ea.targets || !ea.ce_ref || !ea.part_max || !ea.part_sum || !ea.tgt_logit ||
                                ea.vocab_off % 128 || ea.ce_slots < (ea.vocab_off + N + 127) / 128))
    return cudaErrorInvalidValue;
  if (ea.ksplit > 1 && (epi != Epi::kStoreF32 || !ea.accumulate)) return cudaErrorInvalidValue;
  const int n_main = ea.n_main > 0 ? ea.n_main : N;
  if (n_main < N) {  // side output: only for the plain stores, from a tile boundary
    if ((epi != Epi::kStoreF16 && epi != Epi::kStoreF16Delta && epi != Epi::kResidF32 &&
         epi != Epi::kQKNormRope && epi != Epi::kSwiGLU && epi != Epi::kSwiGLUBwd) ||
        n_main % BN ||
        (N - n_main) % 8 || !ea.side ||
        ea.ld_side % 8 || reinterpret_cast<uintptr_t>(ea.side) % 16)
      return cudaErrorInvalidValue;
  }
  // CTA pairs (cta_group::2) for the 256-wide tiles of matrices with more
  // than one 128-row block: each pair shares a 256 x 256 tile
  // INT8 B: 256-wide tiles; K-major needs the row scales (the epilogue applies them)
  if (B.q8 && (BN != 256 || (!B.mn && !B.q8_scale) || ea.ksplit > 1)) return cudaErrorInvalidValue;
  const int CG = (BN == 256 && M > kBlockM) ? 2 : 1;
  CUtensorMap maps[4];  // A, B, C, D
  if (!make_map(&maps[0], A, kBlockM)) return cudaErrorInvalidValue;
  if (B.q8 ? !make_map_q8(&maps[1], B, BN / CG) : !make_map(&maps[1], B, BN / CG)) return cudaErrorInvalidValue;
  bool okc = true;
  switch (epi) {
    case Epi::kStoreF16:
    case Epi::kStoreF16Delta:
    case Epi::kCEStream:
      okc = make_io_map(&maps[2], ea.out, M, n_main, ea.ld_out, false);
      maps[3] = maps[2];
      break;
    case Epi::kQKNormRope:  // C = q/k/v [M, n_main], D = normed, rotated q/k [M, n_qk_cols]
      okc = make_io_map(&maps[2], ea.out, M, n_main, ea.ld_out, false) &&
            make_io_map(&maps[3], ea.rope_out, M, ea.n_qk_cols, ea.ld_rope, false);
      break;
    case Epi::kStoreF32:
      okc = make_io_map(&maps[2], ea.out, M, N, ea.ld_out, true);
      maps[3] = maps[2];
      break;
    case Epi::kResidF32:
      okc = make_io_map(&maps[2], ea.out, M, n_main, ea.ld_out, true) &&
            make_io_map(&maps[3], ea.resid, M, n_main, ea.ld_out, true);
      break;
    case Epi::kSwiGLU:  // C = gate/up pre-activations [M, n_main], D = act [M, n_main/2]
      okc = make_io_map(&maps[2], ea.gu, M, n_main, ea.ld_gu, false) &&
            make_io_map(&maps[3], ea.act, M, n_main / 2, ea.ld_act, false);
      break;
    case Epi::kSwiGLUBwd:  // C = dgu [M, 2 n_main] out; D = the stash gu [M, 2 n_main] in 32 x 32 boxes
      okc = make_io_map(&maps[2], ea.gu, M, 2 * n_main, ea.ld_gu, false) && ea.gu_in &&
            make_box32_map(&maps[3], ea.gu_in, M, 2 * n_main, ea.ld_gu);
      break;
  }
  if (!okc) return cudaErrorInvalidValue;
  GemmShape sh;
  sh.M = M;
  sh.N = N;
  sh.K = A.k;
  sh.tiles_m = (M + kBlockM * CG - 1) / (kBlockM * CG);
  sh.tiles_n = (N + BN - 1) / BN;
  sh.num_tiles = sh.tiles_m * sh.tiles_n;
  sh.splits = 1;
  sh.kb_per_split = (A.k + kBlockK - 1) / kBlockK;
  sh.split_row_tiles = 0;
  // walk N first when A outweighs B, so the CTAs that run together share A's rows
  sh.n_fastest = static_cast<int64_t>(M) * A.k > static_cast<int64_t>(N) * B.k ? 1 : 0;
  sh.n_main = n_main;
  sh.side = ea.side;
  sh.ld_side = ea.ld_side;
  sh.fixup = 0;
  sh.fx_ws = nullptr;
  sh.fx_cnt = nullptr;
  sh.b_scale = B.mn ? nullptr : B.q8_scale;
  if (ea.ksplit > 1) {  // K slices reduce-add into the same rows
    const int nk = sh.kb_per_split;
    const int kbps = (nk + ea.ksplit - 1) / ea.ksplit;
    sh.kb_per_split = kbps;
    sh.splits = (nk + kbps - 1) / kbps;
  } else if (t_fx_ws && epi != Epi::kCEStream) {
    // tiles that fill under half a wave: K splits with a fix-up, about one
    // wave of units, at least two 64-deep K blocks each
    const int slots = CG == 2 ? g_num_sms / 2 : g_num_sms;
    const int nk = sh.kb_per_split;
    if (2 * sh.num_tiles <= slots && nk >= 4) {
      // the last split of a tile reads the others' 128 x BN fp32 partials
      // (about 2.7 K blocks' worth of loads each): splits ~ sqrt(K blocks / 2.7)
      const int balance = std::max(2, static_cast<int>(std::lround(std::sqrt(nk / 2.7))));
      int want = std::min({slots / sh.num_tiles, nk / 2, balance, 16});
      const int groups = (BN >= 128 ? 4 * kGemmEpiGroups : 4) / 4;
      const size_t per_split = static_cast<size_t>(sh.num_tiles) * CG * kBlockM * BN;  // floats
      const int cnt = sh.num_tiles * CG * 4 * groups;
      while (want > 1 && per_split * want > t_fx_ws_floats) --want;
      if (want > 1 && cnt <= t_fx_cnt_n) {
        const int kbps = (nk + want - 1) / want;
        sh.kb_per_split = kbps;
        sh.splits = (nk + kbps - 1) / kbps;
        if (sh.splits > 1) {
          sh.fixup = 1;
          sh.fx_ws = t_fx_ws;
          sh.fx_cnt = t_fx_cnt;
        }
      }
    }
  }
  if (B.q8) return CG == 2 ? dispatch_q8<2>(epi, B.mn, ea, maps, sh, err, st) : dispatch_q8<1>(epi, B.mn, ea, maps, sh, err, st);
  if (CG == 2) {
    if (B.mn) return dispatch<256, true, 2>(epi, ea, maps, sh, err, st);
    return dispatch<256, false, 2>(epi, ea, maps, sh, err, st);
  }
  if (B.mn) {
    switch (BN) {
      case 64: return dispatch<64, true, 1>(epi, ea, maps, sh, err, st);
      case 128: return dispatch<128, true, 1>(epi, ea, maps, sh, err, st);
      case 256: return dispatch<256, true, 1>(epi, ea, maps, sh, err, st);
      default: return cudaErrorInvalidValue;
    }
  }
  switch (BN) {
    case 64: return dispatch<64, false, 1>(epi, ea, maps, sh, err, st);
    case 128: return dispatch<128, false, 1>(epi, ea, maps, sh, err, st);
    case 256: return dispatch<256, false, 1>(epi, ea, maps, sh, err, st);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace llmcu
