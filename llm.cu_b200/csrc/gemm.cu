// gemm.cu -- host side of the tcgen05 GEMM: TMA descriptor encoding, tile
// shape choice and the launch of the instantiated kernels.
#include <cudaTypedefs.h>

#include <algorithm>
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

// 2-D fp16 map over rows x k (k contiguous), box = 64 (k) x box_rows, 128-B swizzle.
bool make_map(CUtensorMap* map, const Operand& op, int box_rows) {
  if (!g_encode) return false;
  if (reinterpret_cast<uintptr_t>(op.ptr) % 16 != 0 || (op.ld * 2) % 16 != 0) return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(op.k), static_cast<cuuint64_t>(op.rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(op.ld) * 2};
  cuuint32_t box[2] = {64u, static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1u, 1u};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half*>(op.ptr), dims, strides, box,
                        estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
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

// As many pipeline stages as fit beside the epilogue slabs (at most 8).
template <int BN, int EW, int SLAB>
constexpr int stages_for() {
  constexpr int stage = kBlockM * kBlockK * 2 + BN * kBlockK * 2;
  constexpr int s = (232448 - 1536 - EW * SLAB) / stage;
  return s > 8 ? 8 : s;
}

// 8 epilogue warps (two per TMEM lane quadrant) for 128/256-wide tiles, 4 for 64.
template <int BN>
constexpr int epi_warps() {
  return BN >= 128 ? 4 * kGemmEpiGroups : 4;
}

template <int BN, class E>
cudaError_t launch(const CUtensorMap* maps, const GemmShape& sh, const typename E::Params& p, int* err,
                   cudaStream_t st) {
  constexpr int kEpiWarps = epi_warps<BN>();
  constexpr int S = stages_for<BN, kEpiWarps, E::kSlab>();
  using L = GemmSmem<BN, S, kEpiWarps, E::kSlab>;
  static_assert(L::kBytes <= 232448, "shared memory budget");
  auto kern = gemm_tc_kernel<BN, S, kEpiWarps, E>;
  static bool attr_done = false;  // set once per instantiation
  if (!attr_done) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kBytes);
    if (e != cudaSuccess) return e;
    attr_done = true;
  }
  const int units = sh.num_tiles * sh.splits;
  int grid = units < g_num_sms ? units : g_num_sms;
  kern<<<grid, 64 + 32 * kEpiWarps, L::kBytes, st>>>(maps[0], maps[1], maps[2], maps[3], maps[4], maps[5], sh, p,
                                                     err);
  return cudaGetLastError();
}

template <int BN>
cudaError_t dispatch(Epi epi, const EpiArgs& ea, const CUtensorMap* maps, const GemmShape& sh, int* err,
                     cudaStream_t st) {
  switch (epi) {
    case Epi::kStoreF16:
      return launch<BN, EpiStoreF16>(maps, sh, EpiStoreF16::Params{}, err, st);
    case Epi::kStoreF32:
      return launch<BN, EpiStoreF32>(maps, sh, EpiStoreF32::Params{ea.accumulate}, err, st);
    case Epi::kResidF32:
      return launch<BN, EpiResidF32>(maps, sh, EpiResidF32::Params{}, err, st);
    case Epi::kSwiGLUBwd:
      return launch<BN, EpiSwiGLUBwd>(maps, sh, EpiSwiGLUBwd::Params{}, err, st);
    case Epi::kCEProbs: {
      if constexpr (BN == 256) {
        EpiCEProbs::Params p{ea.targets, ea.part_max, ea.part_sum, ea.tgt_logit, sh.tiles_n * (epi_warps<BN>() / 4)};
        return launch<BN, EpiCEProbs>(maps, sh, p, err, st);
      } else {
        return cudaErrorInvalidValue;
      }
    }
    case Epi::kSwiGLU: {
      if constexpr (BN == 256) {
        return launch<BN, EpiSwiGLU>(maps, sh, EpiSwiGLU::Params{}, err, st);
      } else {
        return cudaErrorInvalidValue;
      }
    }
  }
  return cudaErrorInvalidValue;
}

}  // namespace

int gemm_num_sms() {
  std::call_once(g_once, init_once);
  return g_num_sms;
}

cudaError_t gemm(const Operand& A0, const Operand& B0, const Operand& A1, const Operand& B1, int M, int N, Epi epi,
                 const EpiArgs& ea, int* err, cudaStream_t st, int bn_hint) {
  std::call_once(g_once, init_once);
  if (!g_encode) return cudaErrorNotSupported;
  if (M <= 0 || N <= 0 || A0.k <= 0 || A0.k != B0.k || A1.k != B1.k) return cudaErrorInvalidValue;
  int BN = bn_hint;
  if (BN == 0) BN = (epi == Epi::kSwiGLU) ? 256 : (N <= 64 ? 64 : (N <= 128 ? 128 : 256));
  if (epi == Epi::kSwiGLU && BN != 256) return cudaErrorInvalidValue;
  if (epi == Epi::kCEProbs && BN != 256) return cudaErrorInvalidValue;  // partial slots assume 256-wide tiles
  if (ea.ksplit > 1 && (epi != Epi::kStoreF32 || !ea.accumulate)) return cudaErrorInvalidValue;
  CUtensorMap maps[6];  // A0, B0, A1, B1, C, D
  if (!make_map(&maps[0], A0, kBlockM) || !make_map(&maps[1], B0, BN)) return cudaErrorInvalidValue;
  if (A1.k > 0) {
    if (!make_map(&maps[2], A1, kBlockM) || !make_map(&maps[3], B1, BN)) return cudaErrorInvalidValue;
  } else {
    maps[2] = maps[0];
    maps[3] = maps[1];
  }
  bool okc = true;
  switch (epi) {
    case Epi::kStoreF16:
    case Epi::kCEProbs:
      okc = make_io_map(&maps[4], ea.out, M, N, ea.ld_out, false);
      maps[5] = maps[4];
      break;
    case Epi::kStoreF32:
      okc = make_io_map(&maps[4], ea.out, M, N, ea.ld_out, true);
      maps[5] = maps[4];
      break;
    case Epi::kResidF32:
      okc = make_io_map(&maps[4], ea.out, M, N, ea.ld_out, true) &&
            make_io_map(&maps[5], ea.resid, M, N, ea.ld_out, true);
      break;
    case Epi::kSwiGLU:  // C = gate/up pre-activations [M, N], D = act [M, N/2]
      okc = make_io_map(&maps[4], ea.gu, M, N, ea.ld_gu, false) &&
            make_io_map(&maps[5], ea.act, M, N / 2, ea.ld_act, false);
      break;
    case Epi::kSwiGLUBwd:  // C = dgu [M, 2N] out, D = gu [M, 2N] in
      okc = make_io_map(&maps[4], ea.gu, M, 2 * N, ea.ld_gu, false) &&
            make_io_map(&maps[5], ea.gu_in, M, 2 * N, ea.ld_gu, false);
      break;
  }
  if (!okc) return cudaErrorInvalidValue;
  GemmShape sh;
  sh.M = M;
  sh.N = N;
  sh.K0 = A0.k;
  sh.K1 = A1.k;
  sh.tiles_m = (M + kBlockM - 1) / kBlockM;
  sh.tiles_n = (N + BN - 1) / BN;
  sh.num_tiles = sh.tiles_m * sh.tiles_n;
  sh.splits = 1;
  sh.kb_per_split = (A0.k + kBlockK - 1) / kBlockK + (A1.k + kBlockK - 1) / kBlockK;
  sh.split_row_tiles = 0;
  if (ea.ksplit > 1) {  // K slices reduce-add into the same rows
    const int nk = sh.kb_per_split;
    const int kbps = (nk + ea.ksplit - 1) / ea.ksplit;
    sh.kb_per_split = kbps;
    sh.splits = (nk + kbps - 1) / kbps;
  }
  switch (BN) {
    case 64: return dispatch<64>(epi, ea, maps, sh, err, st);
    case 128: return dispatch<128>(epi, ea, maps, sh, err, st);
    case 256: return dispatch<256>(epi, ea, maps, sh, err, st);
    default: return cudaErrorInvalidValue;
  }
}

namespace {

// out16[m, n] = sum over splits of part[(s * Mp + m) * N + n]
__global__ void splitk_reduce_kernel(const float* __restrict__ part, int splits, int Mp, int M, int N,
                                     __half* __restrict__ out, int ld_out) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;  // over M * N / 2 pairs
  if (i >= M * (N / 2)) return;
  const int m = i / (N / 2), n = 2 * (i % (N / 2));
  float a = 0.f, b = 0.f;
  for (int s = 0; s < splits; ++s) {
    const float2 v = *reinterpret_cast<const float2*>(part + (static_cast<size_t>(s) * Mp + m) * N + n);
    a += v.x;
    b += v.y;
  }
  *reinterpret_cast<__half2*>(out + static_cast<size_t>(m) * ld_out + n) = __floats2half2_rn(a, b);
}

}  // namespace

size_t gemm_skinny_ws_floats(int M, int N) {
  return static_cast<size_t>(kSkinnyMaxSplits) * ((M + kBlockM - 1) / kBlockM) * kBlockM * N;
}

cudaError_t gemm_skinny(const Operand& A, const Operand& B, int M, int N, __half* out, int ld_out, float* ws,
                        int* err, cudaStream_t st) {
  std::call_once(g_once, init_once);
  if (!g_encode) return cudaErrorNotSupported;
  if (M <= 0 || N <= 0 || N > 64 || N % 2 || A.k <= 0 || A.k != B.k) return cudaErrorInvalidValue;
  const int tiles_m = (M + kBlockM - 1) / kBlockM;
  const int nk = (A.k + kBlockK - 1) / kBlockK;
  // enough (tile, split) units to cover the SMs, each with >= 4 k-blocks
  int splits = (g_num_sms + tiles_m - 1) / tiles_m;
  splits = std::min(splits, std::max(1, nk / 4));
  splits = std::min(splits, kSkinnyMaxSplits);
  const int kbps = (nk + splits - 1) / splits;
  splits = (nk + kbps - 1) / kbps;
  const int Mp = tiles_m * kBlockM;
  CUtensorMap maps[6];
  if (!make_map(&maps[0], A, kBlockM) || !make_map(&maps[1], B, 64)) return cudaErrorInvalidValue;
  maps[2] = maps[0];
  maps[3] = maps[1];
  if (!make_io_map(&maps[4], ws, splits * Mp, N, N, true)) return cudaErrorInvalidValue;
  maps[5] = maps[4];
  GemmShape sh;
  sh.M = M;
  sh.N = N;
  sh.K0 = A.k;
  sh.K1 = 0;
  sh.tiles_m = tiles_m;
  sh.tiles_n = 1;
  sh.num_tiles = tiles_m;
  sh.splits = splits;
  sh.kb_per_split = kbps;
  sh.split_row_tiles = tiles_m;
  cudaError_t e = launch<64, EpiStoreF32>(maps, sh, EpiStoreF32::Params{0}, err, st);
  if (e != cudaSuccess) return e;
  const int pairs = M * (N / 2);
  splitk_reduce_kernel<<<(pairs + 255) / 256, 256, 0, st>>>(ws, splits, Mp, M, N, out, ld_out);
  return cudaGetLastError();
}

}  // namespace llmcu
