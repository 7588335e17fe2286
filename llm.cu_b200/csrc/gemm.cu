// gemm.cu -- host side of the tcgen05 GEMM: TMA descriptor encoding, tile
// shape choice and the launch of the instantiated kernels.
#include <cudaTypedefs.h>

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

template <int BN>
constexpr int stages_for() {
  return BN == 256 ? 4 : (BN == 128 ? 6 : 8);
}

template <int BN, class E>
cudaError_t launch(const CUtensorMap& a0, const CUtensorMap& b0, const CUtensorMap& a1, const CUtensorMap& b1,
                   const GemmShape& sh, const typename E::Params& p, int* err, cudaStream_t st) {
  constexpr int S = stages_for<BN>();
  using L = GemmSmem<BN, S>;
  auto kern = gemm_tc_kernel<BN, S, E>;
  static bool attr_done = false;  // set once per instantiation
  if (!attr_done) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kBytes);
    if (e != cudaSuccess) return e;
    attr_done = true;
  }
  int grid = sh.num_tiles < g_num_sms ? sh.num_tiles : g_num_sms;
  kern<<<grid, kGemmThreads, L::kBytes, st>>>(a0, b0, a1, b1, sh, p, err);
  return cudaGetLastError();
}

template <int BN>
cudaError_t dispatch(Epi epi, const EpiArgs& ea, const CUtensorMap& a0, const CUtensorMap& b0,
                     const CUtensorMap& a1, const CUtensorMap& b1, const GemmShape& sh, int* err, cudaStream_t st) {
  switch (epi) {
    case Epi::kStoreF16: {
      EpiStoreF16::Params p{static_cast<__half*>(ea.out), ea.ld_out};
      return launch<BN, EpiStoreF16>(a0, b0, a1, b1, sh, p, err, st);
    }
    case Epi::kStoreF32: {
      EpiStoreF32::Params p{static_cast<float*>(ea.out), ea.ld_out, ea.accumulate};
      return launch<BN, EpiStoreF32>(a0, b0, a1, b1, sh, p, err, st);
    }
    case Epi::kResidF32: {
      EpiResidF32::Params p{static_cast<float*>(ea.out), ea.resid, ea.ld_out};
      return launch<BN, EpiResidF32>(a0, b0, a1, b1, sh, p, err, st);
    }
    case Epi::kSwiGLUBwd: {
      EpiSwiGLUBwd::Params p{ea.gu_in, ea.gu, ea.ld_gu};
      return launch<BN, EpiSwiGLUBwd>(a0, b0, a1, b1, sh, p, err, st);
    }
    case Epi::kCEStats: {
      EpiCEStats::Params p{ea.targets, ea.part_max, ea.part_sum, ea.tgt_logit, sh.tiles_n};
      return launch<BN, EpiCEStats>(a0, b0, a1, b1, sh, p, err, st);
    }
    case Epi::kCEGrad: {
      EpiCEGrad::Params p{ea.targets, ea.lse, ea.valid, static_cast<__half*>(ea.out), ea.ld_out, ea.col_base,
                          ea.gscale};
      return launch<BN, EpiCEGrad>(a0, b0, a1, b1, sh, p, err, st);
    }
    case Epi::kSwiGLU: {
      if constexpr (BN == 256) {
        EpiSwiGLU::Params p{ea.gu, ea.ld_gu, ea.act, ea.ld_act};
        return launch<BN, EpiSwiGLU>(a0, b0, a1, b1, sh, p, err, st);
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
  CUtensorMap a0, b0, a1, b1;
  if (!make_map(&a0, A0, kBlockM) || !make_map(&b0, B0, BN)) return cudaErrorInvalidValue;
  if (A1.k > 0) {
    if (!make_map(&a1, A1, kBlockM) || !make_map(&b1, B1, BN)) return cudaErrorInvalidValue;
  } else {
    a1 = a0;
    b1 = b0;
  }
  GemmShape sh;
  sh.M = M;
  sh.N = N;
  sh.K0 = A0.k;
  sh.K1 = A1.k;
  sh.tiles_m = (M + kBlockM - 1) / kBlockM;
  sh.tiles_n = (N + BN - 1) / BN;
  sh.num_tiles = sh.tiles_m * sh.tiles_n;
  switch (BN) {
    case 64: return dispatch<64>(epi, ea, a0, b0, a1, b1, sh, err, st);
    case 128: return dispatch<128>(epi, ea, a0, b0, a1, b1, sh, err, st);
    case 256: return dispatch<256>(epi, ea, a0, b0, a1, b1, sh, err, st);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace llmcu
