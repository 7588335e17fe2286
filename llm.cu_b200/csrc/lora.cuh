// lora.cuh -- flat adapter layout and the LoRA kernel interfaces.
#pragma once

#include <cstdint>

#include "common.cuh"

namespace llmcu {

// Offsets (in floats) of each adapter inside one layer of the flat fp32
// buffer.  A [r, d_in], B [d_out, r] row-major.
struct LoraDims {
  int r, H, Q, KV;
  float scale;  // alpha / r
  int64_t oAq, oBq, oAk, oBk, oAv, oBv, oAo, oBo, per_layer;

  static LoraDims make(int r, int H, int Q, int KV, float scale) {
    LoraDims d{};
    d.r = r; d.H = H; d.Q = Q; d.KV = KV; d.scale = scale;
    int64_t o = 0;
    d.oAq = o; o += static_cast<int64_t>(r) * H;
    d.oBq = o; o += static_cast<int64_t>(Q) * r;
    d.oAk = o; o += static_cast<int64_t>(r) * H;
    d.oBk = o; o += static_cast<int64_t>(KV) * r;
    d.oAv = o; o += static_cast<int64_t>(r) * H;
    d.oBv = o; o += static_cast<int64_t>(KV) * r;
    d.oAo = o; o += static_cast<int64_t>(r) * Q;
    d.oBo = o; o += static_cast<int64_t>(H) * r;
    d.per_layer = o;
    return d;
  }
  // adapter (proj 0..3 = q, k, v, o) offsets and dims
  __host__ __device__ int64_t offA(int proj) const { return proj == 0 ? oAq : proj == 1 ? oAk : proj == 2 ? oAv : oAo; }
  __host__ __device__ int64_t offB(int proj) const { return proj == 0 ? oBq : proj == 1 ? oBk : proj == 2 ? oBv : oBo; }
  __host__ __device__ int d_in(int proj) const { return proj == 3 ? Q : H; }
  __host__ __device__ int d_out(int proj) const { return proj == 0 ? Q : proj == 3 ? H : KV; }
};

// Merged weights of one layer (see lora.cu): [QKV + 64, H + 64] and [H + 64, Q + 64].
inline int64_t merged_qkv_elems(const LoraDims& d) {
  return (static_cast<int64_t>(d.Q + 2 * d.KV) + 64) * (d.H + 64);
}
inline int64_t merged_o_elems(const LoraDims& d) { return (static_cast<int64_t>(d.H) + 64) * (d.Q + 64); }

// Base q/k/v and o weights of every layer: fp16 (w*) or INT8 rows (q*) with
// per-row scales (s*); *_layer = elements between consecutive layers.
struct MergeWeights {
  const __half *wqkv = nullptr, *wo = nullptr;
  const int8_t *q_qkv = nullptr, *q_o = nullptr;
  const float *s_qkv = nullptr, *s_o = nullptr;
  int64_t w_layer_qkv = 0, w_layer_o = 0, s_layer_qkv = 0, s_layer_o = 0;
};

constexpr int kLoraMaxProbs = 8;
// first column of the k and v rank segments in the 64-wide LoRA operands
constexpr int kSegK = 16;
constexpr int kSegV = 32;
constexpr int kLoraMaxSplits = 16;

// C[a, 16*g + b] = scale * sum_m U[m, a] * W[m, 16*g + b]  for a < A,
// g < groups (<= 4), b < Bn (<= 16); group g is stored at
// out[g][a * sa + b * sb].  One pass over U serves every group, so the three
// dA of q/k/v (which share the normed input) read it once.
struct LoraGradProb {
  const __half* U;
  int ldu;
  const __half* W;  // 64 columns are read from here on (the padded LoRA width)
  int ldw;
  float* out[4];
  int groups;
  int sa, sb;
  int A, Bn;
  float scale;
};
struct LoraGradBatch {
  LoraGradProb p[kLoraMaxProbs];
  int n;
  int a_max;  // >= every A
};

cudaError_t lora_merge(const float* flat, const LoraDims& d, int n_layers, const MergeWeights& base, __half* mqkv,
                       __half* mo, cudaStream_t st);
// Adds into out[] (which the caller zeroes first).
cudaError_t lora_grad(const LoraGradBatch& batch, int M, cudaStream_t st);
int lora_grad_splits(int M, int a_max, int n);

}  // namespace llmcu
