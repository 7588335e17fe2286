// lora.cuh -- flat adapter layout and the LoRA kernel interfaces.
#pragma once

#include <cstdint>

#include "common.cuh"

namespace llmcu {

// Adapter ids: q, k, v, o (the reference's four, include/lora.h:22-27),
// then the MLP's gate, up and down projections.
enum LoraProj : int { kPQ = 0, kPK = 1, kPV = 2, kPO = 3, kPGate = 4, kPUp = 5, kPDown = 6, kNumProj = 7 };
constexpr uint32_t kTargetsAttn = 0x0Fu;
constexpr uint32_t kTargetsMlp = 0x70u;

// Offsets (in floats) of each adapter inside one layer of the flat fp32
// buffer.  A [r, d_in], B [d_out, r] row-major; the enabled adapters follow
// one another in id order (A then B), a disabled one has offsets -1.
struct LoraDims {
  int r, H, Q, KV, I;
  float scale;        // alpha / r
  uint32_t targets;   // bit p: adapter p is trained
  int64_t oA[kNumProj], oB[kNumProj], per_layer;

  static LoraDims make(int r, int H, int Q, int KV, int I, float scale, uint32_t targets) {
    LoraDims d{};
    d.r = r; d.H = H; d.Q = Q; d.KV = KV; d.I = I; d.scale = scale; d.targets = targets;
    int64_t o = 0;
    for (int p = 0; p < kNumProj; ++p) {
      d.oA[p] = d.oB[p] = -1;
      if (!d.has(p)) continue;
      d.oA[p] = o; o += static_cast<int64_t>(r) * d.d_in(p);
      d.oB[p] = o; o += static_cast<int64_t>(d.d_out(p)) * r;
    }
    d.per_layer = o;
    return d;
  }
  __host__ __device__ bool has(int p) const { return (targets >> p) & 1u; }
  __host__ __device__ bool has_mlp() const { return (targets & kTargetsMlp) != 0u; }
  __host__ __device__ int64_t offA(int p) const { return oA[p]; }
  __host__ __device__ int64_t offB(int p) const { return oB[p]; }
  __host__ __device__ int d_in(int p) const { return p == kPO ? Q : p == kPDown ? I : H; }
  __host__ __device__ int d_out(int p) const {
    return p == kPQ ? Q : (p == kPK || p == kPV) ? KV : (p == kPGate || p == kPUp) ? I : H;
  }
};

// Merged weights of one layer (see lora.cu): q/k/v [QKV + 64, H + 64],
// o [H + 64, Q + 64], gate/up (128-row interleaved) [2I + 64, H + 64] and
// down [H + 64, I + 64].
inline int64_t merged_qkv_elems(const LoraDims& d) {
  return (static_cast<int64_t>(d.Q + 2 * d.KV) + 64) * (d.H + 64);
}
inline int64_t merged_o_elems(const LoraDims& d) { return (static_cast<int64_t>(d.H) + 64) * (d.Q + 64); }
inline int64_t merged_gu_elems(const LoraDims& d) { return (2 * static_cast<int64_t>(d.I) + 64) * (d.H + 64); }
inline int64_t merged_d_elems(const LoraDims& d) { return (static_cast<int64_t>(d.H) + 64) * (d.I + 64); }

// One fused base weight of every layer: fp16 (w) or INT8 rows (q) with
// per-row scales (s); *_layer = elements between consecutive layers.
struct MergeBase {
  const __half* w = nullptr;
  const int8_t* q = nullptr;
  const float* s = nullptr;
  int64_t w_layer = 0, s_layer = 0;
};
// The base weights lora_merge reads: q/k/v, o and (for the MLP targets)
// gate/up (interleaved) and down.
struct MergeWeights {
  MergeBase qkv, o, gu, d;
};
// Where lora_merge writes: layer 0 of each merged weight, consecutive layers
// merged_*_elems apart (gu / d are null without MLP targets).
struct MergedOut {
  __half *qkv = nullptr, *o = nullptr, *gu = nullptr, *d = nullptr;
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
// A null out[g] skips group g (an adapter that is not trained).  With ilv
// set, U's columns are the gate/up interleave (128-column blocks, gate
// first): a column a belongs to group sel = (a >> 7) & 1 alone, and lands
// in out[sel] at row ((a >> 8) << 7) + (a & 127).
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
  int ilv;
};
struct LoraGradBatch {
  LoraGradProb p[kLoraMaxProbs];
  int n;
  int a_max;  // >= every A
  // split reduction: each m-split's fp32 partial [64 columns][128 a-rows] of
  // an (a-tile, problem) goes to ws (fewer splits when it would not fit, one
  // without ws), and a second kernel sums them in split order -- the same
  // sums whatever the order in which the splits finish.  err receives the bit
  // of a bounded wait that gave up (null: none).
  float* ws = nullptr;
  size_t ws_floats = 0;
  int* err = nullptr;
};

cudaError_t lora_merge(const float* flat, const LoraDims& d, int n_layers, const MergeWeights& base,
                       const MergedOut& out, cudaStream_t st);
// Stores into out[] (each element written once, in a fixed summation order);
// two launches when the m range is split.
cudaError_t lora_grad(const LoraGradBatch& batch, int M, cudaStream_t st);
// m-splits of a lora_grad launch (the kernels it launches: 1, or 2 when split)
int lora_grad_splits(int M, const LoraGradBatch& batch);

}  // namespace llmcu
