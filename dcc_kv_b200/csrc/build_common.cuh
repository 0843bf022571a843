// Per-problem descriptor shared by the build kernels (scoring, top-k,
// calibration).  One problem = one (source block, destination, KV head) edge.
#pragma once

#include "common.cuh"

namespace dcc {

constexpr int kMaxRepr = 64;      // representative queries per problem
constexpr int kMaxDim = 128;      // head_dim / value_dim of the CUDA-core path
constexpr int kMaxTopk = 8192;    // budget sorted in shared memory
constexpr int kScoreTile = 32;    // keys per shared-memory tile

template <typename Acc>
struct BuildDesc {
  const void* keys;
  const void* values;
  const void* repr;
  int64_t L_s, ld_k, ld_v;
  int32_t budget;     // B' = min(budget, L_s)
  int32_t M;          // representative queries
  int32_t n_chunks;   // key chunks of the scoring passes
  int32_t chunk_len;  // keys per chunk (multiple of kScoreTile)
  void* out_keys;
  void* out_values;
  void* out_bias;
  int64_t* out_idx;
  double* out_mass;
  // workspace slices
  Acc* stats;    // [n_chunks, M, 2]  (running max, sum) per chunk
  Acc* massp;    // [n_chunks, M]
  Acc* yp;       // [n_chunks, M, dv]
  Acc* u;        // [L_s] RMS scores
  double* G;     // [M, B']
  double* X;     // [M, B']  (logits, then X)
  double* Y;     // [M, dv]
  double* wv;    // [B'] NNLS weights, then beta
  double* gpart; // [n_btiles, 64, 64] partial Gram G G^T per 64-key tile (M < B')
  double* W;     // [64, dv] (X X^T + lam I)^-1 Y
  int32_t n_btiles;
  int32_t pad2;
  // per-function entry points: given inputs instead of computed ones
  const void* in_mass;  // [M] block mass (input dtype), replaces the pass-2 sums
  const void* in_beta;  // [B'] logit bias (input dtype), replaces the NNLS
  int32_t stages;       // kStageBeta | kStageValues
  int32_t pad;
};

constexpr int kStageBeta = 1;
constexpr int kStageValues = 2;

constexpr int kBuildCap = 128;
template <typename Acc>
using BuildBatch = Batch<BuildDesc<Acc>, kBuildCap>;

struct BuildParams {
  int d, dv;
  double scale;       // 1 / sqrt(head_dim)
  double lambda_beta, lambda_value;
};

}  // namespace dcc
