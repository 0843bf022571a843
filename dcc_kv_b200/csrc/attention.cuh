// Shared declarations of the attention kernels.
#pragma once

#include "common.cuh"

namespace dcc {

constexpr int kAttnCap = 24;  // problems per launch (kernel-parameter batch)
using AttnBatch = Batch<dcc_attn_problem, kAttnCap>;

struct AttnParams {
  int n_q_heads, n_kv_heads, group, d;
  double scale;
};

template <typename TIn, typename Acc>
int launch_attn_simt(const AttnBatch& b, const AttnParams& prm, int64_t max_lq, cudaStream_t st);

int launch_attn_mma_bf16(const AttnBatch& b, const AttnParams& prm, int64_t max_lq, cudaStream_t st);

// tcgen05 path: bf16, head_dim 128, an even number of query heads per KV head,
// at most 8 KV segments per problem.
bool attn_tc05_supported(const dcc_attn_problem& p, const AttnParams& prm);
int launch_attn_tc05(const dcc_attn_problem* probs, int n, const AttnParams& prm, cudaStream_t st);

}  // namespace dcc
