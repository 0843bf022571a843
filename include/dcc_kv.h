/*
 * dcc_kv.h -- C ABI of the B200 (sm_100a) DCC-KV compact-KV library.
 *
 * Every entry point takes plain device pointers, sizes and a cudaStream_t
 * (passed as void*), returns an int status (DCC_OK == 0) and never allocates
 * device memory: scratch comes in through (workspace, workspace_bytes), sized
 * by the matching *_workspace_bytes() query.  Work is enqueued on the given
 * stream; the call returns without synchronising.  A failed call leaves a
 * message for dcc_last_error() (per host thread).
 *
 * Names follow the reference (lfei7199-star/dcc-kv, src/dcc_kv_ref and
 * src/distributed); each declaration cites the reference interface it
 * replaces.  Tensors are row-major; strides are in elements.
 */
#ifndef DCC_KV_H_
#define DCC_KV_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes (the Python host maps them to exceptions) ------------ */
enum {
  DCC_OK = 0,
  DCC_ERR_INVALID_ARGUMENT = 1, /* ValueError (comm.py:202-222 style checks) */
  DCC_ERR_SHAPE = 2,            /* shape contract (compact_kv.py:39-47 asserts) */
  DCC_ERR_DTYPE = 3,            /* unsupported element type */
  DCC_ERR_WORKSPACE = 4,        /* workspace smaller than *_workspace_bytes() */
  DCC_ERR_CUDA = 5,             /* a CUDA runtime call failed */
  DCC_ERR_UNSUPPORTED = 6,      /* size outside what the kernels handle */
  DCC_ERR_TIMEOUT = 7           /* a bounded device-side wait expired */
};

/* ---- element types -------------------------------------------------------
 * DCC_F32 and DCC_F64 inputs run the parity path: every reduction, solve and
 * score is computed in FP64 on CUDA cores.  DCC_BF16 inputs run the
 * throughput path: contractions in bf16 with fp32 accumulation, the small
 * ridge / NNLS systems still in FP64. */
enum { DCC_F32 = 0, DCC_BF16 = 1, DCC_F64 = 2 };

const char* dcc_status_string(int status);
const char* dcc_last_error(void);
/* ABI version: 2 added the initial state of dcc_attn_problem. */
int dcc_version(void);
/* sizeof of an ABI struct by its name ("dcc_query_set", "dcc_build_problem",
 * "dcc_kv_segment", "dcc_attn_problem"), 0 for an unknown name -- lets a
 * foreign-function binding check its struct layouts. */
size_t dcc_struct_size(const char* name);

/* ---- host-side random draws (torch.Generator-compatible mt19937) ---------
 * Replaces representative_query.py:10-31 (rademacher_projection): writes
 * P[projection_dim, head_dim] = (2*randint{0,1}-1)/sqrt(projection_dim) in
 * float32, bit-identical to torch's CPU generator seeded with `seed`. */
int dcc_rademacher_projection(int head_dim, int projection_dim, uint64_t seed, float* out_host);
/* Replaces representative_query.py:68: int(torch.randint(0, N, (1,), generator=seed)). */
int64_t dcc_fps_start_index(int64_t num_points, uint64_t seed);

/* ---- representative queries ----------------------------------------------
 * Replaces representative_query.py:82-110 (select_representative_queries,
 * with farthest_point_sampling :34-79).  One query set = the destination
 * queries of one (destination block, KV head): n_seg segments of seg_rows
 * rows (row stride row_stride, segment starts seg_stride elements apart),
 * concatenated in segment order.  Output: the first min(M, N) rows of
 * out_repr [M, head_dim] (same dtype as the queries, contiguous) and of
 * out_idx [M] (indices into the concatenated rows). */
typedef struct dcc_query_set {
  const void* queries;
  int64_t seg_rows;
  int64_t seg_stride;
  int64_t row_stride;
  int32_t n_seg;
  int32_t reserved;
  void* out_repr;
  int64_t* out_idx;
} dcc_query_set;

size_t dcc_select_representative_queries_workspace_bytes(const dcc_query_set* sets, int n_sets,
                                                         int head_dim, int projection_dim);
int dcc_select_representative_queries(const dcc_query_set* sets, int n_sets, int head_dim,
                                      int num_samples, int projection_dim, uint64_t seed, int dtype,
                                      void* workspace, size_t workspace_bytes, void* stream);

/* ---- compact KV build from representative queries ------------------------
 * Replaces compact_kv.py:50-118 stages 2-4: select_topk_keys
 * (key_selection.py:29-62), block mass (compact_kv.py:97-101), fit_logit_bias
 * (calibration.py:63-94, nonneg_least_squares :17-60) and fit_compact_value
 * (value_regression.py:38-78).  One problem = one (source block, destination,
 * KV head) edge.  B' = min(budget, L_s) rows are written:
 *   out_keys [B', head_dim] and out_values [B', value_dim] in the input dtype,
 *   out_bias [B'] (double for DCC_F64, float otherwise), out_idx [B'] int64,
 *   out_mass [num_repr] double (optional, may be NULL). */
typedef struct dcc_build_problem {
  const void* keys;   /* [L_s, head_dim], row stride ld_k */
  const void* values; /* [L_s, value_dim], row stride ld_v */
  const void* repr;   /* [num_repr, head_dim] contiguous */
  int64_t L_s;
  int64_t ld_k;
  int64_t ld_v;
  int32_t budget;
  int32_t num_repr;
  void* out_keys;
  void* out_values;
  void* out_bias;
  int64_t* out_idx;
  double* out_mass;
} dcc_build_problem;

size_t dcc_build_compact_kv_workspace_bytes(const dcc_build_problem* problems, int n_problems,
                                            int head_dim, int value_dim, int dtype);
int dcc_build_compact_kv_batched(const dcc_build_problem* problems, int n_problems, int head_dim,
                                 int value_dim, double lambda_beta, double lambda_value, int dtype,
                                 void* workspace, size_t workspace_bytes, void* stream);

/* Single-head drop-in for build_compact_kv (compact_kv.py:50-60): source_keys
 * [L_s, head_dim], source_values [L_s, value_dim], destination_queries
 * [L_r, head_dim], all contiguous.  Outputs as above with num_repr =
 * min(num_representative_queries, L_r); out_repr_idx [num_repr] may be NULL. */
size_t dcc_build_compact_kv_workspace(int64_t L_s, int64_t L_r, int head_dim, int value_dim,
                                      int budget, int num_representative_queries,
                                      int projection_dim, int dtype);
int dcc_build_compact_kv(const void* source_keys, const void* source_values,
                         const void* destination_queries, int64_t L_s, int64_t L_r, int head_dim,
                         int value_dim, int budget, int num_representative_queries,
                         int projection_dim, double lambda_beta, double lambda_value,
                         uint64_t seed, int dtype, void* out_keys, void* out_bias,
                         void* out_values, int64_t* out_selected_indices, int64_t* out_repr_idx,
                         void* workspace, size_t workspace_bytes, void* stream);

/* No counterpart in the reference.  The single-head build above for callers
 * that cannot call cudaMalloc: a plugin inside a host application that owns
 * all device memory through its own fixed pool, or a latency-critical path
 * where an allocation could fail or stall.  Same arguments and outputs as
 * dcc_build_compact_kv without the workspace; the scratch is a fixed
 * DCC_NOALLOC_SCRATCH_BYTES (16 MiB) device array inside the library, held
 * by every GPU that loads it until the process exits.  Problems whose
 * dcc_build_compact_kv_workspace() exceeds that size are rejected with
 * DCC_ERR_UNSUPPORTED.  The first call on a device looks up the array's
 * address (cudaGetSymbolAddress); make that first call before any stream
 * capture.  All calls share the one array and nothing in it has to start at
 * zero: calls that overlap on the GPU (other streams, other threads) race,
 * so serialise them. */
#define DCC_NOALLOC_SCRATCH_BYTES (16u << 20)
int dcc_build_compact_kv_noalloc(const void* source_keys, const void* source_values,
                                 const void* destination_queries, int64_t L_s, int64_t L_r,
                                 int head_dim, int value_dim, int budget,
                                 int num_representative_queries, int projection_dim,
                                 double lambda_beta, double lambda_value, uint64_t seed, int dtype,
                                 void* out_keys, void* out_bias, void* out_values,
                                 int64_t* out_selected_indices, int64_t* out_repr_idx,
                                 void* stream);

/* ---- stage kernels exposed for the per-function API -----------------------
 * Scratch for the three single-problem stage entry points below. */
size_t dcc_stage_workspace_bytes(int64_t L_s, int M, int budget, int head_dim, int value_dim, int dtype);
/* select_topk_keys (key_selection.py:29-62): keys [L_s, head_dim], repr
 * [M, head_dim] -> out_keys [B', head_dim], out_idx [B'] (B' = min(budget, L_s)). */
int dcc_select_topk_keys(const void* keys, const void* repr, int64_t L_s, int head_dim, int M,
                         int budget, int dtype, void* out_keys, int64_t* out_idx, void* workspace,
                         size_t workspace_bytes, void* stream);
/* fit_logit_bias (calibration.py:63-94): repr [M, head_dim], compact_keys
 * [B, head_dim], block_mass [M] -> out_beta [B].  block_mass and out_beta are
 * double for DCC_F64 and float for DCC_F32 / DCC_BF16. */
int dcc_fit_logit_bias(const void* repr, const void* compact_keys, const void* block_mass, int M,
                       int budget, int head_dim, double lambda_reg, int dtype, void* out_beta,
                       void* workspace, size_t workspace_bytes, void* stream);
/* fit_compact_value (value_regression.py:38-78): repr [M, head_dim], keys
 * [L_s, head_dim], values [L_s, value_dim], compact_keys [B, head_dim],
 * logit_bias [B] (double for DCC_F64, float otherwise) -> out_values
 * [B, value_dim] (input dtype). */
int dcc_fit_compact_value(const void* repr, const void* keys, const void* values,
                          const void* compact_keys, const void* logit_bias, int64_t L_s, int M,
                          int budget, int head_dim, int value_dim, double lambda_reg, int dtype,
                          void* out_values, void* workspace, size_t workspace_bytes, void* stream);
/* farthest_point_sampling (representative_query.py:34-79): features [N, dim]
 * (normalised once more inside, as the reference does) -> out_idx
 * [min(num_samples, N)] int64. */
size_t dcc_farthest_point_sampling_workspace_bytes(int64_t N, int dim);
int dcc_farthest_point_sampling(const void* features, int64_t N, int dim, int num_samples,
                                uint64_t seed, int dtype, int64_t* out_idx, void* workspace,
                                size_t workspace_bytes, void* stream);
/* rms_per_token_score (key_selection.py:14-26): attention [M, L] -> u [L]. */
int dcc_rms_per_token_score(const void* attention, int64_t M, int64_t L, int dtype, void* out,
                            void* stream);
/* nonneg_least_squares (calibration.py:17-60): G [M, B], target [M] -> w [B],
 * FP64 throughout (inputs converted); dtype of G/target/w given by `dtype`. */
size_t dcc_nnls_workspace_bytes(int64_t M, int64_t B);
int dcc_nonneg_least_squares(const void* G, const void* target, int64_t M, int64_t B,
                             double lambda_reg, int n_iter, int dtype, void* out_w,
                             void* workspace, size_t workspace_bytes, void* stream);
/* ridge_regression_value (value_regression.py:15-35): X [M, B], Y [M, D] -> [B, D]. */
size_t dcc_ridge_workspace_bytes(int64_t M, int64_t B, int64_t D);
int dcc_ridge_regression_value(const void* X, const void* Y, int64_t M, int64_t B, int64_t D,
                               double lambda_reg, int dtype, void* out, void* workspace,
                               size_t workspace_bytes, void* stream);

/* ---- attention over KV segments with optional per-key logit bias ---------
 * Computes, per query row, the normalised softmax(q K^T * scale + bias) V and
 * its natural-log LSE over the concatenation of up to DCC_MAX_SEGMENTS KV
 * segments.  Segment 0 may be causal: query row i then sees its keys
 * j <= i + causal_offset.  This is the local-block path of
 * dcc_kv_sync_cpu.py:52-55 and the compact path :71-74 (bias added at full
 * weight), batched over heads with GQA (query head h reads KV head
 * h / (n_q_heads / n_kv_heads)). */
#define DCC_MAX_SEGMENTS 16
typedef struct dcc_kv_segment {
  const void* k;       /* [n_kv_heads, len, head_dim] */
  const void* v;
  const float* bias;   /* [n_kv_heads, len] or NULL */
  int64_t k_head_stride;
  int64_t v_head_stride;
  int64_t row_stride;  /* K and V row stride */
  int64_t bias_head_stride;
  int64_t len;
} dcc_kv_segment;

typedef struct dcc_attn_problem {
  const void* q;       /* [n_q_heads, Lq, head_dim] */
  int64_t q_head_stride, q_row_stride;
  void* o;             /* [n_q_heads, Lq, head_dim], query dtype */
  int64_t o_head_stride, o_row_stride;
  float* lse;          /* [n_q_heads, Lq] or NULL */
  int64_t lse_head_stride;
  int64_t Lq;
  int32_t n_seg;
  int32_t causal;
  int64_t causal_offset;
  dcc_kv_segment seg[DCC_MAX_SEGMENTS];
  /* Optional initial online-softmax state (NULL: none): a normalised partial
   * output o_init (o's shape and strides, may alias o) with its log-sum-exp
   * lse_init ([n_q_heads, Lq], may alias lse).  The rows continue from
   * (m = lse_init, l = 1, o = o_init), so the result is the merge of that
   * state with the attention over the segments (online_softmax.py:92-111). */
  const void* o_init;
  const float* lse_init;
  int64_t lse_init_head_stride;
} dcc_attn_problem;

int dcc_attention_fwd(const dcc_attn_problem* problems, int n_problems, int n_q_heads,
                      int n_kv_heads, int head_dim, double scale, int dtype, void* stream);
/* Synchronises the current device and reports whether a bounded device-side
 * wait of the tcgen05 attention kernel expired since the last clear
 * (DCC_ERR_TIMEOUT), clearing the flag when `clear` is non-zero. */
int dcc_device_error_status(int clear);
/* The same for the tcgen05 scoring passes of the compact-KV build. */
int dcc_build_error_status(int clear);
/* Enqueues on `stream` one tiny kernel that writes the two bounded-wait
 * error words (host_flags[0]: tcgen05 attention, host_flags[1]: tcgen05
 * scoring) into caller-owned pinned host memory, device-accessible under
 * unified addressing (no copy engine, no synchronisation).  Non-zero once
 * the stream has passed the kernel means a wait expired; the
 * layers read the pair at their next call instead of synchronising.  No
 * counterpart in the reference, whose CPU path has no device waits; the
 * timeout maps to the RuntimeError style of comm.py:97-99. */
int dcc_device_error_flags_async(unsigned int* host_flags, void* stream);
/* Test hook for the error path: one warp waits `limit_ns` (at most 100 ms)
 * on an mbarrier that nothing arrives at, then records a timeout in the
 * attention error word -- a wait that runs out without any fault. */
int dcc_debug_expire_wait(uint64_t limit_ns, void* stream);

/* ---- online softmax ------------------------------------------------------
 * online_softmax_from_attention (online_softmax.py:52-89), batched: logits
 * [R, L] (+ bias [L]) and values [L, D] shared by every row (values_row_stride
 * == 0) or [R, L, D] -> m [R], l [R], o [R, D] (o unnormalised). */
int dcc_online_softmax_from_attention(const void* logits, const void* values,
                                      const void* logit_bias, int64_t R, int64_t L, int64_t D,
                                      int64_t values_row_stride, int dtype, void* out_m,
                                      void* out_l, void* out_o, void* stream);
/* merge_softmax_states (online_softmax.py:92-111), elementwise over R rows:
 * (m, l, o[D]) x 2 -> (m, l, o). */
int dcc_merge_softmax_states(const void* m_a, const void* l_a, const void* o_a, const void* m_b,
                             const void* l_b, const void* o_b, int64_t R, int64_t D, int dtype,
                             void* out_m, void* out_l, void* out_o, void* stream);
/* P-way merge of normalised partial outputs: O = sum_p exp(lse_p - lse) O_p,
 * lse = log sum_p exp(lse_p) -- the (m=lse, l=1, o=O) form of
 * merge_softmax_states folded over P states.  o_parts[p] [R, D] contiguous,
 * lse_parts[p] [R] float32; out [R, D] (dtype), lse_out [R] (may be NULL). */
int dcc_merge_lse(const void* const* o_parts, const float* const* lse_parts, int n_parts, int64_t R,
                  int64_t D, int dtype, void* out, float* lse_out, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* DCC_KV_H_ */
