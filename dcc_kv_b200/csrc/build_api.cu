// C entry points of the compact-KV build: argument checks, workspace
// carving and the stream-ordered kernel sequence
//   score_stats -> score_probs -> topk (+ C_K gather) -> calibrate.
#include <string>
#include <type_traits>
#include <vector>

#include "build_common.cuh"

namespace dcc {

template <typename TIn, typename Acc>
int launch_scoring(const BuildBatch<Acc>&, const BuildParams&, int, cudaStream_t);
template <typename TIn, typename Acc>
int launch_topk(const BuildBatch<Acc>&, const BuildParams&, int, cudaStream_t);
template <typename TIn, typename Acc>
int launch_calibrate(const BuildBatch<Acc>&, const BuildParams&, cudaStream_t);

// Keys per scoring chunk: a function of L_s alone, so a problem's partial
// sums combine in the same order whatever batch it is launched in.
static int chunk_len_for(int64_t L_s) {
  int64_t c = (L_s + 7) / 8;
  c = (c + kScoreTile - 1) / kScoreTile * kScoreTile;
  if (c < 256) c = 256;
  if (c > 2048) c = 2048;
  return (int)c;
}


// Lays out (or sizes, when ws.base is null) one problem's scratch.
template <typename Acc>
static void carve(Workspace& ws, const dcc_build_problem& q, int dv, BuildDesc<Acc>& d) {
  const int64_t Bp = q.budget < q.L_s ? q.budget : q.L_s;
  d.chunk_len = chunk_len_for(q.L_s);
  d.n_chunks = (int)((q.L_s + d.chunk_len - 1) / d.chunk_len);
  d.stats = ws.take<Acc>((size_t)d.n_chunks * q.num_repr * 2);
  d.massp = ws.take<Acc>((size_t)d.n_chunks * q.num_repr);
  d.yp = ws.take<Acc>((size_t)d.n_chunks * q.num_repr * dv);
  d.u = ws.take<Acc>((size_t)q.L_s);
  d.G = ws.take<double>((size_t)q.num_repr * Bp);
  d.X = ws.take<double>((size_t)q.num_repr * Bp);
  d.Y = ws.take<double>((size_t)q.num_repr * dv);
  d.wv = ws.take<double>((size_t)Bp);
  d.n_btiles = (int)((Bp + 63) / 64);
  const size_t parts = q.num_repr < Bp ? (size_t)d.n_btiles * 64 * 64 : 0;
  d.gpart = ws.take<double>(parts);
  d.W = ws.take<double>((size_t)64 * dv);
}

static size_t build_ws_bytes(const dcc_build_problem* probs, int n, int dv, int dtype) {
  Workspace ws(nullptr, 0);
  for (int i = 0; i < n; ++i) {
    if (dtype == DCC_BF16) {
      BuildDesc<float> d{};
      carve(ws, probs[i], dv, d);
    } else {
      BuildDesc<double> d{};
      carve(ws, probs[i], dv, d);
    }
  }
  return ws.used + 256;
}

enum BuildMode { kModeFull, kModeTopk, kModeBeta, kModeValues };

struct GivenInputs {  // per-function entry points (single problem)
  const void* mass = nullptr;
  const void* beta = nullptr;
};

template <typename TIn, typename Acc>
static int run_build(const dcc_build_problem* probs, int n, const BuildParams& prm, void* workspace,
                     size_t bytes, cudaStream_t st, BuildMode mode = kModeFull,
                     GivenInputs given = GivenInputs()) {
  Workspace ws(workspace, bytes);
  BuildBatch<Acc> b{};
  int max_chunks = 0, max_budget = 1;
  auto flush = [&]() -> int {
    if (b.n == 0) return DCC_OK;
    if (mode != kModeBeta) DCC_CHECK((launch_scoring<TIn, Acc>(b, prm, max_chunks, st)));
    if (mode == kModeFull || mode == kModeTopk) DCC_CHECK((launch_topk<TIn, Acc>(b, prm, max_budget, st)));
    if (mode != kModeTopk) DCC_CHECK((launch_calibrate<TIn, Acc>(b, prm, st)));
    b.n = 0;
    max_chunks = 0;
    max_budget = 1;
    return DCC_OK;
  };
  for (int i = 0; i < n; ++i) {
    const dcc_build_problem& q = probs[i];
    BuildDesc<Acc>& d = b.p[b.n++];
    d = BuildDesc<Acc>{};
    d.keys = q.keys;
    d.values = q.values;
    d.repr = q.repr;
    d.L_s = q.L_s;
    d.ld_k = q.ld_k;
    d.ld_v = q.ld_v;
    d.budget = (int32_t)(q.budget < q.L_s ? q.budget : q.L_s);
    d.M = q.num_repr;
    d.out_keys = q.out_keys;
    d.out_values = q.out_values;
    d.out_bias = q.out_bias;
    d.out_idx = q.out_idx;
    d.out_mass = q.out_mass;
    d.in_mass = given.mass;
    d.in_beta = given.beta;
    d.stages = mode == kModeFull ? (kStageBeta | kStageValues)
             : mode == kModeBeta ? kStageBeta : mode == kModeValues ? kStageValues : 0;
    carve(ws, q, prm.dv, d);
    if (d.n_chunks > max_chunks) max_chunks = d.n_chunks;
    if (d.budget < d.L_s && d.budget > max_budget) max_budget = d.budget;
    if (b.n == kBuildCap) DCC_CHECK(flush());
  }
  return flush();
}

static int check_problems(const dcc_build_problem* probs, int n, int d, int dv) {
  if (n < 0 || (n > 0 && probs == nullptr))
    return fail(DCC_ERR_INVALID_ARGUMENT, "build_compact_kv: bad problem list");
  if (d <= 0 || dv <= 0 || d > kMaxDim || dv > kMaxDim)
    return fail(DCC_ERR_UNSUPPORTED, "build_compact_kv: head_dim and value_dim must be in [1, 128]");
  for (int i = 0; i < n; ++i) {
    const dcc_build_problem& q = probs[i];
    if (!q.keys || !q.values || !q.repr || !q.out_keys || !q.out_values || !q.out_bias || !q.out_idx)
      return fail(DCC_ERR_INVALID_ARGUMENT, "build_compact_kv: null pointer in problem " + std::to_string(i));
    if (q.L_s <= 0 || q.budget <= 0)
      return fail(DCC_ERR_INVALID_ARGUMENT, "build_compact_kv: L_s and budget must be positive");
    if (q.L_s > 0x7fffffff)
      return fail(DCC_ERR_UNSUPPORTED, "build_compact_kv: L_s above 2^31");
    if (q.ld_k < d || q.ld_v < dv)
      return fail(DCC_ERR_SHAPE, "build_compact_kv: row stride smaller than the row");
    if (q.num_repr <= 0 || q.num_repr > kMaxRepr)
      return fail(DCC_ERR_UNSUPPORTED, "build_compact_kv: num_repr must be in [1, 64]");
    if (q.budget < q.L_s && q.budget > kMaxTopk)
      return fail(DCC_ERR_UNSUPPORTED, "build_compact_kv: budget above 8192 (below L_s)");
  }
  return DCC_OK;
}

}  // namespace dcc

using namespace dcc;

extern "C" size_t dcc_build_compact_kv_workspace_bytes(const dcc_build_problem* problems, int n_problems,
                                                       int head_dim, int value_dim, int dtype) {
  (void)head_dim;
  if (n_problems <= 0 || !problems) return 256;
  return build_ws_bytes(problems, n_problems, value_dim, dtype);
}

extern "C" int dcc_build_compact_kv_batched(const dcc_build_problem* problems, int n_problems,
                                            int head_dim, int value_dim, double lambda_beta,
                                            double lambda_value, int dtype, void* workspace,
                                            size_t workspace_bytes, void* stream) {
  DCC_CHECK(check_problems(problems, n_problems, head_dim, value_dim));
  if (n_problems == 0) return DCC_OK;
  const size_t need = build_ws_bytes(problems, n_problems, value_dim, dtype);
  if (!workspace || workspace_bytes < need)
    return fail(DCC_ERR_WORKSPACE, "build_compact_kv: workspace too small (need " + std::to_string(need) + " bytes)");
  BuildParams prm{head_dim, value_dim, 1.0 / sqrt((double)head_dim), lambda_beta, lambda_value};
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case DCC_F32: return run_build<float, double>(problems, n_problems, prm, workspace, workspace_bytes, st);
    case DCC_F64: return run_build<double, double>(problems, n_problems, prm, workspace, workspace_bytes, st);
    case DCC_BF16: return run_build<__nv_bfloat16, float>(problems, n_problems, prm, workspace, workspace_bytes, st);
    default: return fail(DCC_ERR_DTYPE, "build_compact_kv: unsupported dtype");
  }
}

// ---- single-head drop-in ------------------------------------------------------
static size_t elem_size(int dtype) { return dtype == DCC_BF16 ? 2 : dtype == DCC_F32 ? 4 : 8; }

static void single_problem(const void* K, const void* V, int64_t L_s, int d, int dv, int budget, int m,
                           dcc_build_problem& q) {
  q = dcc_build_problem{};
  q.keys = K;
  q.values = V;
  q.L_s = L_s;
  q.ld_k = d;
  q.ld_v = dv;
  q.budget = budget;
  q.num_repr = m;
}

extern "C" size_t dcc_build_compact_kv_workspace(int64_t L_s, int64_t L_r, int head_dim, int value_dim,
                                                 int budget, int num_representative_queries,
                                                 int projection_dim, int dtype) {
  const int m = (int)(num_representative_queries < L_r ? num_representative_queries : L_r);
  dcc_query_set qs{};
  qs.queries = nullptr;
  qs.seg_rows = L_r;
  qs.seg_stride = 0;
  qs.row_stride = head_dim;
  qs.n_seg = 1;
  size_t total = align_up((size_t)m * head_dim * elem_size(dtype), 256) + align_up((size_t)m * 8, 256);
  total += align_up(dcc_select_representative_queries_workspace_bytes(&qs, 1, head_dim, projection_dim), 256);
  dcc_build_problem q;
  single_problem(nullptr, nullptr, L_s, head_dim, value_dim, budget, m, q);
  total += build_ws_bytes(&q, 1, value_dim, dtype);
  return total + 256;
}

extern "C" int dcc_build_compact_kv(const void* source_keys, const void* source_values,
                                    const void* destination_queries, int64_t L_s, int64_t L_r,
                                    int head_dim, int value_dim, int budget,
                                    int num_representative_queries, int projection_dim,
                                    double lambda_beta, double lambda_value, uint64_t seed, int dtype,
                                    void* out_keys, void* out_bias, void* out_values,
                                    int64_t* out_selected_indices, int64_t* out_repr_idx,
                                    void* workspace, size_t workspace_bytes, void* stream) {
  if (L_s <= 0 || L_r <= 0 || budget <= 0 || num_representative_queries <= 0)
    return fail(DCC_ERR_INVALID_ARGUMENT, "build_compact_kv: empty input or non-positive budget");
  const size_t need = dcc_build_compact_kv_workspace(L_s, L_r, head_dim, value_dim, budget,
                                                     num_representative_queries, projection_dim, dtype);
  if (!workspace || workspace_bytes < need)
    return fail(DCC_ERR_WORKSPACE, "build_compact_kv: workspace too small (need " + std::to_string(need) + " bytes)");
  const int m = (int)(num_representative_queries < L_r ? num_representative_queries : L_r);
  Workspace ws(workspace, workspace_bytes);
  void* repr = ws.take<unsigned char>((size_t)m * head_dim * elem_size(dtype));
  int64_t* ridx = ws.take<int64_t>((size_t)m);
  dcc_query_set qs{};
  qs.queries = destination_queries;
  qs.seg_rows = L_r;
  qs.seg_stride = 0;
  qs.row_stride = head_dim;
  qs.n_seg = 1;
  qs.out_repr = repr;
  qs.out_idx = ridx;
  const size_t pws = dcc_select_representative_queries_workspace_bytes(&qs, 1, head_dim, projection_dim);
  void* pool_ws = ws.take<unsigned char>(pws);
  DCC_CHECK(dcc_select_representative_queries(&qs, 1, head_dim, num_representative_queries,
                                              projection_dim, seed, dtype, pool_ws, pws, stream));
  dcc_build_problem q;
  single_problem(source_keys, source_values, L_s, head_dim, value_dim, budget, m, q);
  q.repr = repr;
  q.out_keys = out_keys;
  q.out_values = out_values;
  q.out_bias = out_bias;
  q.out_idx = out_selected_indices;
  const size_t bws = build_ws_bytes(&q, 1, value_dim, dtype);
  void* build_ws = ws.take<unsigned char>(bws);
  if (!ws.ok()) return fail(DCC_ERR_WORKSPACE, "build_compact_kv: workspace layout overflow");
  DCC_CHECK(dcc_build_compact_kv_batched(&q, 1, head_dim, value_dim, lambda_beta, lambda_value, dtype,
                                         build_ws, bws, stream));
  if (out_repr_idx)
    DCC_CHECK(check_cuda(cudaMemcpyAsync(out_repr_idx, ridx, (size_t)m * 8, cudaMemcpyDeviceToDevice,
                                         static_cast<cudaStream_t>(stream)),
                         "build_compact_kv: copy repr idx"));
  return DCC_OK;
}

// ---- per-function entry points --------------------------------------------------
template <typename F>
static int dispatch_dtype(int dtype, F&& f) {
  switch (dtype) {
    case DCC_F32: return f((float*)nullptr, (double*)nullptr);
    case DCC_F64: return f((double*)nullptr, (double*)nullptr);
    case DCC_BF16: return f((__nv_bfloat16*)nullptr, (float*)nullptr);
    default: return fail(DCC_ERR_DTYPE, "unsupported dtype");
  }
}

extern "C" size_t dcc_stage_workspace_bytes(int64_t L_s, int M, int budget, int head_dim, int value_dim,
                                            int dtype) {
  dcc_build_problem q;
  single_problem(nullptr, nullptr, L_s, head_dim, value_dim, budget, M, q);
  return build_ws_bytes(&q, 1, value_dim, dtype);
}

extern "C" int dcc_select_topk_keys(const void* keys, const void* repr, int64_t L_s, int head_dim, int M,
                                    int budget, int dtype, void* out_keys, int64_t* out_idx,
                                    void* workspace, size_t workspace_bytes, void* stream) {
  dcc_build_problem q;
  single_problem(keys, keys, L_s, head_dim, head_dim, budget, M, q);
  q.repr = repr;
  q.out_keys = out_keys;
  q.out_values = out_keys;
  q.out_bias = out_keys;
  q.out_idx = out_idx;
  DCC_CHECK(check_problems(&q, 1, head_dim, head_dim));
  if (!workspace || workspace_bytes < build_ws_bytes(&q, 1, head_dim, dtype))
    return fail(DCC_ERR_WORKSPACE, "select_topk_keys: workspace too small");
  BuildParams prm{head_dim, head_dim, 1.0 / sqrt((double)head_dim), 0.0, 0.0};
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  return dispatch_dtype(dtype, [&](auto* tin, auto* acc) {
    using TIn = std::remove_pointer_t<decltype(tin)>;
    using Acc = std::remove_pointer_t<decltype(acc)>;
    return run_build<TIn, Acc>(&q, 1, prm, workspace, workspace_bytes, st, kModeTopk);
  });
}

extern "C" int dcc_fit_logit_bias(const void* repr, const void* compact_keys, const void* block_mass, int M,
                                  int budget, int head_dim, double lambda_reg, int dtype, void* out_beta,
                                  void* workspace, size_t workspace_bytes, void* stream) {
  dcc_build_problem q;
  single_problem(compact_keys, compact_keys, budget, head_dim, head_dim, budget, M, q);
  q.repr = repr;
  q.out_keys = const_cast<void*>(compact_keys);  // read as C_K by the calibration kernel
  q.out_values = out_beta;
  q.out_bias = out_beta;
  q.out_idx = reinterpret_cast<int64_t*>(out_beta);
  DCC_CHECK(check_problems(&q, 1, head_dim, head_dim));
  if (!block_mass) return fail(DCC_ERR_INVALID_ARGUMENT, "fit_logit_bias: null block mass");
  if (!workspace || workspace_bytes < build_ws_bytes(&q, 1, head_dim, dtype))
    return fail(DCC_ERR_WORKSPACE, "fit_logit_bias: workspace too small");
  BuildParams prm{head_dim, head_dim, 1.0 / sqrt((double)head_dim), lambda_reg, 0.0};
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  GivenInputs g;
  g.mass = block_mass;
  return dispatch_dtype(dtype, [&](auto* tin, auto* acc) {
    using TIn = std::remove_pointer_t<decltype(tin)>;
    using Acc = std::remove_pointer_t<decltype(acc)>;
    return run_build<TIn, Acc>(&q, 1, prm, workspace, workspace_bytes, st, kModeBeta, g);
  });
}

extern "C" int dcc_fit_compact_value(const void* repr, const void* keys, const void* values,
                                     const void* compact_keys, const void* logit_bias, int64_t L_s, int M,
                                     int budget, int head_dim, int value_dim, double lambda_reg, int dtype,
                                     void* out_values, void* workspace, size_t workspace_bytes,
                                     void* stream) {
  dcc_build_problem q;
  single_problem(keys, values, L_s, head_dim, value_dim, budget, M, q);
  q.repr = repr;
  q.out_keys = const_cast<void*>(compact_keys);
  q.out_values = out_values;
  q.out_bias = out_values;
  q.out_idx = reinterpret_cast<int64_t*>(out_values);
  DCC_CHECK(check_problems(&q, 1, head_dim, value_dim));
  if (budget > L_s) return fail(DCC_ERR_SHAPE, "fit_compact_value: more compact keys than source keys");
  if (!logit_bias) return fail(DCC_ERR_INVALID_ARGUMENT, "fit_compact_value: null logit bias");
  if (!workspace || workspace_bytes < build_ws_bytes(&q, 1, value_dim, dtype))
    return fail(DCC_ERR_WORKSPACE, "fit_compact_value: workspace too small");
  BuildParams prm{head_dim, value_dim, 1.0 / sqrt((double)head_dim), 0.0, lambda_reg};
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  GivenInputs g;
  g.beta = logit_bias;
  return dispatch_dtype(dtype, [&](auto* tin, auto* acc) {
    using TIn = std::remove_pointer_t<decltype(tin)>;
    using Acc = std::remove_pointer_t<decltype(acc)>;
    return run_build<TIn, Acc>(&q, 1, prm, workspace, workspace_bytes, st, kModeValues, g);
  });
}
