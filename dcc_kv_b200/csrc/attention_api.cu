// C entry point of the segmented, biased attention.
#include <string>

#include "attention.cuh"

using namespace dcc;

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

extern "C" int dcc_attention_fwd(const dcc_attn_problem* problems, int n_problems, int n_q_heads,
                                 int n_kv_heads, int head_dim, double scale, int dtype, void* stream) {
  if (n_problems < 0 || (n_problems > 0 && !problems))
    return fail(DCC_ERR_INVALID_ARGUMENT, "attention_fwd: bad problem list");
  if (n_q_heads <= 0 || n_kv_heads <= 0 || n_q_heads % n_kv_heads != 0)
    return fail(DCC_ERR_INVALID_ARGUMENT, "attention_fwd: n_q_heads must be a multiple of n_kv_heads");
  if (head_dim <= 0 || head_dim > 128)
    return fail(DCC_ERR_UNSUPPORTED, "attention_fwd: head_dim must be in [1, 128]");
  if (n_q_heads > 65535) return fail(DCC_ERR_UNSUPPORTED, "attention_fwd: too many heads");
  bool mma = dtype == DCC_BF16 && head_dim == 128;
  for (int i = 0; i < n_problems; ++i) {
    const dcc_attn_problem& p = problems[i];
    if (!p.q || !p.o || p.Lq < 0 || p.n_seg < 0 || p.n_seg > DCC_MAX_SEGMENTS)
      return fail(DCC_ERR_INVALID_ARGUMENT, "attention_fwd: bad problem " + std::to_string(i));
    if (p.q_row_stride < head_dim || p.o_row_stride < head_dim)
      return fail(DCC_ERR_SHAPE, "attention_fwd: row stride smaller than head_dim");
    if ((p.o_init == nullptr) != (p.lse_init == nullptr))
      return fail(DCC_ERR_INVALID_ARGUMENT, "attention_fwd: o_init and lse_init come together");
    mma = mma && (!p.o_init || aligned16(p.o_init)) && aligned16(p.q) && aligned16(p.o) && p.q_row_stride % 8 == 0 &&
          p.q_head_stride % 8 == 0 && p.o_row_stride % 8 == 0 && p.o_head_stride % 8 == 0;
    for (int s = 0; s < p.n_seg; ++s) {
      const dcc_kv_segment& g = p.seg[s];
      if (g.len < 0 || (g.len > 0 && (!g.k || !g.v)) || g.row_stride < head_dim)
        return fail(DCC_ERR_INVALID_ARGUMENT, "attention_fwd: bad KV segment");
      if (g.len == 0) continue;  // no keys: nothing is read
      mma = mma && aligned16(g.k) && aligned16(g.v) && g.row_stride % 8 == 0 &&
            g.k_head_stride % 8 == 0 && g.v_head_stride % 8 == 0;
    }
  }
  if (n_problems == 0) return DCC_OK;
  AttnParams prm{n_q_heads, n_kv_heads, n_q_heads / n_kv_heads, head_dim, scale};
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (mma) {  // bf16, d 128, 16-byte aligned rows: the tcgen05 kernel when the shape allows
    bool tc = true;
    for (int i = 0; i < n_problems; ++i) tc = tc && attn_tc05_supported(problems[i], prm);
    if (tc) return launch_attn_tc05(problems, n_problems, prm, st);
  }
  AttnBatch b{};
  int64_t max_lq = 0;
  auto flush = [&]() -> int {
    if (b.n == 0 || max_lq == 0) { b.n = 0; return DCC_OK; }
    if ((max_lq + 15) / 16 > 2147483647LL) return fail(DCC_ERR_UNSUPPORTED, "attention_fwd: Lq too large");
    int rc;
    if (mma) rc = launch_attn_mma_bf16(b, prm, max_lq, st);
    else if (dtype == DCC_BF16) rc = launch_attn_simt<__nv_bfloat16, float>(b, prm, max_lq, st);
    else if (dtype == DCC_F32) rc = launch_attn_simt<float, double>(b, prm, max_lq, st);
    else if (dtype == DCC_F64) rc = launch_attn_simt<double, double>(b, prm, max_lq, st);
    else rc = fail(DCC_ERR_DTYPE, "attention_fwd: unsupported dtype");
    b.n = 0;
    max_lq = 0;
    return rc;
  };
  for (int i = 0; i < n_problems; ++i) {
    b.p[b.n++] = problems[i];
    if (problems[i].Lq > max_lq) max_lq = problems[i].Lq;
    if (b.n == kAttnCap) DCC_CHECK(flush());
  }
  return flush();
}
