// dcc_build_compact_kv_noalloc: the single-head compact-KV build for callers
// that must not allocate device memory.
//
// Its scratch is a file-scope device array of DCC_NOALLOC_SCRATCH_BYTES.  In
// host code the array's name only stands for the symbol, not for a device
// address, so the address is fetched with cudaGetSymbolAddress once per
// device (with that device current) and cached; the kernels receive that
// address like any other workspace pointer.
#include <mutex>
#include <string>

#include "common.cuh"

namespace {

static __device__ __align__(256) unsigned char g_noalloc_scratch[DCC_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_scratch_addr[kMaxDevices] = {};

int scratch_for_current_device(void** out) {
  int dev = 0;
  DCC_CHECK(dcc::check_cuda(cudaGetDevice(&dev), "build_compact_kv_noalloc: cudaGetDevice"));
  if (dev < 0 || dev >= kMaxDevices)
    return dcc::fail(DCC_ERR_UNSUPPORTED, "build_compact_kv_noalloc: device ordinal above 63");
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_scratch_addr[dev] == nullptr) {
    void* p = nullptr;
    DCC_CHECK(dcc::check_cuda(cudaGetSymbolAddress(&p, g_noalloc_scratch),
                              "build_compact_kv_noalloc: cudaGetSymbolAddress"));
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return DCC_OK;
}

}  // namespace

extern "C" int dcc_build_compact_kv_noalloc(const void* source_keys, const void* source_values,
                                            const void* destination_queries, int64_t L_s, int64_t L_r,
                                            int head_dim, int value_dim, int budget,
                                            int num_representative_queries, int projection_dim,
                                            double lambda_beta, double lambda_value, uint64_t seed,
                                            int dtype, void* out_keys, void* out_bias, void* out_values,
                                            int64_t* out_selected_indices, int64_t* out_repr_idx,
                                            void* stream) {
  if (L_s <= 0 || L_r <= 0 || budget <= 0 || num_representative_queries <= 0)
    return dcc::fail(DCC_ERR_INVALID_ARGUMENT, "build_compact_kv_noalloc: empty input or non-positive budget");
  const size_t need = dcc_build_compact_kv_workspace(L_s, L_r, head_dim, value_dim, budget,
                                                     num_representative_queries, projection_dim, dtype);
  if (need > (size_t)DCC_NOALLOC_SCRATCH_BYTES)
    return dcc::fail(DCC_ERR_UNSUPPORTED,
                     "build_compact_kv_noalloc: this problem needs " + std::to_string(need) +
                         " bytes of scratch, above the fixed " +
                         std::to_string((size_t)DCC_NOALLOC_SCRATCH_BYTES) +
                         " bytes; use dcc_build_compact_kv with a caller workspace");
  void* scratch = nullptr;
  DCC_CHECK(scratch_for_current_device(&scratch));
  // Every scratch element is written by a kernel before any kernel reads it,
  // so nothing has to be cleared between calls.
  return dcc_build_compact_kv(source_keys, source_values, destination_queries, L_s, L_r, head_dim,
                              value_dim, budget, num_representative_queries, projection_dim, lambda_beta,
                              lambda_value, seed, dtype, out_keys, out_bias, out_values,
                              out_selected_indices, out_repr_idx, scratch,
                              (size_t)DCC_NOALLOC_SCRATCH_BYTES, stream);
}
