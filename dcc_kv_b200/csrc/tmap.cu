// Host-side TMA descriptor encoding through the driver entry point (no
// link-time dependency on libcuda).
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"
#include "tc05.cuh"

namespace dcc {

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

int make_tmap_bf16_3d(CUtensorMap* map, const void* base, uint64_t dim0, uint64_t dim1, uint64_t dim2,
                      uint64_t stride1, uint64_t stride2, uint32_t box_rows) {
  auto fn = encode_fn();
  if (!fn) return fail(DCC_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  if ((reinterpret_cast<uintptr_t>(base) & 15u) || (stride1 * 2) % 16 || (stride2 * 2) % 16)
    return fail(DCC_ERR_UNSUPPORTED, "tensor map: base and strides must be 16-byte aligned");
  cuuint64_t dims[3] = {dim0, dim1 > 0 ? dim1 : 1, dim2 > 0 ? dim2 : 1};
  cuuint64_t strides[2] = {stride1 * 2, stride2 * 2};
  if (dims[2] == 1) strides[1] = strides[0] * dims[1];  // unused dimension: any consistent stride
  cuuint32_t box[3] = {64, box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(DCC_ERR_CUDA, "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
  return DCC_OK;
}

}  // namespace dcc
