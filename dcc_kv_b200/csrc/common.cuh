// Shared helpers for the DCC-KV sm_100a kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "dcc_kv.h"

namespace dcc {

// ---- error plumbing -------------------------------------------------------
void set_error(const std::string& msg);
int fail(int status, const std::string& msg);
int check_cuda(cudaError_t e, const char* what);
int check_launch(const char* what);

inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// Bump allocator over a caller-provided workspace (256-byte aligned slices).
struct Workspace {
  char* base;
  size_t cap;
  size_t used = 0;
  Workspace(void* p, size_t n) : base(static_cast<char*>(p)), cap(n) {}
  template <typename T>
  T* take(size_t count) {
    size_t off = align_up(used, 256);
    used = off + count * sizeof(T);
    return base ? reinterpret_cast<T*>(base + off) : nullptr;
  }
  bool ok() const { return used <= cap; }
};

int num_sms();

// ---- element conversion ---------------------------------------------------
template <typename T> __device__ __forceinline__ double to_f64(T x);
template <> __device__ __forceinline__ double to_f64<float>(float x) { return (double)x; }
template <> __device__ __forceinline__ double to_f64<double>(double x) { return x; }
template <> __device__ __forceinline__ double to_f64<__nv_bfloat16>(__nv_bfloat16 x) {
  return (double)__bfloat162float(x);
}

template <typename T> __device__ __forceinline__ float to_f32(T x);
template <> __device__ __forceinline__ float to_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ float to_f32<double>(double x) { return (float)x; }
template <> __device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 x) {
  return __bfloat162float(x);
}

template <typename A, typename T> __device__ __forceinline__ A to_acc(T x);
template <> __device__ __forceinline__ double to_acc<double, float>(float x) { return x; }
template <> __device__ __forceinline__ double to_acc<double, double>(double x) { return x; }
template <> __device__ __forceinline__ double to_acc<double, __nv_bfloat16>(__nv_bfloat16 x) {
  return (double)__bfloat162float(x);
}
template <> __device__ __forceinline__ float to_acc<float, float>(float x) { return x; }
template <> __device__ __forceinline__ float to_acc<float, double>(double x) { return (float)x; }
template <> __device__ __forceinline__ float to_acc<float, __nv_bfloat16>(__nv_bfloat16 x) {
  return __bfloat162float(x);
}

template <typename T> __device__ __forceinline__ T from_f64(double x);
template <> __device__ __forceinline__ float from_f64<float>(double x) { return (float)x; }
template <> __device__ __forceinline__ double from_f64<double>(double x) { return x; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f64<__nv_bfloat16>(double x) {
  return __float2bfloat16_rn((float)x);
}
template <typename T> __device__ __forceinline__ T from_f32(float x);
template <> __device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ double from_f32<double>(float x) { return x; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) {
  return __float2bfloat16_rn(x);
}

__device__ __forceinline__ double acc_exp(double x) { return exp(x); }
__device__ __forceinline__ float acc_exp(float x) { return expf(x); }
__device__ __forceinline__ double acc_log(double x) { return log(x); }
__device__ __forceinline__ float acc_log(float x) { return logf(x); }
__device__ __forceinline__ double acc_sqrt(double x) { return sqrt(x); }
__device__ __forceinline__ float acc_sqrt(float x) { return sqrtf(x); }

template <typename T> struct NegInf;
template <> struct NegInf<float> { static __device__ __forceinline__ float v() { return -INFINITY; } };
template <> struct NegInf<double> { static __device__ __forceinline__ double v() { return -(double)INFINITY; } };

// ---- warp reductions --------------------------------------------------------
template <typename T>
__device__ __forceinline__ T warp_sum(T v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
template <typename T>
__device__ __forceinline__ T warp_max(T v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Kernel argument batches travel by value in the launch parameters (up to
// 32 KB on sm_90+), so a batched launch needs no descriptor upload.
template <typename P, int CAP>
struct Batch {
  int n;
  P p[CAP];
};

}  // namespace dcc

#define DCC_CHECK(expr)                  \
  do {                                   \
    int _s = (expr);                     \
    if (_s != DCC_OK) return _s;         \
  } while (0)
