// Online-softmax kernels: P-way LSE merge, pairwise (m, l, o) merge and the
// (m, l, o) state of a row of logits.
//
// dcc_merge_lse is the HBM-bound merge of the partial attention outputs
// (online_softmax.py:92-111 folded over P states in (m=lse, l=1, o=O) form).
// Each thread owns 16 bytes of one output row and streams the same 16-byte
// slice of every part, so a warp keeps P independent 512-byte loads in flight
// per row pair; the grid is a multiple of the SM count and grid-strides.
#include "common.cuh"

namespace dcc {

constexpr int kMaxParts = 64;

struct MergeArgs {
  const void* o[kMaxParts];
  const float* lse[kMaxParts];
  int n_parts;
  int64_t rows;
  int64_t dim;
  void* out;
  float* lse_out;
};

template <typename T> struct Vec16 { static constexpr int N = 16 / sizeof(T); };

template <typename T, typename Acc>
__device__ __forceinline__ void load_vec(const T* p, Acc* v) {
  constexpr int N = Vec16<T>::N;
  uint4 raw = __ldcs(reinterpret_cast<const uint4*>(p));  // streamed once
  const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
  for (int i = 0; i < N; ++i) v[i] = to_acc<Acc, T>(e[i]);
}

template <typename T, typename Acc>
__device__ __forceinline__ void store_vec(T* p, const Acc* v) {
  constexpr int N = Vec16<T>::N;
  uint4 raw;
  T* e = reinterpret_cast<T*>(&raw);
#pragma unroll
  for (int i = 0; i < N; ++i) e[i] = from_f64<T>((double)v[i]);
  __stcs(reinterpret_cast<uint4*>(p), raw);
}

template <> __device__ __forceinline__ void store_vec<__nv_bfloat16, float>(__nv_bfloat16* p, const float* v) {
  uint4 raw;
  __nv_bfloat162* e = reinterpret_cast<__nv_bfloat162*>(&raw);
#pragma unroll
  for (int i = 0; i < 4; ++i) e[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
  __stcs(reinterpret_cast<uint4*>(p), raw);
}

// Vectorised path: dim % (16 / sizeof(T)) == 0 and 16-byte aligned rows.
template <typename T, typename Acc, int P>
__global__ void __launch_bounds__(256) merge_lse_vec_kernel(const __grid_constant__ MergeArgs a) {
  constexpr int N = Vec16<T>::N;
  const int64_t vec_per_row = a.dim / N;
  const int64_t total = a.rows * vec_per_row;
  const int np = P > 0 ? P : a.n_parts;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = i / vec_per_row;
    const int64_t col = (i - row * vec_per_row) * N;
    float lse[P > 0 ? P : kMaxParts];
    float m = -INFINITY;
#pragma unroll
    for (int p = 0; p < (P > 0 ? P : kMaxParts); ++p) {
      if (p < np) {
        lse[p] = __ldg(a.lse[p] + row);
        m = fmaxf(m, lse[p]);
      }
    }
    Acc acc[N];
#pragma unroll
    for (int j = 0; j < N; ++j) acc[j] = Acc(0);
    Acc wsum = Acc(0);
    if (m != -INFINITY) {
#pragma unroll
      for (int p = 0; p < (P > 0 ? P : kMaxParts); ++p) {
        if (p < np) {
          const Acc w = acc_exp(Acc(lse[p]) - Acc(m));
          wsum += w;
          Acc v[N];
          load_vec<T, Acc>(static_cast<const T*>(a.o[p]) + row * a.dim + col, v);
#pragma unroll
          for (int j = 0; j < N; ++j) acc[j] += w * v[j];
        }
      }
      const Acc inv = Acc(1) / wsum;
#pragma unroll
      for (int j = 0; j < N; ++j) acc[j] *= inv;
    }
    store_vec<T, Acc>(static_cast<T*>(a.out) + row * a.dim + col, acc);
    if (a.lse_out != nullptr && col == 0)
      a.lse_out[row] = (m == -INFINITY) ? -INFINITY : (float)(Acc(m) + acc_log(wsum));
  }
}

// Scalar path for any dim / alignment.
template <typename T, typename Acc>
__global__ void __launch_bounds__(256) merge_lse_scalar_kernel(const __grid_constant__ MergeArgs a) {
  const int64_t total = a.rows * a.dim;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = i / a.dim;
    float m = -INFINITY;
    for (int p = 0; p < a.n_parts; ++p) m = fmaxf(m, a.lse[p][row]);
    Acc acc = 0, wsum = 0;
    if (m != -INFINITY) {
      for (int p = 0; p < a.n_parts; ++p) {
        const Acc w = acc_exp(Acc(a.lse[p][row]) - Acc(m));
        wsum += w;
        acc += w * to_acc<Acc, T>(static_cast<const T*>(a.o[p])[i]);
      }
      acc /= wsum;
    }
    static_cast<T*>(a.out)[i] = from_f64<T>((double)acc);
    if (a.lse_out != nullptr && i - row * a.dim == 0)
      a.lse_out[row] = (m == -INFINITY) ? -INFINITY : (float)(Acc(m) + acc_log(wsum));
  }
}

template <typename T, typename Acc>
static int launch_merge_lse(const MergeArgs& a, cudaStream_t s) {
  constexpr int N = Vec16<T>::N;
  bool vec = (a.dim % N == 0) && (reinterpret_cast<uintptr_t>(a.out) % 16 == 0);
  for (int p = 0; p < a.n_parts; ++p) vec = vec && (reinterpret_cast<uintptr_t>(a.o[p]) % 16 == 0);
  const int threads = 256;
  const int64_t work = vec ? a.rows * (a.dim / N) : a.rows * a.dim;
  const int64_t want = (work + threads - 1) / threads;
  const int64_t cap = (int64_t)num_sms() * 8;  // 8 CTAs of 256 per SM, grid-stride beyond
  const int grid = (int)(want < cap ? (want > 0 ? want : 1) : cap);
  if (vec) {
    switch (a.n_parts) {
      case 2: merge_lse_vec_kernel<T, Acc, 2><<<grid, threads, 0, s>>>(a); break;
      case 4: merge_lse_vec_kernel<T, Acc, 4><<<grid, threads, 0, s>>>(a); break;
      case 8: merge_lse_vec_kernel<T, Acc, 8><<<grid, threads, 0, s>>>(a); break;
      default: merge_lse_vec_kernel<T, Acc, 0><<<grid, threads, 0, s>>>(a); break;
    }
  } else {
    merge_lse_scalar_kernel<T, Acc><<<grid, threads, 0, s>>>(a);
  }
  return check_launch("merge_lse");
}

// ---- pairwise (m, l, o) merge ------------------------------------------------
template <typename T, typename Acc>
__global__ void merge_states_kernel(const T* ma, const T* la, const T* oa, const T* mb, const T* lb,
                                    const T* ob, int64_t R, int64_t D, T* mo, T* lo, T* oo) {
  const int64_t total = R * D;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / D;
    const Acc xa = to_acc<Acc, T>(ma[r]), xb = to_acc<Acc, T>(mb[r]);
    const Acc m = max(xa, xb);
    const Acc ea = acc_exp(xa - m), eb = acc_exp(xb - m);
    oo[i] = from_f64<T>((double)(ea * to_acc<Acc, T>(oa[i]) + eb * to_acc<Acc, T>(ob[i])));
    if (i - r * D == 0) {
      mo[r] = from_f64<T>((double)m);
      lo[r] = from_f64<T>((double)(ea * to_acc<Acc, T>(la[r]) + eb * to_acc<Acc, T>(lb[r])));
    }
  }
}

// ---- (m, l, o) of one row of logits --------------------------------------------
// One CTA per row: max over L, then e_j = exp(x_j - m) for a tile of 256
// logits into shared memory, each thread accumulating its output columns.
template <typename T, typename Acc>
__global__ void __launch_bounds__(256) online_softmax_kernel(const T* logits, const T* values,
                                                             const T* bias, int64_t L, int64_t D,
                                                             int64_t vstride, T* out_m, T* out_l,
                                                             T* out_o) {
  __shared__ Acc tile[256];
  __shared__ Acc red[32];
  const int64_t r = blockIdx.x;
  const T* x = logits + r * L;
  const T* vals = values + r * vstride;
  Acc m = NegInf<Acc>::v();
  for (int64_t j = threadIdx.x; j < L; j += blockDim.x) {
    Acc v = to_acc<Acc, T>(x[j]);
    if (bias) v += to_acc<Acc, T>(bias[j]);
    m = max(m, v);
  }
  m = warp_max(m);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x < 32) {
    Acc v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : NegInf<Acc>::v();
    v = warp_max(v);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  m = red[0];
  __syncthreads();
  Acc lsum = 0;
  Acc acc[4] = {0, 0, 0, 0};  // columns threadIdx.x + 256 * c, D <= 1024
  for (int64_t j0 = 0; j0 < L; j0 += 256) {
    const int64_t j = j0 + threadIdx.x;
    Acc e = 0;
    if (j < L) {
      Acc v = to_acc<Acc, T>(x[j]);
      if (bias) v += to_acc<Acc, T>(bias[j]);
      e = acc_exp(v - m);
    }
    lsum += e;
    tile[threadIdx.x] = e;
    __syncthreads();
    const int64_t jn = (L - j0) < 256 ? (L - j0) : 256;
    for (int64_t jj = 0; jj < jn; ++jj) {
      const Acc e2 = tile[jj];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int64_t col = threadIdx.x + 256 * c;
        if (col < D) acc[c] += e2 * to_acc<Acc, T>(vals[(j0 + jj) * D + col]);
      }
    }
    __syncthreads();
  }
  lsum = warp_sum(lsum);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = lsum;
  __syncthreads();
  if (threadIdx.x == 0) {
    Acc s = 0;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) s += red[w];
    out_m[r] = from_f64<T>((double)m);
    out_l[r] = from_f64<T>((double)s);
  }
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const int64_t col = threadIdx.x + 256 * c;
    if (col < D) out_o[r * D + col] = from_f64<T>((double)acc[c]);
  }
}

}  // namespace dcc

using namespace dcc;

extern "C" int dcc_merge_lse(const void* const* o_parts, const float* const* lse_parts, int n_parts,
                             int64_t R, int64_t D, int dtype, void* out, float* lse_out,
                             void* stream) {
  if (n_parts < 1 || n_parts > kMaxParts)
    return fail(DCC_ERR_INVALID_ARGUMENT, "merge_lse: n_parts must be in [1, 64]");
  if (R < 0 || D <= 0 || out == nullptr || o_parts == nullptr || lse_parts == nullptr)
    return fail(DCC_ERR_INVALID_ARGUMENT, "merge_lse: bad sizes or null pointer");
  if (R == 0) return DCC_OK;
  MergeArgs a{};
  for (int p = 0; p < n_parts; ++p) {
    if (!o_parts[p] || !lse_parts[p]) return fail(DCC_ERR_INVALID_ARGUMENT, "merge_lse: null part");
    a.o[p] = o_parts[p];
    a.lse[p] = lse_parts[p];
  }
  a.n_parts = n_parts;
  a.rows = R;
  a.dim = D;
  a.out = out;
  a.lse_out = lse_out;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case DCC_BF16: return launch_merge_lse<__nv_bfloat16, float>(a, s);
    case DCC_F32: return launch_merge_lse<float, double>(a, s);
    case DCC_F64: return launch_merge_lse<double, double>(a, s);
    default: return fail(DCC_ERR_DTYPE, "merge_lse: unsupported dtype");
  }
}

extern "C" int dcc_merge_softmax_states(const void* m_a, const void* l_a, const void* o_a,
                                        const void* m_b, const void* l_b, const void* o_b, int64_t R,
                                        int64_t D, int dtype, void* out_m, void* out_l, void* out_o,
                                        void* stream) {
  if (R < 0 || D <= 0) return fail(DCC_ERR_INVALID_ARGUMENT, "merge_softmax_states: bad sizes");
  if (R == 0) return DCC_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t total = R * D;
  const int grid = (int)((total + 255) / 256 < 65535 ? (total + 255) / 256 : 65535);
#define DCC_MS(T, A)                                                                             \
  merge_states_kernel<T, A><<<grid, 256, 0, s>>>(                                               \
      (const T*)m_a, (const T*)l_a, (const T*)o_a, (const T*)m_b, (const T*)l_b, (const T*)o_b, \
      R, D, (T*)out_m, (T*)out_l, (T*)out_o)
  switch (dtype) {
    case DCC_BF16: DCC_MS(__nv_bfloat16, float); break;
    case DCC_F32: DCC_MS(float, double); break;
    case DCC_F64: DCC_MS(double, double); break;
    default: return fail(DCC_ERR_DTYPE, "merge_softmax_states: unsupported dtype");
  }
#undef DCC_MS
  return check_launch("merge_softmax_states");
}

extern "C" int dcc_online_softmax_from_attention(const void* logits, const void* values,
                                                 const void* logit_bias, int64_t R, int64_t L,
                                                 int64_t D, int64_t values_row_stride, int dtype,
                                                 void* out_m, void* out_l, void* out_o,
                                                 void* stream) {
  if (R < 0 || L <= 0 || D <= 0 || D > 1024)
    return fail(DCC_ERR_INVALID_ARGUMENT, "online_softmax_from_attention: need L > 0 and 0 < D <= 1024");
  if (R == 0) return DCC_OK;
  if (R > 2147483647) return fail(DCC_ERR_UNSUPPORTED, "online_softmax_from_attention: too many rows");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
#define DCC_OS(T, A)                                                                         \
  online_softmax_kernel<T, A><<<(unsigned)R, 256, 0, s>>>((const T*)logits, (const T*)values, \
                                                          (const T*)logit_bias, L, D,         \
                                                          values_row_stride, (T*)out_m,       \
                                                          (T*)out_l, (T*)out_o)
  switch (dtype) {
    case DCC_BF16: DCC_OS(__nv_bfloat16, float); break;
    case DCC_F32: DCC_OS(float, double); break;
    case DCC_F64: DCC_OS(double, double); break;
    default: return fail(DCC_ERR_DTYPE, "online_softmax_from_attention: unsupported dtype");
  }
#undef DCC_OS
  return check_launch("online_softmax_from_attention");
}
