// Small dense FP64 solvers shared by the calibration kernels (calib.cu) and
// the standalone nonneg_least_squares / ridge_regression_value entry points.
//
// beta (calibration.py:63-94): G = exp(Q^ C_K^T * scale) [M, B];
//   B > M : w = clamp(G^T (G G^T + lam I)^-1 t, 0)      -- push-through of the
//           reference's B x B ridge solve clamp(solve(G^T G + lam I, G^T t), 0)
//           (:44-47): the same vector in exact arithmetic, an M x M system;
//   B <= M: the literal B x B solve, then 100 projected-gradient steps,
//           lr 1e-2, ridge toward 1 (:54-60);
//   beta = log(max(w, 1e-6)).
// values (value_regression.py:38-78): X = softmax(Q^ C_K^T * scale + beta/M),
//   B > M : C_V = X^T (X X^T + lam I)^-1 Y ; B <= M : (X^T X + lam I)^-1 X^T Y.
// Symmetric positive definite systems (lam > 0) are solved by Cholesky in
// shared memory.
#include "dense_fp64.cuh"

namespace dcc {

// ---- standalone NNLS and ridge (per-function API) ----------------------------
// Both run on one CTA: they are the reference's small dense solves on their own.
struct SolveArgs {
  const void* A;   // G [M, B] or X [M, B]
  const void* Y;   // target [M] or Y [M, D]
  int64_t M, B, D;
  double lam;
  int n_iter;
  void* out;
  double* Zd;      // workspace [M, B] double copy
  double* Yd;      // workspace [M, D] double
};

template <typename T>
__global__ void __launch_bounds__(256) nnls_kernel(const SolveArgs s) {
  extern __shared__ double sm[];
  double* gram = sm;                     // [64][65]
  double* gs = gram + kMaxRepr * kLdG;   // [64][65]
  double* tile = gs + kMaxRepr * kLdG;   // [64][33]
  double* tv = tile + kMaxRepr * 33;
  double* vv = tv + kMaxRepr;
  double* res = vv + kMaxRepr;
  const int M = (int)s.M, Bp = (int)s.B;
  for (int64_t e = threadIdx.x; e < s.M * s.B; e += blockDim.x) s.Zd[e] = to_f64<T>(static_cast<const T*>(s.A)[e]);
  if (threadIdx.x < M) tv[threadIdx.x] = to_f64<T>(static_cast<const T*>(s.Y)[threadIdx.x]);
  __syncthreads();
  double* wout = s.Yd;  // [B] scratch
  if (M < Bp) {
    gram_rows(s.Zd, M, Bp, s.lam, gram, tile);
    chol_inplace(gram, kLdG, M);
    if (threadIdx.x < kMaxRepr) vv[threadIdx.x] = threadIdx.x < M ? tv[threadIdx.x] : 0.0;
    __syncthreads();
    chol_solve_cols(gram, kLdG, M, vv, 1, 1);
    for (int bb = threadIdx.x; bb < Bp; bb += blockDim.x) {
      double w = 0.0;
      for (int a = 0; a < M; ++a) w = fma(s.Zd[(int64_t)a * Bp + bb], vv[a], w);
      wout[bb] = w > 0.0 ? w : 0.0;
    }
  } else {
    for (int e = threadIdx.x; e < M * Bp; e += blockDim.x) gs[(e / Bp) * kLdG + e % Bp] = s.Zd[e];
    __syncthreads();
    gram_cols(gs, M, Bp, s.lam, gram);
    for (int bb = threadIdx.x; bb < Bp; bb += blockDim.x) {
      double acc = 0.0;
      for (int a = 0; a < M; ++a) acc = fma(gs[a * kLdG + bb], tv[a], acc);
      vv[bb] = acc;
    }
    __syncthreads();
    chol_inplace(gram, kLdG, Bp);
    chol_solve_cols(gram, kLdG, Bp, vv, 1, 1);
    if (threadIdx.x < Bp) vv[threadIdx.x] = fmax(vv[threadIdx.x], 0.0);
    __syncthreads();
    for (int it = 0; it < s.n_iter; ++it) {
      if (threadIdx.x < M) {
        double acc = 0.0;
        for (int bb = 0; bb < Bp; ++bb) acc = fma(gs[threadIdx.x * kLdG + bb], vv[bb], acc);
        res[threadIdx.x] = acc - tv[threadIdx.x];
      }
      __syncthreads();
      if (threadIdx.x < Bp) {
        double g = 0.0;
        for (int a = 0; a < M; ++a) g = fma(gs[a * kLdG + threadIdx.x], res[a], g);
        g += s.lam * (vv[threadIdx.x] - 1.0);
        vv[threadIdx.x] = fmax(vv[threadIdx.x] - 1e-2 * g, 0.0);
      }
      __syncthreads();
    }
    if (threadIdx.x < Bp) wout[threadIdx.x] = vv[threadIdx.x];
  }
  __syncthreads();
  for (int bb = threadIdx.x; bb < Bp; bb += blockDim.x) static_cast<T*>(s.out)[bb] = from_f64<T>(wout[bb]);
}

template <typename T>
__global__ void __launch_bounds__(256) ridge_kernel(const SolveArgs s) {
  extern __shared__ double sm[];
  double* gram = sm;                     // [64][65]
  double* gs = gram + kMaxRepr * kLdG;   // [64][65]
  double* tile = gs + kMaxRepr * kLdG;   // [64][33]
  double* ws = tile + kMaxRepr * 33;     // [64][D+1]
  const int M = (int)s.M, Bp = (int)s.B, D = (int)s.D, ldw = D + 1;
  for (int64_t e = threadIdx.x; e < s.M * s.B; e += blockDim.x) s.Zd[e] = to_f64<T>(static_cast<const T*>(s.A)[e]);
  for (int64_t e = threadIdx.x; e < s.M * s.D; e += blockDim.x) s.Yd[e] = to_f64<T>(static_cast<const T*>(s.Y)[e]);
  __syncthreads();
  T* out = static_cast<T*>(s.out);
  if (M < Bp) {
    gram_rows(s.Zd, M, Bp, s.lam, gram, tile);
    chol_inplace(gram, kLdG, M);
    for (int e = threadIdx.x; e < M * D; e += blockDim.x) ws[(e / D) * ldw + e % D] = s.Yd[e];
    __syncthreads();
    chol_solve_cols(gram, kLdG, M, ws, ldw, D);
    for (int64_t e = threadIdx.x; e < (int64_t)Bp * D; e += blockDim.x) {
      const int bb = (int)(e / D), c = (int)(e % D);
      double acc = 0.0;
      for (int a = 0; a < M; ++a) acc = fma(s.Zd[(int64_t)a * Bp + bb], ws[a * ldw + c], acc);
      out[e] = from_f64<T>(acc);
    }
  } else {
    for (int e = threadIdx.x; e < M * Bp; e += blockDim.x) gs[(e / Bp) * kLdG + e % Bp] = s.Zd[e];
    __syncthreads();
    gram_cols(gs, M, Bp, s.lam, gram);
    for (int e = threadIdx.x; e < Bp * D; e += blockDim.x) {
      const int bb = e / D, c = e % D;
      double acc = 0.0;
      for (int a = 0; a < M; ++a) acc = fma(gs[a * kLdG + bb], s.Yd[(int64_t)a * D + c], acc);
      ws[bb * ldw + c] = acc;
    }
    __syncthreads();
    chol_inplace(gram, kLdG, Bp);
    chol_solve_cols(gram, kLdG, Bp, ws, ldw, D);
    for (int e = threadIdx.x; e < Bp * D; e += blockDim.x) out[e] = from_f64<T>(ws[(e / D) * ldw + e % D]);
  }
}

}  // namespace dcc

using namespace dcc;

extern "C" size_t dcc_nnls_workspace_bytes(int64_t M, int64_t B) {
  return align_up((size_t)(M * B) * 8, 256) + align_up((size_t)(B > 64 ? B : 64) * 8, 256) + 256;
}

extern "C" size_t dcc_ridge_workspace_bytes(int64_t M, int64_t B, int64_t D) {
  return align_up((size_t)(M * B) * 8, 256) + align_up((size_t)(M * D) * 8, 256) + 256;
}

static int solve_checks(int64_t M, int64_t B, const char* who) {
  if (M <= 0 || B <= 0) return fail(DCC_ERR_INVALID_ARGUMENT, std::string(who) + ": empty system");
  if (M > kMaxRepr) return fail(DCC_ERR_UNSUPPORTED, std::string(who) + ": more than 64 rows");
  if (M >= B && B > kMaxRepr) return fail(DCC_ERR_UNSUPPORTED, std::string(who) + ": bad size");
  return DCC_OK;
}

extern "C" int dcc_nonneg_least_squares(const void* G, const void* target, int64_t M, int64_t B,
                                        double lambda_reg, int n_iter, int dtype, void* out_w,
                                        void* workspace, size_t workspace_bytes, void* stream) {
  DCC_CHECK(solve_checks(M, B, "nonneg_least_squares"));
  if (workspace_bytes < dcc_nnls_workspace_bytes(M, B) || !workspace)
    return fail(DCC_ERR_WORKSPACE, "nonneg_least_squares: workspace too small");
  Workspace ws(workspace, workspace_bytes);
  SolveArgs s{G, target, M, B, 1, lambda_reg, n_iter, out_w, nullptr, nullptr};
  s.Zd = ws.take<double>((size_t)(M * B));
  s.Yd = ws.take<double>((size_t)(B > 64 ? B : 64));
  const size_t smem = (2 * (size_t)kMaxRepr * kLdG + (size_t)kMaxRepr * 33 + 3 * kMaxRepr) * 8;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
#define DCC_NN(T)                                                                                  \
  do {                                                                                             \
    DCC_CHECK(check_cuda(cudaFuncSetAttribute(nnls_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem), "nnls smem")); \
    nnls_kernel<T><<<1, 256, smem, st>>>(s);                                                       \
  } while (0)
  switch (dtype) {
    case DCC_F32: DCC_NN(float); break;
    case DCC_F64: DCC_NN(double); break;
    case DCC_BF16: DCC_NN(__nv_bfloat16); break;
    default: return fail(DCC_ERR_DTYPE, "nonneg_least_squares: unsupported dtype");
  }
#undef DCC_NN
  return check_launch("nonneg_least_squares");
}

extern "C" int dcc_ridge_regression_value(const void* X, const void* Y, int64_t M, int64_t B, int64_t D,
                                          double lambda_reg, int dtype, void* out, void* workspace,
                                          size_t workspace_bytes, void* stream) {
  DCC_CHECK(solve_checks(M, B, "ridge_regression_value"));
  if (D <= 0 || D > kMaxDim) return fail(DCC_ERR_UNSUPPORTED, "ridge_regression_value: need 0 < D <= 128");
  if (workspace_bytes < dcc_ridge_workspace_bytes(M, B, D) || !workspace)
    return fail(DCC_ERR_WORKSPACE, "ridge_regression_value: workspace too small");
  Workspace ws(workspace, workspace_bytes);
  SolveArgs s{X, Y, M, B, D, lambda_reg, 0, out, nullptr, nullptr};
  s.Zd = ws.take<double>((size_t)(M * B));
  s.Yd = ws.take<double>((size_t)(M * D));
  const size_t smem = (2 * (size_t)kMaxRepr * kLdG + (size_t)kMaxRepr * 33 + (size_t)kMaxRepr * (D + 1)) * 8;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
#define DCC_RR(T)                                                                                  \
  do {                                                                                             \
    DCC_CHECK(check_cuda(cudaFuncSetAttribute(ridge_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem), "ridge smem")); \
    ridge_kernel<T><<<1, 256, smem, st>>>(s);                                                      \
  } while (0)
  switch (dtype) {
    case DCC_F32: DCC_RR(float); break;
    case DCC_F64: DCC_RR(double); break;
    case DCC_BF16: DCC_RR(__nv_bfloat16); break;
    default: return fail(DCC_ERR_DTYPE, "ridge_regression_value: unsupported dtype");
  }
#undef DCC_RR
  return check_launch("ridge_regression_value");
}
