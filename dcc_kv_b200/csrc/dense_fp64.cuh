// Small dense FP64 linear algebra in shared memory, one CTA (block-wide
// __syncthreads inside): Cholesky, triangular solves, Gram products.
#pragma once

#include "build_common.cuh"

namespace dcc {

constexpr int kLdG = kMaxRepr + 1;  // [64][65] shared matrices

// Side vectors (block mass, logit bias) are double for FP64 inputs and float
// for FP32 / bf16 inputs.
template <typename TIn>
__device__ __forceinline__ double load_side(const void* p, int i) {
  if (sizeof(TIn) == 8) return static_cast<const double*>(p)[i];
  return (double)static_cast<const float*>(p)[i];
}

// In-place Cholesky of the leading n x n block of A (lower triangle).
__device__ __forceinline__ void chol_inplace(double* A, int lda, int n) {
  for (int k = 0; k < n; ++k) {
    if (threadIdx.x == 0) A[k * lda + k] = sqrt(A[k * lda + k]);
    __syncthreads();
    const double piv = A[k * lda + k];
    for (int i = k + 1 + threadIdx.x; i < n; i += blockDim.x) A[i * lda + k] /= piv;
    __syncthreads();
    const int m = n - k - 1;
    for (int e = threadIdx.x; e < m * m; e += blockDim.x) {
      const int i = k + 1 + e / m, j = k + 1 + e % m;
      if (j <= i) A[i * lda + j] -= A[i * lda + k] * A[j * lda + k];
    }
    __syncthreads();
  }
}

// Solve (L L^T) x = rhs in place for `ncols` right-hand-side columns stored
// column c at X[i * ldx + c]; one thread per column.
__device__ __forceinline__ void chol_solve_cols(const double* L, int lda, int n, double* X, int ldx, int ncols) {
  for (int c = threadIdx.x; c < ncols; c += blockDim.x) {
    for (int i = 0; i < n; ++i) {
      double s = X[i * ldx + c];
      for (int j = 0; j < i; ++j) s -= L[i * lda + j] * X[j * ldx + c];
      X[i * ldx + c] = s / L[i * lda + i];
    }
    for (int i = n - 1; i >= 0; --i) {
      double s = X[i * ldx + c];
      for (int j = i + 1; j < n; ++j) s -= L[j * lda + i] * X[j * ldx + c];
      X[i * ldx + c] = s / L[i * lda + i];
    }
  }
  __syncthreads();
}

// gram[a][a2] = sum_b Z[a][b] Z[a2][b] (+ lam on the diagonal), Z [M, Bp] in
// global memory, streamed through a [64][33] shared tile.
__device__ __forceinline__ void gram_rows(const double* Z, int M, int Bp, double lam, double* gram, double* tile) {
  const int a = threadIdx.x & 63, g = threadIdx.x >> 6;  // 4 groups of 16 columns a2
  double acc[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) acc[i] = 0.0;
  for (int b0 = 0; b0 < Bp; b0 += 32) {
    __syncthreads();
    for (int e = threadIdx.x; e < 64 * 32; e += blockDim.x) {
      const int r = e >> 5, c = e & 31;
      tile[r * 33 + c] = (r < M && b0 + c < Bp) ? Z[(int64_t)r * Bp + b0 + c] : 0.0;
    }
    __syncthreads();
    const int jn = min(32, Bp - b0);
    for (int j = 0; j < jn; ++j) {
      const double za = tile[a * 33 + j];
#pragma unroll
      for (int i = 0; i < 16; ++i) acc[i] = fma(za, tile[(g * 16 + i) * 33 + j], acc[i]);
    }
  }
  __syncthreads();
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const int a2 = g * 16 + i;
    if (a < M && a2 < M) gram[a * kLdG + a2] = acc[i] + (a == a2 ? lam : 0.0);
  }
  __syncthreads();
}

// gram[b][b2] = sum_a Z[a][b] Z[a][b2] (+ lam), Z [M, Bp] fully in shared
// memory (Bp <= M <= 64).
__device__ __forceinline__ void gram_cols(const double* Zs, int M, int Bp, double lam, double* gram) {
  for (int e = threadIdx.x; e < Bp * Bp; e += blockDim.x) {
    const int b = e / Bp, b2 = e % Bp;
    double s = 0.0;
    for (int a = 0; a < M; ++a) s = fma(Zs[a * kLdG + b], Zs[a * kLdG + b2], s);
    gram[b * kLdG + b2] = s + (b == b2 ? lam : 0.0);
  }
  __syncthreads();
}


// Solve (L L^T) X = B in place, B [n, ncols] at X[i * ldx + c], right-looking:
// each of the 2n steps updates all remaining rows and columns in parallel.
__device__ __forceinline__ void chol_solve_parallel(const double* L, int lda, int n, double* X, int ldx,
                                                    int ncols) {
  for (int i = 0; i < n; ++i) {
    const double inv = 1.0 / L[i * lda + i];
    for (int c = threadIdx.x; c < ncols; c += blockDim.x) X[i * ldx + c] *= inv;
    __syncthreads();
    const int rest = (n - i - 1) * ncols;
    for (int e = threadIdx.x; e < rest; e += blockDim.x) {
      const int k = i + 1 + e / ncols, c = e % ncols;
      X[k * ldx + c] -= L[k * lda + i] * X[i * ldx + c];
    }
    __syncthreads();
  }
  for (int i = n - 1; i >= 0; --i) {
    const double inv = 1.0 / L[i * lda + i];
    for (int c = threadIdx.x; c < ncols; c += blockDim.x) X[i * ldx + c] *= inv;
    __syncthreads();
    const int rest = i * ncols;
    for (int e = threadIdx.x; e < rest; e += blockDim.x) {
      const int k = e / ncols, c = e % ncols;
      X[k * ldx + c] -= L[i * lda + k] * X[i * ldx + c];
    }
    __syncthreads();
  }
}

}  // namespace dcc
