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

// ---- register-resident factor and solves for n <= 64 (the build's hot path) ----

__device__ __forceinline__ void bar_sync_64() { asm volatile("bar.sync 2, 64;\n" ::: "memory"); }

// Cholesky of the leading n x n block (n <= 64) of the SPD matrix A (lower
// triangle), in place: A = L L^T, zeros written above the diagonal of the
// n x n block, 1 / L_ii to inv_diag[i].  The block's first 64 threads each
// hold one row in registers as a window that shifts left by one column per
// step (r[m] = A_i,k+m at step k), so every register index is static while
// the step loop stays rolled (straight-line code of this size would be
// instruction-fetch-bound: it runs once per CTA).  Step k: one 64-thread
// barrier, then L_ik = A_ik / sqrt(A_kk) and A_ij -= A_ik A_jk / A_kk for
// k < j <= i, with 1 / sqrt(A_kk) and 1 / A_kk read from shared memory.
// The step is pipelined: each row first updates the entry that becomes
// column k + 1 and publishes it (colbuf, two alternating [66] buffers), and
// the next pivot row computes the next step's two reciprocals right there,
// so neither a division nor a square root sits between two barriers; the
// other 62 updates of the row follow.  Every thread of the block calls
// chol64 (it ends with __syncthreads()).  colbuf: 132 doubles.
__device__ __forceinline__ void chol64_rows(double* A, int lda, int n, double* inv_diag, double* colbuf);
__device__ __forceinline__ void chol64(double* A, int lda, int n, double* inv_diag, double* colbuf) {
  if (threadIdx.x < 64) chol64_rows(A, lda, n, inv_diag, colbuf);
  __syncthreads();
}

// The factorisation itself, run by threads 0-63 only (64-thread named
// barrier): the other threads of the block may do independent work
// meanwhile; the caller synchronises the block afterwards.
__device__ __forceinline__ void chol64_rows(double* A, int lda, int n, double* inv_diag, double* colbuf) {
  const int i = threadIdx.x;
  {
    double r[64];
#pragma unroll
    for (int m = 0; m < 64; ++m) r[m] = (i < n && m <= i) ? A[i * lda + m] : 0.0;
    colbuf[i] = r[0];
    if (i == 0) {
      colbuf[64] = 1.0 / sqrt(r[0]);
      colbuf[65] = 1.0 / r[0];
    }
    for (int k = 0; k < n; ++k) {
      const double* col = colbuf + (k & 1) * 66;
      double* nxt = colbuf + ((k + 1) & 1) * 66;
      bar_sync_64();
      const double isd = col[64], id = col[65];
      const bool below = i > k && i < n;
      if (i == k) {
        A[i * lda + k] = sqrt(r[0]);
        inv_diag[k] = isd;
      } else if (below) {
        A[i * lda + k] = r[0] * isd;
      }
      const double t = below ? r[0] * id : 0.0;
      const int span = below ? i - k : 0;  // columns k+1 .. i are updated
      // the entry that becomes column k + 1, published for the next step
      const double u1 = fma(-t, col[min(k + 1, 63)], r[1]);
      const double n0 = 1 <= span ? u1 : r[1];
      nxt[i] = n0;
      if (i == k + 1 && i < n) {
        nxt[64] = 1.0 / sqrt(n0);
        nxt[65] = 1.0 / n0;
      }
      // branch-free: every lane loads (clamped index, a broadcast) and
      // computes; the select keeps rows that are not updated unchanged
#pragma unroll
      for (int m = 2; m < 64; ++m) {
        const double cj = col[min(k + m, 63)];
        const double u = fma(-t, cj, r[m]);
        r[m - 1] = m <= span ? u : r[m];
      }
      r[0] = n0;
      r[63] = 0.0;
    }
    if (i < n)
      for (int j = i + 1; j < n; ++j) A[i * lda + j] = 0.0;
  }
}

// Solve (L L^T) X = B in place for ncols <= 128 right-hand sides, L from
// chol64 (any n <= 64): column c of B at X[i * ldx + c], rows i < n.
// Blocked over 8-row panels with every thread of the block: per panel, the
// 8 x 8 triangle is solved by one thread per column, then the rows below
// (forward) or above (backward) are updated by a rank-8 product spread over
// all threads, so only 2 x ceil(n / 8) short serial steps remain.
__device__ __forceinline__ void chol64_solve(const double* L, int lda, const double* inv_diag, int n, double* X,
                                             int ldx, int ncols) {
  constexpr int kP = 8;
  const int nt = blockDim.x;
  // forward: L Y = B
  for (int r0 = 0; r0 < n; r0 += kP) {
    const int r1 = min(r0 + kP, n);
    for (int c = threadIdx.x; c < ncols; c += nt) {
      double y[kP];
#pragma unroll
      for (int q = 0; q < kP; ++q) {
        const int i = r0 + q;
        if (i < r1) {
          double s = X[i * ldx + c];
#pragma unroll
          for (int j = 0; j < q; ++j) s = fma(-L[i * lda + r0 + j], y[j], s);
          y[q] = s * inv_diag[i];
          X[i * ldx + c] = y[q];
        }
      }
    }
    __syncthreads();
    const int rows = n - r1;
    for (int e = threadIdx.x; e < rows * ncols; e += nt) {
      const int i = r1 + e / ncols, c = e % ncols;
      double s = X[i * ldx + c];
#pragma unroll
      for (int j = 0; j < kP; ++j)
        if (r0 + j < r1) s = fma(-L[i * lda + r0 + j], X[(r0 + j) * ldx + c], s);
      X[i * ldx + c] = s;
    }
    __syncthreads();
  }
  // backward: L^T X = Y
  for (int r1 = n; r1 > 0; r1 -= kP) {
    const int r0 = max(r1 - kP, 0);
    for (int c = threadIdx.x; c < ncols; c += nt) {
      double x[kP];
#pragma unroll
      for (int q = kP - 1; q >= 0; --q) {
        const int i = r0 + q;
        if (i < r1) {
          double s = X[i * ldx + c];
#pragma unroll
          for (int j = q + 1; j < kP; ++j)
            if (r0 + j < r1) s = fma(-L[(r0 + j) * lda + i], x[j], s);
          x[q] = s * inv_diag[i];
          X[i * ldx + c] = x[q];
        }
      }
    }
    __syncthreads();
    for (int e = threadIdx.x; e < r0 * ncols; e += nt) {
      const int i = e / ncols, c = e % ncols;
      double s = X[i * ldx + c];
#pragma unroll
      for (int j = 0; j < kP; ++j)
        if (r0 + j < r1) s = fma(-L[(r0 + j) * lda + i], X[(r0 + j) * ldx + c], s);
      X[i * ldx + c] = s;
    }
    __syncthreads();
  }
}

// Solve (L L^T) v = v in place for one right-hand side v[n] in shared
// memory, L from chol64 (n <= 64).  One warp: lane l holds rows l and
// l + 32; each column step broadcasts the solved entry by shuffle.  Called
// by the 32 threads of one warp only.
__device__ __forceinline__ void chol64_solve_vec(const double* L, int lda, const double* inv_diag, int n,
                                                 double* v) {
  const int l = threadIdx.x & 31;
  double x0 = l < n ? v[l] : 0.0, x1 = l + 32 < n ? v[l + 32] : 0.0;
  // branch-free column steps: loads use clamped indices, selects apply them
  const int r0 = min(l, n - 1), r1 = min(l + 32, n - 1);
  for (int i = 0; i < n; ++i) {  // forward: L y = v, column by column
    const double xi = __shfl_sync(0xffffffffu, i < 32 ? x0 : x1, i & 31) * inv_diag[i];
    const double u0 = fma(-L[r0 * lda + i], xi, x0), u1 = fma(-L[r1 * lda + i], xi, x1);
    x0 = l == i ? xi : (l > i && l < n ? u0 : x0);
    x1 = l + 32 == i ? xi : (l + 32 > i && l + 32 < n ? u1 : x1);
  }
  for (int i = n - 1; i >= 0; --i) {  // backward: L^T x = y
    const double xi = __shfl_sync(0xffffffffu, i < 32 ? x0 : x1, i & 31) * inv_diag[i];
    const double u0 = fma(-L[i * lda + r0], xi, x0), u1 = fma(-L[i * lda + r1], xi, x1);
    x0 = l == i ? xi : (l < i ? u0 : x0);
    x1 = l + 32 == i ? xi : (l + 32 < i ? u1 : x1);
  }
  if (l < n) v[l] = x0;
  if (l + 32 < n) v[l + 32] = x1;
  __syncwarp();
}

}  // namespace dcc
