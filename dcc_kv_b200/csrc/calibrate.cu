// Logit-bias calibration and compact-value regression, FP64, one CTA per
// problem.
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
__device__ void chol_inplace(double* A, int lda, int n) {
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
__device__ void chol_solve_cols(const double* L, int lda, int n, double* X, int ldx, int ncols) {
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
__device__ void gram_rows(const double* Z, int M, int Bp, double lam, double* gram, double* tile) {
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
__device__ void gram_cols(const double* Zs, int M, int Bp, double lam, double* gram) {
  for (int e = threadIdx.x; e < Bp * Bp; e += blockDim.x) {
    const int b = e / Bp, b2 = e % Bp;
    double s = 0.0;
    for (int a = 0; a < M; ++a) s = fma(Zs[a * kLdG + b], Zs[a * kLdG + b2], s);
    gram[b * kLdG + b2] = s + (b == b2 ? lam : 0.0);
  }
  __syncthreads();
}

template <typename TIn, typename Acc>
__global__ void __launch_bounds__(256) calibrate_kernel(const __grid_constant__ BuildBatch<Acc> b,
                                                        const BuildParams prm) {
  const BuildDesc<Acc>& p = b.p[blockIdx.x];
  const int M = p.M, d = prm.d, dv = prm.dv;
  const int Bp = (int)((int64_t)p.budget < p.L_s ? (int64_t)p.budget : p.L_s);
  extern __shared__ double sm[];
  const int ldq = kMaxDim + 1;
  double* qs = sm;                        // [64][129]  Q^, later W / R
  double* ks = qs + kMaxRepr * ldq;       // [32][129]  C_K tile
  double* gram = ks + 32 * ldq;           // [64][65]
  double* gs = gram + kMaxRepr * kLdG;    // [64][65]   G or X when Bp <= 64
  double* tile = gs + kMaxRepr * kLdG;    // [64][33]
  double* tv = tile + kMaxRepr * 33;      // [64] mass target
  double* vv = tv + kMaxRepr;             // [64] solution vector
  double* res = vv + kMaxRepr;            // [64] residual

  // (1) block mass and Y from the chunk partials, fixed chunk order
  for (int a = threadIdx.x; a < kMaxRepr; a += blockDim.x) {
    double s = 0.0;
    if (a < M) {
      if (p.in_mass)
        s = load_side<TIn>(p.in_mass, a);
      else
        for (int c = 0; c < p.n_chunks; ++c) s += (double)p.massp[(int64_t)c * M + a];
    }
    tv[a] = s;
    if (a < M && p.out_mass) p.out_mass[a] = s;
  }
  if (p.stages & kStageValues) {
    for (int e = threadIdx.x; e < M * dv; e += blockDim.x) {
      double s = 0.0;
      for (int c = 0; c < p.n_chunks; ++c) s += (double)p.yp[(int64_t)c * M * dv + e];
      p.Y[e] = s;
    }
  }
  // (2) logits Q^ C_K^T * scale -> X (kept), G = exp(logits)
  const TIn* rq = static_cast<const TIn*>(p.repr);
  const TIn* ck = static_cast<const TIn*>(p.out_keys);
  for (int e = threadIdx.x; e < kMaxRepr * d; e += blockDim.x) {
    const int r = e / d, c = e - r * d;
    qs[r * ldq + c] = r < M ? to_f64<TIn>(rq[r * d + c]) : 0.0;
  }
  const int ty = threadIdx.x >> 4, tx = threadIdx.x & 15;
  for (int b0 = 0; b0 < Bp; b0 += 32) {
    __syncthreads();
    for (int e = threadIdx.x; e < 32 * d; e += blockDim.x) {
      const int r = e / d, c = e - r * d;
      ks[r * ldq + c] = b0 + r < Bp ? to_f64<TIn>(ck[(int64_t)(b0 + r) * d + c]) : 0.0;
    }
    __syncthreads();
    double s[4][2] = {{0, 0}, {0, 0}, {0, 0}, {0, 0}};
    for (int c = 0; c < d; ++c) {
      const double k0 = ks[tx * ldq + c], k1 = ks[(tx + 16) * ldq + c];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const double q = qs[(ty + 16 * i) * ldq + c];
        s[i][0] = fma(q, k0, s[i][0]);
        s[i][1] = fma(q, k1, s[i][1]);
      }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int a = ty + 16 * i;
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int bb = b0 + tx + 16 * j;
        if (a < M && bb < Bp) {
          const double lg = s[i][j] * prm.scale;
          p.X[(int64_t)a * Bp + bb] = lg;
          p.G[(int64_t)a * Bp + bb] = exp(lg);
        }
      }
    }
  }
  __syncthreads();

  // (3) NNLS for w, then beta (or the caller's beta)
  const double lb = prm.lambda_beta;
  if (!(p.stages & kStageBeta)) {
    for (int bb = threadIdx.x; bb < Bp; bb += blockDim.x)
      p.wv[bb] = load_side<TIn>(p.in_beta, bb);
    __syncthreads();
  } else if (M < Bp) {
    gram_rows(p.G, M, Bp, lb, gram, tile);
    chol_inplace(gram, kLdG, M);
    if (threadIdx.x < kMaxRepr) vv[threadIdx.x] = tv[threadIdx.x];
    __syncthreads();
    chol_solve_cols(gram, kLdG, M, vv, 1, 1);
    for (int bb = threadIdx.x; bb < Bp; bb += blockDim.x) {
      double w = 0.0;
      for (int a = 0; a < M; ++a) w = fma(p.G[(int64_t)a * Bp + bb], vv[a], w);
      p.wv[bb] = w > 0.0 ? w : 0.0;
    }
    __syncthreads();
  } else {
    for (int e = threadIdx.x; e < M * Bp; e += blockDim.x) {
      const int a = e / Bp, bb = e % Bp;
      gs[a * kLdG + bb] = p.G[e];
    }
    __syncthreads();
    gram_cols(gs, M, Bp, lb, gram);
    for (int bb = threadIdx.x; bb < Bp; bb += blockDim.x) {
      double s = 0.0;
      for (int a = 0; a < M; ++a) s = fma(gs[a * kLdG + bb], tv[a], s);
      vv[bb] = s;
    }
    __syncthreads();
    chol_inplace(gram, kLdG, Bp);
    chol_solve_cols(gram, kLdG, Bp, vv, 1, 1);
    if (threadIdx.x < Bp) vv[threadIdx.x] = vv[threadIdx.x] > 0.0 ? vv[threadIdx.x] : 0.0;
    __syncthreads();
    for (int it = 0; it < 100; ++it) {
      if (threadIdx.x < M) {  // res = G w - t
        const int a = threadIdx.x;
        double s = 0.0;
        for (int bb = 0; bb < Bp; ++bb) s = fma(gs[a * kLdG + bb], vv[bb], s);
        res[a] = s - tv[a];
      }
      __syncthreads();
      if (threadIdx.x < Bp) {  // w = max(w - lr (G^T res + lam (w - 1)), 0)
        const int bb = threadIdx.x;
        double g = 0.0;
        for (int a = 0; a < M; ++a) g = fma(gs[a * kLdG + bb], res[a], g);
        g += lb * (vv[bb] - 1.0);
        const double w = vv[bb] - 1e-2 * g;
        vv[bb] = w > 0.0 ? w : 0.0;
      }
      __syncthreads();
    }
    if (threadIdx.x < Bp) p.wv[threadIdx.x] = vv[threadIdx.x];
    __syncthreads();
  }
  for (int bb = threadIdx.x; bb < Bp && (p.stages & kStageBeta); bb += blockDim.x) {
    const double beta = log(fmax(p.wv[bb], 1e-6));
    p.wv[bb] = beta;
    if (sizeof(TIn) == 8)
      static_cast<double*>(p.out_bias)[bb] = beta;
    else
      static_cast<float*>(p.out_bias)[bb] = (float)beta;
  }
  __syncthreads();

  if (!(p.stages & kStageValues)) return;
  // (4) X = softmax_b(logits + beta / M), one warp per row
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int a = warp; a < M; a += blockDim.x >> 5) {
    double* xr = p.X + (int64_t)a * Bp;
    double mx = -INFINITY;
    for (int bb = lane; bb < Bp; bb += 32) {
      const double v = xr[bb] + p.wv[bb] / (double)M;
      xr[bb] = v;
      mx = fmax(mx, v);
    }
    mx = warp_max(mx);
    double sum = 0.0;
    for (int bb = lane; bb < Bp; bb += 32) {
      const double e = exp(xr[bb] - mx);
      xr[bb] = e;
      sum += e;
    }
    sum = warp_sum(sum);
    for (int bb = lane; bb < Bp; bb += 32) xr[bb] = xr[bb] / sum;
  }
  __syncthreads();

  // (5) compact values
  const double lv = prm.lambda_value;
  const int ldw = kMaxDim + 1;
  TIn* outv = static_cast<TIn*>(p.out_values);
  if (M < Bp) {
    gram_rows(p.X, M, Bp, lv, gram, tile);
    chol_inplace(gram, kLdG, M);
    for (int e = threadIdx.x; e < M * dv; e += blockDim.x) {
      const int a = e / dv, c = e - a * dv;
      qs[a * ldw + c] = p.Y[e];
    }
    __syncthreads();
    chol_solve_cols(gram, kLdG, M, qs, ldw, dv);  // W = (X X^T + lam I)^-1 Y
    // C_V = X^T W, streamed over column tiles of X
    for (int b0 = 0; b0 < Bp; b0 += 32) {
      __syncthreads();
      for (int e = threadIdx.x; e < 64 * 32; e += blockDim.x) {
        const int r = e >> 5, c = e & 31;
        tile[r * 33 + c] = (r < M && b0 + c < Bp) ? p.X[(int64_t)r * Bp + b0 + c] : 0.0;
      }
      __syncthreads();
      for (int e = threadIdx.x; e < 32 * dv; e += blockDim.x) {
        const int j = e / dv, c = e - j * dv;
        if (b0 + j >= Bp) continue;
        double s = 0.0;
        for (int a = 0; a < M; ++a) s = fma(tile[a * 33 + j], qs[a * ldw + c], s);
        outv[(int64_t)(b0 + j) * dv + c] = from_f64<TIn>(s);
      }
    }
  } else {
    for (int e = threadIdx.x; e < M * Bp; e += blockDim.x) {
      const int a = e / Bp, bb = e % Bp;
      gs[a * kLdG + bb] = p.X[e];
    }
    __syncthreads();
    gram_cols(gs, M, Bp, lv, gram);
    for (int e = threadIdx.x; e < Bp * dv; e += blockDim.x) {  // R = X^T Y
      const int bb = e / dv, c = e - bb * dv;
      double s = 0.0;
      for (int a = 0; a < M; ++a) s = fma(gs[a * kLdG + bb], p.Y[(int64_t)a * dv + c], s);
      qs[bb * ldw + c] = s;
    }
    __syncthreads();
    chol_inplace(gram, kLdG, Bp);
    chol_solve_cols(gram, kLdG, Bp, qs, ldw, dv);
    for (int e = threadIdx.x; e < Bp * dv; e += blockDim.x) {
      const int bb = e / dv, c = e - bb * dv;
      outv[e] = from_f64<TIn>(qs[bb * ldw + c]);
    }
  }
}

size_t calibrate_smem_bytes() {
  return ((size_t)kMaxRepr * (kMaxDim + 1) + 32 * (kMaxDim + 1) + 2 * (size_t)kMaxRepr * kLdG +
          (size_t)kMaxRepr * 33 + 3 * kMaxRepr) * sizeof(double);
}

template <typename TIn, typename Acc>
int launch_calibrate(const BuildBatch<Acc>& b, const BuildParams& prm, cudaStream_t st) {
  const size_t smem = calibrate_smem_bytes();
  auto k = calibrate_kernel<TIn, Acc>;
  DCC_CHECK(check_cuda(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                       "calibrate smem"));
  k<<<b.n, 256, smem, st>>>(b, prm);
  return check_launch("calibrate");
}

template int launch_calibrate<float, double>(const BuildBatch<double>&, const BuildParams&, cudaStream_t);
template int launch_calibrate<double, double>(const BuildBatch<double>&, const BuildParams&, cudaStream_t);
template int launch_calibrate<__nv_bfloat16, float>(const BuildBatch<float>&, const BuildParams&, cudaStream_t);

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
