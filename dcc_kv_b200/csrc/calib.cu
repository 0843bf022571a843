// Logit-bias calibration and compact-value regression of the build, FP64.
//
// beta (calibration.py:63-94): G = exp(Q^ C_K^T * scale) [M, B'];
//   M < B' : w = clamp(G^T (G G^T + lam I)^-1 t, 0) -- the push-through form of
//            the reference's B x B ridge solve clamp(solve(G^T G + lam I, G^T t), 0)
//            (:44-47): the same vector in exact arithmetic, an M x M system;
//   B' <= M: the literal B x B solve, then 100 projected-gradient steps (lr
//            1e-2, ridge toward 1, :54-60);
//   beta = log(max(w, 1e-6)).
// values (value_regression.py:38-78): X = softmax(Q^ C_K^T * scale + beta / M),
//   M < B' : C_V = X^T (X X^T + lam I)^-1 Y ;  B' <= M : (X^T X + lam I)^-1 X^T Y.
//
// Three launches: the two wide GEMM-shaped ends run as grids over (64-key
// tile, problem); everything between them is one CTA per problem, so the
// latency-bound middle of the chain costs one launch instead of four:
//   calib_logits  logits, G and partial Grams G_t G_t^T per tile   [tiles x problems]
//   calib_solve   sum of partial Grams, Cholesky, w, beta; X = row softmax of
//                 (logits + beta / M); X X^T over all tiles; Y from the
//                 scoring partials, Cholesky, W                     [problems]
//   calib_cv      C_V = X^T W per tile                              [tiles x problems]
// Every sum runs in a fixed order, so results do not depend on timing.
#include "dense_fp64.cuh"

namespace dcc {

constexpr int kCalTile = 64;

template <typename Acc>
__device__ __forceinline__ int cal_bp(const BuildDesc<Acc>& p) {
  return (int)((int64_t)p.budget < p.L_s ? (int64_t)p.budget : p.L_s);
}

// sum_t base[t * stride] for t < n, accumulated in t order (the result does
// not depend on timing), with eight loads in flight per step.
template <typename S>
__device__ __forceinline__ double ordered_sum(const S* base, int64_t stride, int n) {
  double s = 0.0;
  for (int t0 = 0; t0 < n; t0 += 8) {
    double v[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) v[q] = t0 + q < n ? (double)base[(int64_t)(t0 + q) * stride] : 0.0;
#pragma unroll
    for (int q = 0; q < 8; ++q) s += v[q];
  }
  return s;
}

// out[k] = ordered_sum(base + e0 + k * step, stride, n) for k < 4 (0 for
// entries at or past `count`): four independent sums, so 32 loads are in
// flight per step instead of 8; each sum adds in the same order.
template <typename S>
__device__ __forceinline__ void ordered_sum4(const S* base, int64_t e0, int64_t step, int64_t count,
                                             int64_t stride, int n, double* out) {
  double s[4] = {0.0, 0.0, 0.0, 0.0};
  for (int t0 = 0; t0 < n; t0 += 8) {
    double v[4][8];
#pragma unroll
    for (int k = 0; k < 4; ++k)
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const int64_t e = e0 + k * step;
        v[k][q] = (e < count && t0 + q < n) ? (double)base[e + (int64_t)(t0 + q) * stride] : 0.0;
      }
#pragma unroll
    for (int k = 0; k < 4; ++k)
#pragma unroll
      for (int q = 0; q < 8; ++q) s[k] += v[k][q];
  }
#pragma unroll
  for (int k = 0; k < 4; ++k) out[k] = s[k];
}

// 64 x 64 partial Gram of a [64][kLdG] shared tile: out[a][a2] = sum_b Z[a][b] Z[a2][b]
// (thread owns rows ta + 16 i and columns tb + 16 j, i, j < 4; 256 threads).
__device__ __forceinline__ void tile_gram(const double* zs, double* out) {
  const int ta = threadIdx.x & 15, tb = threadIdx.x >> 4;
  double acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.0;
  for (int c = 0; c < kCalTile; ++c) {
    double za[4], zb[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      za[i] = zs[(ta + 16 * i) * kLdG + c];
      zb[i] = zs[(tb + 16 * i) * kLdG + c];
    }
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[i][j] = fma(za[i], zb[j], acc[i][j]);
  }
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) out[(ta + 16 * i) * 64 + tb + 16 * j] = acc[i][j];
}

// ---- 1. logits, G, partial Gram of G --------------------------------------------------
// The 64 x 64 logit tile accumulates over the head dimension in 64-column
// halves staged as FP64 in shared memory (no conversion inside the FMA loop;
// 2 x [64][65] doubles + the G tile keep two CTAs per SM).
template <typename TIn, typename Acc>
__global__ void __launch_bounds__(256) calib_logits_kernel(const __grid_constant__ BuildBatch<Acc> b,
                                                           const BuildParams prm) {
  const BuildDesc<Acc>& p = b.p[blockIdx.y];
  const int Bp = cal_bp(p), M = p.M, d = prm.d;
  const int tile = blockIdx.x;
  if (tile >= p.n_btiles) return;
  const int b0 = tile * kCalTile;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  double* qs = reinterpret_cast<double*>(smem_raw);  // [64][kLdG]: 64 columns of the head dim
  double* ks = qs + 64 * kLdG;                       // [64][kLdG]
  double* gs = ks + 64 * kLdG;                       // [64][kLdG]
  const TIn* rq = static_cast<const TIn*>(p.repr);
  const TIn* ck = static_cast<const TIn*>(p.out_keys);
  const int ta = threadIdx.x & 15, tb = threadIdx.x >> 4;
  double acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.0;
  for (int c0 = 0; c0 < d; c0 += 64) {
    const int w = d - c0 < 64 ? d - c0 : 64;
    __syncthreads();  // the previous half is consumed
    for (int e = threadIdx.x; e < 64 * 64; e += blockDim.x) {
      const int r = e >> 6, c = e & 63;
      qs[r * kLdG + c] = (r < M && c < w) ? to_f64<TIn>(rq[r * d + c0 + c]) : 0.0;
      ks[r * kLdG + c] = (b0 + r < Bp && c < w) ? to_f64<TIn>(ck[(int64_t)(b0 + r) * d + c0 + c]) : 0.0;
    }
    __syncthreads();
#pragma unroll 4
    for (int c = 0; c < w; ++c) {
      double qa[4], kb[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        qa[i] = qs[(ta + 16 * i) * kLdG + c];
        kb[i] = ks[(tb + 16 * i) * kLdG + c];
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fma(qa[i], kb[j], acc[i][j]);
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int a = ta + 16 * i;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int bb = tb + 16 * j;
      const bool ok = a < M && b0 + bb < Bp;
      const double lg = acc[i][j] * prm.scale;  // (Q^ C_K^T) * scale, calibration.py:84
      const double g = ok ? exp(lg) : 0.0;
      if (ok) {
        p.X[(int64_t)a * Bp + b0 + bb] = lg;
        p.G[(int64_t)a * Bp + b0 + bb] = g;
      }
      gs[a * kLdG + bb] = g;
    }
  }
  if (!(p.stages & kStageBeta) || M >= Bp) return;
  __syncthreads();
  tile_gram(gs, p.gpart + (int64_t)tile * 4096);
}

// ---- 2. beta (one CTA per problem; shared scratch from calib_solve) ---------------------
struct SolveSmem {
  double* gram;    // [64][kLdG]
  double* gsm;     // [64][kLdG]  G / X (B' <= M), X tiles (M < B')
  double* tv;      // [64] block mass
  double* vv;      // [64]
  double* res;     // [64]
  double* diag;    // [64]
  double* colbuf;  // [132]
  double* rsum;    // [128] row sums of the exponentials, then their reciprocals
  double* xt;      // [64 keys][kLdT] X tile, transposed, 2 doubles of padding per 8 rows
  double* ws;      // [64][dv + 1]
};

// Y = sum over the scoring chunks of the partial A V products, in chunk order,
// into p.Y and the right-hand sides ws [M][dv + 1]; threads [t0, t0 + nt).
template <typename Acc>
__device__ __forceinline__ void y_sums(const BuildDesc<Acc>& p, int dv, double* ws, int tid, int nt) {
  const int M = p.M, ldw = dv + 1;
  for (int e0 = tid; e0 < M * dv; e0 += 4 * nt) {
    double y[4];
    ordered_sum4(p.yp, e0, nt, (int64_t)M * dv, (int64_t)M * dv, p.n_chunks, y);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int e = e0 + k * nt;
      if (e < M * dv) {
        p.Y[e] = y[k];
        ws[(e / dv) * ldw + e % dv] = y[k];
      }
    }
  }
}

template <typename TIn, typename Acc>
__device__ __forceinline__ void beta_stage(const BuildDesc<Acc>& p, const BuildParams& prm, const SolveSmem& sm) {
  const int Bp = cal_bp(p), M = p.M;
  double *gram = sm.gram, *gsm = sm.gsm, *tv = sm.tv, *vv = sm.vv, *res = sm.res;
  // block mass: given, or the pass-2 chunk sums in chunk order
  for (int a = threadIdx.x; a < 64; a += blockDim.x) {
    double s = 0.0;
    if (a < M) {
      if (p.in_mass)
        s = load_side<TIn>(p.in_mass, a);
      else
        s = ordered_sum(p.massp + a, M, p.n_chunks);
    }
    tv[a] = s;
    if (a < M && p.out_mass) p.out_mass[a] = s;
  }
  if (!(p.stages & kStageBeta)) {
    for (int bb = threadIdx.x; bb < Bp; bb += blockDim.x) p.wv[bb] = load_side<TIn>(p.in_beta, bb) / (double)M;
    __syncthreads();
    return;
  }
  __syncthreads();
  const double lb = prm.lambda_beta;
  if (M < Bp) {
    const int nt = blockDim.x;
    for (int e0 = threadIdx.x; e0 < 64 * 64; e0 += 4 * nt) {
      // four Gram entries per thread at once (32 loads in flight); entry e is
      // (a, a2) = (e / 64, e % 64) of the 64 x 64 partials, summed over the
      // tiles in tile order
      double v[4][8], acc[4] = {0.0, 0.0, 0.0, 0.0};
      for (int t0 = 0; t0 < p.n_btiles; t0 += 8) {
#pragma unroll
        for (int k = 0; k < 4; ++k)
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const int e = e0 + k * nt;
            const bool in = e < 4096 && (e >> 6) < M && (e & 63) < M && t0 + q < p.n_btiles;
            v[k][q] = in ? p.gpart[(int64_t)(t0 + q) * 4096 + e] : 0.0;
          }
#pragma unroll
        for (int k = 0; k < 4; ++k)
#pragma unroll
          for (int q = 0; q < 8; ++q) acc[k] += v[k][q];
      }
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int e = e0 + k * nt, a = e >> 6, a2 = e & 63;
        if (e < 4096 && a < M && a2 < M) gram[a * kLdG + a2] = acc[k] + (a == a2 ? lb : 0.0);
      }
    }
    __syncthreads();
    // the factorisation takes threads 0-63; the others sum Y (needed only by
    // the value fit) meanwhile
    if (threadIdx.x < 64)
      chol64_rows(gram, kLdG, M, sm.diag, sm.colbuf);
    else if (p.stages & kStageValues)
      y_sums(p, prm.dv, sm.ws, threadIdx.x - 64, blockDim.x - 64);
    __syncthreads();
    if (threadIdx.x < 64) vv[threadIdx.x] = tv[threadIdx.x];  // zero past M
    __syncthreads();
    if (threadIdx.x < 32) chol64_solve_vec(gram, kLdG, sm.diag, M, vv);
    __syncthreads();
    // w = G^T v: four columns per thread at once (32 loads in flight)
    for (int b0 = threadIdx.x; b0 < Bp; b0 += 4 * nt) {
      double w[4] = {0.0, 0.0, 0.0, 0.0};
      for (int a0 = 0; a0 < M; a0 += 8) {
        double g[4][8];
#pragma unroll
        for (int k = 0; k < 4; ++k)
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const int bb = b0 + k * nt;
            g[k][q] = (a0 + q < M && bb < Bp) ? p.G[(int64_t)(a0 + q) * Bp + bb] : 0.0;
          }
#pragma unroll
        for (int k = 0; k < 4; ++k)
#pragma unroll
          for (int q = 0; q < 8; ++q)
            if (a0 + q < M) w[k] = fma(g[k][q], vv[a0 + q], w[k]);
      }
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int bb = b0 + k * nt;
        if (bb < Bp) p.wv[bb] = w[k] > 0.0 ? w[k] : 0.0;
      }
    }
  } else {
    for (int e = threadIdx.x; e < M * Bp; e += blockDim.x) gsm[(e / Bp) * kLdG + e % Bp] = p.G[e];
    __syncthreads();
    gram_cols(gsm, M, Bp, lb, gram);
    for (int bb = threadIdx.x; bb < 64; bb += blockDim.x) {
      double s = 0.0;
      if (bb < Bp)
        for (int a = 0; a < M; ++a) s = fma(gsm[a * kLdG + bb], tv[a], s);
      vv[bb] = s;
    }
    __syncthreads();
    chol64(gram, kLdG, Bp, sm.diag, sm.colbuf);
    if (threadIdx.x < 32) chol64_solve_vec(gram, kLdG, sm.diag, Bp, vv);
    __syncthreads();
    if (threadIdx.x < Bp) vv[threadIdx.x] = fmax(vv[threadIdx.x], 0.0);
    __syncthreads();
    for (int it = 0; it < 100; ++it) {
      if (threadIdx.x < M) {  // res = G w - t
        double s = 0.0;
        for (int bb = 0; bb < Bp; ++bb) s = fma(gsm[threadIdx.x * kLdG + bb], vv[bb], s);
        res[threadIdx.x] = s - tv[threadIdx.x];
      }
      __syncthreads();
      if (threadIdx.x < Bp) {  // w = max(w - lr (G^T res + lam (w - 1)), 0)
        double g = 0.0;
        for (int a = 0; a < M; ++a) g = fma(gsm[a * kLdG + threadIdx.x], res[a], g);
        g += lb * (vv[threadIdx.x] - 1.0);
        vv[threadIdx.x] = fmax(vv[threadIdx.x] - 1e-2 * g, 0.0);
      }
      __syncthreads();
    }
    if (threadIdx.x < Bp) p.wv[threadIdx.x] = vv[threadIdx.x];
  }
  __syncthreads();
  for (int bb = threadIdx.x; bb < Bp; bb += blockDim.x) {
    const double beta = log(fmax(p.wv[bb], 1e-6));
    // the value fit adds beta / M to every row of logits (value_regression.py:72-73):
    // wv keeps that quotient from here on
    p.wv[bb] = beta / (double)M;
    if (sizeof(TIn) == 8)
      static_cast<double*>(p.out_bias)[bb] = beta;
    else
      static_cast<float*>(p.out_bias)[bb] = (float)beta;
  }
  __syncthreads();
}

// ---- 3. X = softmax_b(logits + beta / M), one warp per row ------------------------------
// Passes over the row (logits + beta / M and the max; exponentials and their
// sum), each issuing eight independent loads per lane before it stores: the
// row lives in L2, and a load-store chain per element would wait on every
// access.  The row sums go to rsum; the division by them happens in
// xgram_stage (M < B', where X is also needed in shared memory for X X^T)
// or in a third pass here (B' <= M).
template <typename Acc>
__device__ __forceinline__ void x_stage(const BuildDesc<Acc>& p, double* rsum) {
  const int Bp = cal_bp(p), M = p.M;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
  const double* __restrict__ bm = p.wv;  // beta / M
  constexpr int kU = 8;
  for (int a = warp; a < M; a += nwarps) {
    double* __restrict__ xr = p.X + (int64_t)a * Bp;
    double mx = -INFINITY;
    for (int b0 = 0; b0 < Bp; b0 += 32 * kU) {
      double v[kU];
#pragma unroll
      for (int q = 0; q < kU; ++q) {
        const int bb = b0 + q * 32 + lane;
        v[q] = bb < Bp ? xr[bb] + bm[bb] : -INFINITY;
      }
#pragma unroll
      for (int q = 0; q < kU; ++q) {
        const int bb = b0 + q * 32 + lane;
        if (bb < Bp) xr[bb] = v[q];
        mx = fmax(mx, v[q]);
      }
    }
    mx = warp_max(mx);
    double sum = 0.0;
    for (int b0 = 0; b0 < Bp; b0 += 32 * kU) {
      double v[kU];
#pragma unroll
      for (int q = 0; q < kU; ++q) {
        const int bb = b0 + q * 32 + lane;
        v[q] = bb < Bp ? xr[bb] : -INFINITY;
      }
#pragma unroll
      for (int q = 0; q < kU; ++q) {
        const int bb = b0 + q * 32 + lane;
        const double e = exp(v[q] - mx);
        if (bb < Bp) {
          xr[bb] = e;
          sum += e;
        }
      }
    }
    sum = warp_sum(sum);
    if (lane == 0) rsum[a] = sum;
    if (M < Bp) continue;
    for (int b0 = 0; b0 < Bp; b0 += 32 * kU) {
      double v[kU];
#pragma unroll
      for (int q = 0; q < kU; ++q) {
        const int bb = b0 + q * 32 + lane;
        v[q] = bb < Bp ? xr[bb] : 0.0;
      }
#pragma unroll
      for (int q = 0; q < kU; ++q) {
        const int bb = b0 + q * 32 + lane;
        if (bb < Bp) xr[bb] = v[q] / sum;
      }
    }
  }
  __syncthreads();
}

// ---- 4. X = exponentials / row sums, tile by tile, and X X^T + lam I (M < B') -----------
constexpr int kLdT = 80;  // transposed X tile: 64 rows + 2 doubles of padding per 8
// Each 64-key tile of the exponentials is loaded once (16 loads per thread in
// flight), scaled by the reciprocal row sums, stored as X (global, for C_V)
// and into shared memory, and folded into the Gram.  The Gram is symmetric:
// 252 threads each own one 8 x 8 block of its lower triangle (36 blocks) for
// one of 7 groups of the tile's columns (c = g, g + 7, ...), 64 accumulators
// in registers, so a thread reads 16 shared values per 64 FMAs; the 7 group
// partials are added in group order at the end and mirrored to the upper
// triangle.
template <typename Acc>
__device__ __forceinline__ void xgram_stage(const BuildDesc<Acc>& p, double lam, double* rsum,
                                            const SolveSmem& sm) {
  const int Bp = cal_bp(p), M = p.M;
  constexpr int kGroups = 7, kBlocks = 36;
  const int t = threadIdx.x;
  const bool active = t < kGroups * kBlocks;
  const int grp = t / kBlocks, blk = t % kBlocks;
  int bi = 0;
  while ((bi + 1) * (bi + 2) / 2 <= blk) ++bi;
  const int bj = blk - bi * (bi + 1) / 2;
  double acc[8][8];
#pragma unroll
  for (int u = 0; u < 8; ++u)
#pragma unroll
    for (int v = 0; v < 8; ++v) acc[u][v] = 0.0;
  if (t < 64) rsum[64 + t] = t < M ? 1.0 / rsum[t] : 0.0;  // reciprocal row sums
  __syncthreads();
  const double* inv = rsum + 64;
  double* xt = sm.xt;
  constexpr int kPer = 64 * kCalTile / 256;  // elements per thread per tile (blockDim.x == 256)
  for (int b0 = 0; b0 < Bp; b0 += kCalTile) {
    double v[kPer];
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int e = t + i * 256, a = e / kCalTile, bb = e % kCalTile;
      v[i] = (a < M && b0 + bb < Bp) ? p.X[(int64_t)a * Bp + b0 + bb] : 0.0;
    }
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int e = t + i * 256, a = e / kCalTile, bb = e % kCalTile;
      const bool in = a < M && b0 + bb < Bp;
      const double x = in ? v[i] * inv[a] : 0.0;
      if (in) p.X[(int64_t)a * Bp + b0 + bb] = x;
      xt[bb * kLdT + a + 2 * (a >> 3)] = x;
    }
    __syncthreads();
    if (active) {
      for (int c = grp; c < kCalTile; c += kGroups) {
        // rows bi*8 .. bi*8+7 are 8 contiguous, 16-byte aligned doubles at
        // bi * 10 (the padding spreads the 8 row blocks over distinct banks)
        double xa[8], xb[8];
        const double2* ra = reinterpret_cast<const double2*>(xt + c * kLdT + bi * 10);
        const double2* rb = reinterpret_cast<const double2*>(xt + c * kLdT + bj * 10);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const double2 a2 = ra[u], b2 = rb[u];
          xa[2 * u] = a2.x;
          xa[2 * u + 1] = a2.y;
          xb[2 * u] = b2.x;
          xb[2 * u + 1] = b2.y;
        }
#pragma unroll
        for (int u = 0; u < 8; ++u)
#pragma unroll
          for (int w = 0; w < 8; ++w) acc[u][w] = fma(xa[u], xb[w], acc[u][w]);
      }
    }
    __syncthreads();
  }
  double* gram = sm.gram;
  for (int g = 0; g < kGroups; ++g) {
    if (active && grp == g) {
#pragma unroll
      for (int u = 0; u < 8; ++u)
#pragma unroll
        for (int w = 0; w < 8; ++w) {
          double* dst = gram + (bi * 8 + u) * kLdG + bj * 8 + w;
          *dst = g == 0 ? acc[u][w] : *dst + acc[u][w];
        }
    }
    __syncthreads();
  }
  for (int e = t; e < 64 * 64; e += blockDim.x) {
    const int a = e >> 6, a2 = e & 63;
    if (a < M && a2 < M) {
      if (a2 > a) gram[a * kLdG + a2] = gram[a2 * kLdG + a];
      else if (a2 == a) gram[a * kLdG + a] += lam;
    }
  }
  __syncthreads();
}

// ---- 5. Y, then W = (X X^T + lam I)^-1 Y   (B' <= M: C_V directly) ----------------------
// For M < B' the Gram (with lam) is already in sm.gram.
// y_done: Y is already in p.Y and ws (summed during the beta factorisation).
template <typename TIn, typename Acc>
__device__ __forceinline__ void w_stage(const BuildDesc<Acc>& p, const BuildParams& prm, const SolveSmem& sm,
                                        bool y_done) {
  const int Bp = cal_bp(p), M = p.M, dv = prm.dv;
  double *gram = sm.gram, *gsm = sm.gsm, *ws = sm.ws;
  const int ldw = dv + 1;
  if (!y_done) y_sums(p, dv, ws, threadIdx.x, blockDim.x);
  const double lv = prm.lambda_value;
  // system size: M x M (push-through form) or B' x B' (literal form)
  const int n = M < Bp ? M : Bp;
  if (M >= Bp) {
    __syncthreads();
    for (int e = threadIdx.x; e < M * Bp; e += blockDim.x) gsm[(e / Bp) * kLdG + e % Bp] = p.X[e];
    __syncthreads();
    gram_cols(gsm, M, Bp, lv, gram);
    // R = X^T Y into ws rows [0, Bp) (Bp <= M <= 64 rows; Y is kept in p.Y)
    __syncthreads();
    for (int e = threadIdx.x; e < Bp * dv; e += blockDim.x) {
      const int bb = e / dv, c = e % dv;
      double s = 0.0;
      for (int a = 0; a < M; ++a) s = fma(gsm[a * kLdG + bb], p.Y[(int64_t)a * dv + c], s);
      ws[bb * ldw + c] = s;
    }
  }
  __syncthreads();
  chol64(gram, kLdG, n, sm.diag, sm.colbuf);
  chol64_solve(gram, kLdG, sm.diag, n, ws, ldw, dv);
  if (M < Bp) {
    for (int e = threadIdx.x; e < M * dv; e += blockDim.x) p.W[e] = ws[(e / dv) * ldw + e % dv];
  } else {
    TIn* outv = static_cast<TIn*>(p.out_values);
    for (int e = threadIdx.x; e < Bp * dv; e += blockDim.x) outv[e] = from_f64<TIn>(ws[(e / dv) * ldw + e % dv]);
  }
}

// stages 2-5, one CTA per problem
template <typename TIn, typename Acc>
__global__ void __launch_bounds__(256) calib_solve_kernel(const __grid_constant__ BuildBatch<Acc> b,
                                                          const BuildParams prm) {
  const BuildDesc<Acc>& p = b.p[blockIdx.x];
  extern __shared__ __align__(16) unsigned char smem_raw[];
  SolveSmem sm;
  sm.gram = reinterpret_cast<double*>(smem_raw);
  sm.gsm = sm.gram + 64 * kLdG;
  sm.tv = sm.gsm + 64 * kLdG;
  sm.vv = sm.tv + 64;
  sm.res = sm.vv + 64;
  sm.diag = sm.res + 64;
  sm.colbuf = sm.diag + 64;
  sm.rsum = sm.colbuf + 132;
  sm.xt = sm.rsum + 128;
  sm.ws = sm.xt + 64 * kLdT;
  beta_stage<TIn, Acc>(p, prm, sm);
  if (!(p.stages & kStageValues)) return;
  x_stage(p, sm.rsum);
  if (p.M < cal_bp(p)) xgram_stage(p, prm.lambda_value, sm.rsum, sm);
  // Y was summed during the beta factorisation on the push-through path
  w_stage<TIn, Acc>(p, prm, sm, (p.stages & kStageBeta) && p.M < cal_bp(p));
}

// ---- 6. C_V = X^T W per 64-key tile --------------------------------------------------------
template <typename TIn, typename Acc>
__global__ void __launch_bounds__(256) calib_cv_kernel(const __grid_constant__ BuildBatch<Acc> b,
                                                       const BuildParams prm) {
  const BuildDesc<Acc>& p = b.p[blockIdx.y];
  const int Bp = cal_bp(p), M = p.M, dv = prm.dv;
  const int tile = blockIdx.x;
  if (!(p.stages & kStageValues) || M >= Bp || tile >= p.n_btiles) return;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  double* xs = reinterpret_cast<double*>(smem_raw);  // [64 a][65]
  double* wsm = xs + 64 * kLdG;                       // [64 a][dv + 1]
  const int ldw = dv + 1;
  const int b0 = tile * kCalTile;
  for (int e = threadIdx.x; e < 64 * kCalTile; e += blockDim.x) {
    const int a = e / kCalTile, bb = e % kCalTile;
    xs[a * kLdG + bb] = (a < M && b0 + bb < Bp) ? p.X[(int64_t)a * Bp + b0 + bb] : 0.0;
  }
  for (int e = threadIdx.x; e < 64 * dv; e += blockDim.x) {
    const int a = e / dv, c = e % dv;
    wsm[a * ldw + c] = a < M ? p.W[(int64_t)a * dv + c] : 0.0;
  }
  __syncthreads();
  // thread: keys tb + 16 i (i < 4), value columns tc + 16 j (j < 8)
  const int tc = threadIdx.x & 15, tb = threadIdx.x >> 4;
  TIn* outv = static_cast<TIn*>(p.out_values);
  for (int c0 = 0; c0 < dv; c0 += 128) {
    double acc[4][8];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[i][j] = 0.0;
    for (int a = 0; a < M; ++a) {
      double xv[4], wv[8];
#pragma unroll
      for (int i = 0; i < 4; ++i) xv[i] = xs[a * kLdG + tb + 16 * i];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int c = c0 + tc + 16 * j;
        wv[j] = c < dv ? wsm[a * ldw + c] : 0.0;
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fma(xv[i], wv[j], acc[i][j]);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int bb = b0 + tb + 16 * i;
      if (bb >= Bp) continue;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int c = c0 + tc + 16 * j;
        if (c < dv) outv[(int64_t)bb * dv + c] = from_f64<TIn>(acc[i][j]);
      }
    }
  }
}

template <typename TIn, typename Acc>
int launch_calibrate(const BuildBatch<Acc>& b, const BuildParams& prm, cudaStream_t st) {
  int tmax = 1;
  for (int i = 0; i < b.n; ++i) tmax = b.p[i].n_btiles > tmax ? b.p[i].n_btiles : tmax;
  const size_t smem1 = 3 * 64 * kLdG * sizeof(double);
  const size_t smem2 = (2 * 64 * kLdG + 4 * 64 + 132 + 128 + 64 * kLdT + 64 * (size_t)(prm.dv + 1)) * sizeof(double);
  const size_t smem6 = (64 * kLdG + 64 * (size_t)(prm.dv + 1)) * sizeof(double);
  auto k1 = calib_logits_kernel<TIn, Acc>;
  auto k2 = calib_solve_kernel<TIn, Acc>;
  auto k6 = calib_cv_kernel<TIn, Acc>;
  DCC_CHECK(check_cuda(cudaFuncSetAttribute(k1, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem1), "calib smem"));
  DCC_CHECK(check_cuda(cudaFuncSetAttribute(k2, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem2), "calib smem"));
  DCC_CHECK(check_cuda(cudaFuncSetAttribute(k6, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem6), "calib smem"));
  const dim3 tiles(tmax, b.n);
  k1<<<tiles, 256, smem1, st>>>(b, prm);
  DCC_CHECK(check_launch("calib_logits"));
  k2<<<b.n, 256, smem2, st>>>(b, prm);
  DCC_CHECK(check_launch("calib_solve"));
  k6<<<tiles, 256, smem6, st>>>(b, prm);
  return check_launch("calib_cv");
}

template int launch_calibrate<float, double>(const BuildBatch<double>&, const BuildParams&, cudaStream_t);
template int launch_calibrate<double, double>(const BuildBatch<double>&, const BuildParams&, cudaStream_t);
template int launch_calibrate<__nv_bfloat16, float>(const BuildBatch<float>&, const BuildParams&, cudaStream_t);

}  // namespace dcc
