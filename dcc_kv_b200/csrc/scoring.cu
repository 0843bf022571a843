// Scoring passes of the compact-KV build (CUDA cores, Acc = FP64 for the
// parity path, FP32 for bf16 inputs).
//
// With S = Q^ K^T * scale over the L_s source keys (key_selection.py:52-53):
//   pass 1: per key chunk, the running row max and sum of exp  (online softmax)
//   pass 2: A = exp(S - m) / l exactly as torch.softmax normalises, then
//           u_j = sqrt(sum_a A_aj^2 / M)          (key_selection.py:14-26)
//           mass_a = sum_j A_aj                    (compact_kv.py:97-101)
//           Y_a = sum_j A_aj V_j                   (value_regression.py:65-67)
// so the three softmaxes of the reference over the same logits become two
// streaming reads of K and one of V.  Chunk partials are combined in a fixed
// order (deterministic).
#include <type_traits>

#include "build_common.cuh"

namespace dcc {

// Thread layout: 256 threads = 16 (ty) x 16 (tx).  A thread owns queries
// ty + 16 i (i < 4) and tile keys tx, tx + 16.
template <typename TIn, typename Acc>
__device__ __forceinline__ void load_tile(Acc* dst, int ld_dst, const TIn* src, int64_t ld_src,
                                          int64_t row0, int64_t nrows_total, int rows, int cols) {
  for (int e = threadIdx.x; e < rows * cols; e += blockDim.x) {
    const int r = e / cols, c = e - r * cols;
    const int64_t gr = row0 + r;
    dst[r * ld_dst + c] = gr < nrows_total ? to_acc<Acc, TIn>(src[gr * ld_src + c]) : Acc(0);
  }
}

template <typename TIn, typename Acc>
__device__ __forceinline__ void tile_logits(const Acc* qs, const Acc* ks, int ld, int d, int ty,
                                            int tx, Acc s[4][2]) {
#pragma unroll
  for (int i = 0; i < 4; ++i) s[i][0] = s[i][1] = Acc(0);
  for (int c = 0; c < d; ++c) {
    const Acc k0 = ks[tx * ld + c], k1 = ks[(tx + 16) * ld + c];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const Acc qv = qs[(ty + 16 * i) * ld + c];
      s[i][0] = fma(qv, k0, s[i][0]);
      s[i][1] = fma(qv, k1, s[i][1]);
    }
  }
}

template <typename TIn, typename Acc>
__global__ void __launch_bounds__(256) score_stats_kernel(const __grid_constant__ BuildBatch<Acc> b,
                                                          const BuildParams prm) {
  const BuildDesc<Acc>& p = b.p[blockIdx.y];
  const int chunk = blockIdx.x;
  if (chunk >= p.n_chunks) return;
  extern __shared__ unsigned char smem_raw[];
  Acc* smem = reinterpret_cast<Acc*>(smem_raw);
  const int ld = prm.d + 1;
  Acc* qs = smem;                 // [64, d+1]
  Acc* ks = qs + kMaxRepr * ld;   // [32, d+1]
  const int ty = threadIdx.x >> 4, tx = threadIdx.x & 15;
  load_tile<TIn, Acc>(qs, ld, static_cast<const TIn*>(p.repr), prm.d, 0, p.M, kMaxRepr, prm.d);
  const Acc scale = Acc(prm.scale);
  Acc m[4], l[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) { m[i] = NegInf<Acc>::v(); l[i] = Acc(0); }
  const int64_t k0 = (int64_t)chunk * p.chunk_len;
  const int64_t k1 = min(p.L_s, k0 + p.chunk_len);
  for (int64_t t0 = k0; t0 < k1; t0 += kScoreTile) {
    __syncthreads();
    load_tile<TIn, Acc>(ks, ld, static_cast<const TIn*>(p.keys), p.ld_k, t0, k1, kScoreTile, prm.d);
    __syncthreads();
    Acc s[4][2];
    tile_logits<TIn, Acc>(qs, ks, ld, prm.d, ty, tx, s);
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      if (t0 + tx + 16 * j < k1) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const Acc x = s[i][j] * scale;
          const Acc mn = max(m[i], x);
          l[i] = l[i] * acc_exp(m[i] - mn) + acc_exp(x - mn);
          m[i] = mn;
        }
      }
    }
  }
  // combine the 16 tx lanes (same half-warp) per query
#pragma unroll
  for (int i = 0; i < 4; ++i) {
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) {
      const Acc m2 = __shfl_xor_sync(0xffffffffu, m[i], o);
      const Acc l2 = __shfl_xor_sync(0xffffffffu, l[i], o);
      const Acc mn = max(m[i], m2);
      if (mn == NegInf<Acc>::v()) continue;
      l[i] = l[i] * acc_exp(m[i] - mn) + l2 * acc_exp(m2 - mn);
      m[i] = mn;
    }
    const int a = ty + 16 * i;
    if (tx == 0 && a < p.M) {
      p.stats[((int64_t)chunk * p.M + a) * 2 + 0] = m[i];
      p.stats[((int64_t)chunk * p.M + a) * 2 + 1] = l[i];
    }
  }
}

template <typename TIn, typename Acc>
__global__ void __launch_bounds__(256) score_probs_kernel(const __grid_constant__ BuildBatch<Acc> b,
                                                          const BuildParams prm) {
  const BuildDesc<Acc>& p = b.p[blockIdx.y];
  const int chunk = blockIdx.x;
  if (chunk >= p.n_chunks) return;
  extern __shared__ unsigned char smem_raw[];
  Acc* smem = reinterpret_cast<Acc*>(smem_raw);
  const int ld = prm.d + 1, ldv = prm.dv + 1;
  Acc* qs = smem;                       // [64, d+1]
  Acc* ks = qs + kMaxRepr * ld;         // [32, d+1]
  Acc* vs = ks + kScoreTile * ld;       // [32, dv+1]
  Acc* ps = vs + kScoreTile * ldv;      // [64, 33]
  Acc* red = ps + kMaxRepr * (kScoreTile + 1);  // [16, 32]
  __shared__ Acc fin_m[kMaxRepr], fin_l[kMaxRepr];
  const int ty = threadIdx.x >> 4, tx = threadIdx.x & 15;
  load_tile<TIn, Acc>(qs, ld, static_cast<const TIn*>(p.repr), prm.d, 0, p.M, kMaxRepr, prm.d);
  // final row statistics from the pass-1 partials (fixed chunk order)
  if (threadIdx.x < kMaxRepr) {
    const int a = threadIdx.x;
    Acc mm = NegInf<Acc>::v(), ll = Acc(0);
    if (a < p.M) {
      for (int c = 0; c < p.n_chunks; ++c) mm = max(mm, p.stats[((int64_t)c * p.M + a) * 2]);
      for (int c = 0; c < p.n_chunks; ++c) {
        const Acc mc = p.stats[((int64_t)c * p.M + a) * 2];
        if (mc != NegInf<Acc>::v()) ll += p.stats[((int64_t)c * p.M + a) * 2 + 1] * acc_exp(mc - mm);
      }
    }
    fin_m[a] = mm;
    fin_l[a] = ll;
  }
  const Acc scale = Acc(prm.scale);
  Acc mass[4] = {0, 0, 0, 0};
  Acc y[4][8];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int v = 0; v < 8; ++v) y[i][v] = Acc(0);
  const int64_t k0 = (int64_t)chunk * p.chunk_len;
  const int64_t k1 = min(p.L_s, k0 + p.chunk_len);
  for (int64_t t0 = k0; t0 < k1; t0 += kScoreTile) {
    __syncthreads();
    load_tile<TIn, Acc>(ks, ld, static_cast<const TIn*>(p.keys), p.ld_k, t0, k1, kScoreTile, prm.d);
    load_tile<TIn, Acc>(vs, ldv, static_cast<const TIn*>(p.values), p.ld_v, t0, k1, kScoreTile, prm.dv);
    __syncthreads();
    Acc s[4][2];
    tile_logits<TIn, Acc>(qs, ks, ld, prm.d, ty, tx, s);
    Acc sq[2] = {0, 0};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int a = ty + 16 * i;
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const bool ok = a < p.M && (t0 + tx + 16 * j) < k1;
        const Acc pr = ok ? acc_exp(s[i][j] * scale - fin_m[a]) / fin_l[a] : Acc(0);
        ps[a * (kScoreTile + 1) + tx + 16 * j] = pr;
        mass[i] += pr;
        sq[j] = fma(pr, pr, sq[j]);
      }
    }
    red[ty * kScoreTile + tx] = sq[0];
    red[ty * kScoreTile + tx + 16] = sq[1];
    __syncthreads();
    if (threadIdx.x < kScoreTile && t0 + threadIdx.x < k1) {
      Acc tot = 0;
#pragma unroll
      for (int r = 0; r < 16; ++r) tot += red[r * kScoreTile + threadIdx.x];
      p.u[t0 + threadIdx.x] = acc_sqrt(tot / Acc(p.M));  // sqrt(sum / M), key_selection.py:26
    }
    // Y += P V : thread owns queries ty + 16 i, value columns tx + 16 v
    const int jn = (int)((k1 - t0) < kScoreTile ? (k1 - t0) : kScoreTile);
    for (int j = 0; j < jn; ++j) {
      Acc pv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) pv[i] = ps[(ty + 16 * i) * (kScoreTile + 1) + j];
#pragma unroll
      for (int v = 0; v < 8; ++v) {
        const int col = tx + 16 * v;
        const Acc vv = col < prm.dv ? vs[j * ldv + col] : Acc(0);
#pragma unroll
        for (int i = 0; i < 4; ++i) y[i][v] = fma(pv[i], vv, y[i][v]);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    Acc ms = mass[i];
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) ms += __shfl_xor_sync(0xffffffffu, ms, o);
    const int a = ty + 16 * i;
    if (a < p.M) {
      if (tx == 0) p.massp[(int64_t)chunk * p.M + a] = ms;
#pragma unroll
      for (int v = 0; v < 8; ++v) {
        const int col = tx + 16 * v;
        if (col < prm.dv) p.yp[((int64_t)chunk * p.M + a) * prm.dv + col] = y[i][v];
      }
    }
  }
}

bool scoring_tc05_supported(const BuildBatch<float>& b, const BuildParams& prm);
int launch_scoring_tc05(const BuildBatch<float>& b, const BuildParams& prm, int max_chunks, cudaStream_t st);

template <typename TIn, typename Acc>
int launch_scoring(const BuildBatch<Acc>& b, const BuildParams& prm, int max_chunks,
                   cudaStream_t st) {
  if constexpr (std::is_same<TIn, __nv_bfloat16>::value) {
    // bf16, d = dv = 128, M <= 64: the tensor-core passes (scoring_tc05.cu)
    if (scoring_tc05_supported(b, prm)) return launch_scoring_tc05(b, prm, max_chunks, st);
  }
  const int ld = prm.d + 1, ldv = prm.dv + 1;
  const size_t smem1 = (size_t)(kMaxRepr + kScoreTile) * ld * sizeof(Acc);
  const size_t smem2 = ((size_t)(kMaxRepr + kScoreTile) * ld + (size_t)kScoreTile * ldv +
                        (size_t)kMaxRepr * (kScoreTile + 1) + 16 * kScoreTile) * sizeof(Acc);
  auto k1 = score_stats_kernel<TIn, Acc>;
  auto k2 = score_probs_kernel<TIn, Acc>;
  DCC_CHECK(check_cuda(cudaFuncSetAttribute(k1, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem1),
                       "score_stats smem"));
  DCC_CHECK(check_cuda(cudaFuncSetAttribute(k2, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem2),
                       "score_probs smem"));
  dim3 grid(max_chunks, b.n);
  k1<<<grid, 256, smem1, st>>>(b, prm);
  DCC_CHECK(check_launch("score_stats"));
  k2<<<grid, 256, smem2, st>>>(b, prm);
  return check_launch("score_probs");
}

template int launch_scoring<float, double>(const BuildBatch<double>&, const BuildParams&, int, cudaStream_t);
template int launch_scoring<double, double>(const BuildBatch<double>&, const BuildParams&, int, cudaStream_t);
template int launch_scoring<__nv_bfloat16, float>(const BuildBatch<float>&, const BuildParams&, int, cudaStream_t);

// rms_per_token_score: u_j = sqrt(sum_a A_aj^2 / M), A [M, L]
template <typename T, typename Acc>
__global__ void rms_kernel(const T* a, int64_t M, int64_t L, T* out) {
  for (int64_t j = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; j < L;
       j += (int64_t)gridDim.x * blockDim.x) {
    Acc s = 0;
    for (int64_t i = 0; i < M; ++i) {
      const Acc v = to_acc<Acc, T>(a[i * L + j]);
      s = fma(v, v, s);
    }
    out[j] = from_f64<T>((double)acc_sqrt(s / Acc(M)));
  }
}

}  // namespace dcc

using namespace dcc;

extern "C" int dcc_rms_per_token_score(const void* attention, int64_t M, int64_t L, int dtype,
                                       void* out, void* stream) {
  if (M <= 0 || L < 0 || !attention || !out)
    return fail(DCC_ERR_INVALID_ARGUMENT, "rms_per_token_score: bad arguments");
  if (L == 0) return DCC_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t gw = (L + 255) / 256, gc = (int64_t)num_sms() * 16;
  const int grid = (int)(gw < gc ? gw : gc);
  switch (dtype) {
    case DCC_BF16: rms_kernel<__nv_bfloat16, float><<<grid, 256, 0, st>>>((const __nv_bfloat16*)attention, M, L, (__nv_bfloat16*)out); break;
    case DCC_F32: rms_kernel<float, double><<<grid, 256, 0, st>>>((const float*)attention, M, L, (float*)out); break;
    case DCC_F64: rms_kernel<double, double><<<grid, 256, 0, st>>>((const double*)attention, M, L, (double*)out); break;
    default: return fail(DCC_ERR_DTYPE, "rms_per_token_score: unsupported dtype");
  }
  return check_launch("rms_per_token_score");
}
