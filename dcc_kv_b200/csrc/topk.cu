// Top-B key selection over the RMS scores (key_selection.py:56-61) and the
// C_K gather, one CTA per problem.
//
// Scores are non-negative, so their IEEE bit patterns order like unsigned
// integers.  An MSB-first 8-bit radix select finds the B-th largest pattern
// T and how many of the elements equal to T are kept; a block-wide scan in
// index order then takes every element above T and the lowest-index ones at
// T; a shared-memory bitonic sort orders the B winners by (score desc, index
// asc) -- torch.topk's sorted output, with exact ties by lower index.  When
// B >= L_s the reference returns every key in original order (:48-49).
#include "build_common.cuh"

namespace dcc {

template <typename Acc> struct KeyBits;
template <> struct KeyBits<float> { using U = uint32_t; };
template <> struct KeyBits<double> { using U = uint64_t; };

template <typename U>
__device__ __forceinline__ U key_of(float v) { return __float_as_uint(v); }
template <typename U>
__device__ __forceinline__ U key_of(double v) { return (U)__double_as_longlong(v); }

template <typename U>
struct Entry {
  U key;
  int32_t idx;
};

template <typename U>
__device__ __forceinline__ bool before(const Entry<U>& a, const Entry<U>& b) {
  return a.key > b.key || (a.key == b.key && a.idx < b.idx);
}

template <typename TIn, typename Acc>
__global__ void __launch_bounds__(1024) topk_kernel(const __grid_constant__ BuildBatch<Acc> b,
                                                    const BuildParams prm) {
  using U = typename KeyBits<Acc>::U;
  const BuildDesc<Acc>& p = b.p[blockIdx.x];
  const TIn* K = static_cast<const TIn*>(p.keys);
  TIn* outk = static_cast<TIn*>(p.out_keys);
  const int64_t L = p.L_s;
  const int B = p.budget;
  if ((int64_t)B >= L) {  // early exit of the reference: all keys, original order
    for (int64_t e = threadIdx.x; e < L * prm.d; e += blockDim.x) {
      const int64_t r = e / prm.d, c = e - r * prm.d;
      outk[e] = K[r * p.ld_k + c];
    }
    for (int64_t j = threadIdx.x; j < L; j += blockDim.x) p.out_idx[j] = j;
    return;
  }
  extern __shared__ unsigned char smem_raw[];
  Entry<U>* ent = reinterpret_cast<Entry<U>*>(smem_raw);
  __shared__ unsigned int hist[256];
  __shared__ U s_prefix;
  __shared__ int s_take;
  __shared__ int scan_gt[1024], scan_eq[1024];
  const Acc* u = p.u;

  U prefix = 0, mask = 0;
  int need = B;  // elements still to take among those matching prefix
  for (int shift = (int)sizeof(U) * 8 - 8; shift >= 0; shift -= 8) {
    for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0;
    __syncthreads();
    // scores of similar magnitude share their leading digits, so lanes that
    // hit the same bin are merged into one shared-memory atomic
    const int64_t jend = (L + blockDim.x - 1) / blockDim.x * blockDim.x;
    for (int64_t j = threadIdx.x; j < jend; j += blockDim.x) {
      const U k = j < L ? key_of<U>(u[j]) : (U)0;
      const bool act = j < L && (k & mask) == prefix;
      const unsigned am = __ballot_sync(0xffffffffu, act);
      if (act) {
        const unsigned bin = (unsigned)((k >> shift) & 0xFF);
        const unsigned peers = __match_any_sync(am, bin);
        if ((threadIdx.x & 31) == (unsigned)(__ffs(peers) - 1)) atomicAdd(&hist[bin], (unsigned)__popc(peers));
      }
    }
    __syncthreads();
    if (threadIdx.x < 32) {
      // lane l owns digits 255 - 8l .. 248 - 8l; find the digit where the
      // running count from the top first reaches `need`
      const int l = threadIdx.x;
      int h8[8], sum = 0;
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        h8[q] = (int)hist[255 - 8 * l - q];
        sum += h8[q];
      }
      int incl = sum;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, o);
        if (l >= o) incl += v;
      }
      const int before = incl - sum;
      const bool mine = before < need && need <= incl;
      if (mine) {
        int cum = before, dsel = 255 - 8 * l;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          if (cum + h8[q] >= need) { dsel = 255 - 8 * l - q; break; }
          cum += h8[q];
        }
        s_take = need - cum;
        s_prefix = prefix | ((U)dsel << shift);
      }
    }
    __syncthreads();
    need = s_take;
    prefix = s_prefix;
    mask |= (U)0xFF << shift;
    __syncthreads();
  }
  const U T = prefix;  // key of the B-th largest; `need` of the ties at T are taken
  // ordered collection: thread t scans a contiguous index range
  const int64_t per = (L + blockDim.x - 1) / blockDim.x;
  const int64_t j0 = (int64_t)threadIdx.x * per, j1 = min(L, j0 + per);
  int ngt = 0, neq = 0;
  for (int64_t j = j0; j < j1; ++j) {
    const U k = key_of<U>(u[j]);
    ngt += k > T;
    neq += k == T;
  }
  scan_gt[threadIdx.x] = ngt;
  scan_eq[threadIdx.x] = neq;
  __syncthreads();
  for (int off = 1; off < (int)blockDim.x; off <<= 1) {  // inclusive Hillis-Steele scan
    const int a = threadIdx.x >= (unsigned)off ? scan_gt[threadIdx.x - off] : 0;
    const int c = threadIdx.x >= (unsigned)off ? scan_eq[threadIdx.x - off] : 0;
    __syncthreads();
    scan_gt[threadIdx.x] += a;
    scan_eq[threadIdx.x] += c;
    __syncthreads();
  }
  int ogt = scan_gt[threadIdx.x] - ngt;
  int oeq = scan_eq[threadIdx.x] - neq;
  const int n_gt = B - need;
  for (int64_t j = j0; j < j1; ++j) {
    const U k = key_of<U>(u[j]);
    if (k > T) {
      ent[ogt++] = Entry<U>{k, (int32_t)j};
    } else if (k == T) {
      if (oeq < need) ent[n_gt + oeq] = Entry<U>{k, (int32_t)j};
      ++oeq;
    }
  }
  int n2 = 1;
  while (n2 < B) n2 <<= 1;
  for (int i = B + threadIdx.x; i < n2; i += blockDim.x) ent[i] = Entry<U>{(U)0, 0x7fffffff};
  __syncthreads();
  // bitonic sort, "before" order
  for (int k = 2; k <= n2; k <<= 1) {
    for (int jj = k >> 1; jj > 0; jj >>= 1) {
      for (int i = threadIdx.x; i < n2; i += blockDim.x) {
        const int l = i ^ jj;
        if (l > i) {
          const bool up = (i & k) == 0;
          Entry<U> a = ent[i], c = ent[l];
          const bool swap = up ? before(c, a) : before(a, c);
          if (swap) { ent[i] = c; ent[l] = a; }
        }
      }
      __syncthreads();
    }
  }
  for (int i = threadIdx.x; i < B; i += blockDim.x) p.out_idx[i] = ent[i].idx;
  // C_K gather: 16-byte chunks when rows allow it
  const int row_bytes = prm.d * (int)sizeof(TIn);
  if (row_bytes % 16 == 0 && (p.ld_k * (int64_t)sizeof(TIn)) % 16 == 0 &&
      (reinterpret_cast<uintptr_t>(K) & 15) == 0 && (reinterpret_cast<uintptr_t>(outk) & 15) == 0) {
    const int cpr = row_bytes / 16;  // chunks per row
    for (int64_t e = threadIdx.x; e < (int64_t)B * cpr; e += blockDim.x) {
      const int64_t r = e / cpr;
      const int c = (int)(e - r * cpr);
      const uint4* src = reinterpret_cast<const uint4*>(K + (int64_t)ent[r].idx * p.ld_k) + c;
      reinterpret_cast<uint4*>(outk + r * prm.d)[c] = *src;
    }
  } else {
    for (int64_t e = threadIdx.x; e < (int64_t)B * prm.d; e += blockDim.x) {
      const int64_t r = e / prm.d, c = e - r * prm.d;
      outk[e] = K[(int64_t)ent[r].idx * p.ld_k + c];
    }
  }
}

template <typename TIn, typename Acc>
int launch_topk(const BuildBatch<Acc>& b, const BuildParams& prm, int max_budget, cudaStream_t st) {
  using U = typename KeyBits<Acc>::U;
  int n2 = 1;
  while (n2 < max_budget) n2 <<= 1;
  const size_t smem = (size_t)n2 * sizeof(Entry<U>);
  auto k = topk_kernel<TIn, Acc>;
  DCC_CHECK(check_cuda(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                       "topk smem"));
  k<<<b.n, 1024, smem, st>>>(b, prm);
  return check_launch("topk");
}

template int launch_topk<float, double>(const BuildBatch<double>&, const BuildParams&, int, cudaStream_t);
template int launch_topk<double, double>(const BuildBatch<double>&, const BuildParams&, int, cudaStream_t);
template int launch_topk<__nv_bfloat16, float>(const BuildBatch<float>&, const BuildParams&, int, cudaStream_t);

}  // namespace dcc
