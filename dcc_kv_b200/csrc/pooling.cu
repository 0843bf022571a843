// Representative-query pooling: Rademacher projection + double
// normalisation, then farthest-point sampling, all in FP64.
//
// Follows representative_query.py:82-110 (projection :106-108, FPS :34-79).
// FP64 keeps every argmax of the greedy FPS identical to the FP64 reference:
// the top two candidates of a step can sit closer than fp32 resolution.
//
// FPS runs as one thread-block cluster per query set.  Each thread holds one
// projected point (DPP doubles) in registers for all M steps, so a step is a
// register dot product, a warp/CTA argmax, DSMEM stores of each CTA's winner
// into every CTA of the cluster and one cluster barrier -- no N x N matrix,
// no HBM traffic.  The argmax breaks ties toward the lower index, as
// torch.argmax does.
#include <cooperative_groups.h>

#include <type_traits>
#include <vector>

#include "common.cuh"

namespace cg = cooperative_groups;

namespace dcc {

struct SetDesc {
  const void* q;
  int64_t seg_rows, seg_stride, row_stride;
  int32_t n_seg;
  int32_t n;         // total rows N
  int64_t start;     // FPS start index
  double* normed;    // workspace [N, DPP]
  double* mind;      // workspace [N] (global-memory FPS only)
  void* out_repr;
  int64_t* out_idx;
};

constexpr int kSetCap = 64;  // sets per launch (kernel-parameter batch)
using SetBatch = Batch<SetDesc, kSetCap>;

// The Rademacher matrix travels as sign bits (bit k*d+j set = +1) plus the
// float32 magnitude, so it needs no device buffer: d_p <= 64, d <= 256.
struct ProjBits {
  uint32_t bits[512];
  float mag;
};

__device__ __forceinline__ int64_t set_row_offset(const SetDesc& s, int64_t i) {
  const int64_t seg = i / s.seg_rows;
  return seg * s.seg_stride + (i - seg * s.seg_rows) * s.row_stride;
}

// ---- projection: normed[i] = n(n(Q_i P^T)),  n(z) = z / (||z|| + 1e-8) ------
// One thread per query row holds all DPP projected coordinates in registers.
// P[k][c] = +-mag sits in shared memory as FP64 (zero for k >= d_p), so
// z_k = sum_c fma(P[k][c], q_c, .): the product +-mag * q_c is exact in FP64
// for bf16 / fp32 queries (as in the reference's FP64 matmul), only the
// summation order differs.
template <typename T>
__device__ __forceinline__ double load_row_elem(const T* q, int c) { return to_f64<T>(q[c]); }

// Eight consecutive elements from a 16-byte-aligned address, widened to FP64.
template <typename T>
__device__ __forceinline__ void load8(const T* p, double* out);
template <>
__device__ __forceinline__ void load8<__nv_bfloat16>(const __nv_bfloat16* p, double* out) {
  const uint4 v = *reinterpret_cast<const uint4*>(p);
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    out[2 * i] = (double)__uint_as_float(w[i] << 16);
    out[2 * i + 1] = (double)__uint_as_float(w[i] & 0xffff0000u);
  }
}
template <>
__device__ __forceinline__ void load8<float>(const float* p, double* out) {
  const float4 a = reinterpret_cast<const float4*>(p)[0], b = reinterpret_cast<const float4*>(p)[1];
  out[0] = a.x; out[1] = a.y; out[2] = a.z; out[3] = a.w;
  out[4] = b.x; out[5] = b.y; out[6] = b.z; out[7] = b.w;
}
template <>
__device__ __forceinline__ void load8<double>(const double* p, double* out) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const double2 v = reinterpret_cast<const double2*>(p)[i];
    out[2 * i] = v.x;
    out[2 * i + 1] = v.y;
  }
}

template <int DPP>
__device__ __forceinline__ void project_accumulate(double* z, const double* pm_c, double qc) {
#pragma unroll
  for (int k = 0; k < DPP; k += 2) {
    const double2 pv = *reinterpret_cast<const double2*>(pm_c + k);
    z[k] = fma(pv.x, qc, z[k]);
    z[k + 1] = fma(pv.y, qc, z[k + 1]);
  }
}
template <int DPP>
__device__ __forceinline__ void project_accumulate(float* z, const float* pm_c, float qc) {
#pragma unroll
  for (int k = 0; k < DPP; k += 4) {
    const float4 pv = *reinterpret_cast<const float4*>(pm_c + k);
    z[k] = fmaf(pv.x, qc, z[k]);
    z[k + 1] = fmaf(pv.y, qc, z[k + 1]);
    z[k + 2] = fmaf(pv.z, qc, z[k + 2]);
    z[k + 3] = fmaf(pv.w, qc, z[k + 3]);
  }
}

// Projection arithmetic: FP64 for fp32 / fp64 query sets (the parity path:
// FPS argmax identical to the FP64 reference), fp32 for bf16 sets, whose FPS
// runs on fp32 points anyway.
template <typename T> struct ProjAcc { using A = double; };
template <> struct ProjAcc<__nv_bfloat16> { using A = float; };

template <typename T, int DPP>
__global__ void __launch_bounds__(128) project_kernel(const __grid_constant__ SetBatch b,
                                                      const __grid_constant__ ProjBits proj, int d,
                                                      int dp) {
  using A = typename ProjAcc<T>::A;
  extern __shared__ __align__(16) unsigned char pm_raw[];
  A* pm = reinterpret_cast<A*>(pm_raw);  // [d][DPP]
  const SetDesc& s = b.p[blockIdx.y];
  const A mag = (A)proj.mag;
  for (int e = threadIdx.x; e < d * DPP; e += blockDim.x) {
    const int c = e / DPP, k = e - c * DPP;
    const int bit = k * d + c;
    pm[e] = k < dp ? (((proj.bits[bit >> 5] >> (bit & 31)) & 1u) ? mag : -mag) : (A)0;
  }
  __syncthreads();
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= s.n) return;
  const T* q = static_cast<const T*>(s.q) + set_row_offset(s, i);
  A z[DPP];
#pragma unroll
  for (int k = 0; k < DPP; ++k) z[k] = (A)0;
  if (d % 8 == 0 && (reinterpret_cast<uintptr_t>(q) & 15) == 0) {
    for (int c0 = 0; c0 < d; c0 += 8) {
      double qv[8];
      load8<T>(q + c0, qv);
#pragma unroll
      for (int j = 0; j < 8; ++j) project_accumulate<DPP>(z, pm + (c0 + j) * DPP, (A)qv[j]);
    }
  } else {
    for (int c = 0; c < d; ++c) project_accumulate<DPP>(z, pm + c * DPP, (A)load_row_elem<T>(q, c));
  }
  A ss = (A)0;
#pragma unroll
  for (int k = 0; k < DPP; ++k) ss = fma(z[k], z[k], ss);
  A inv = (A)1 / (sqrt(ss) + (A)1e-8);
  ss = (A)0;
#pragma unroll
  for (int k = 0; k < DPP; ++k) {
    z[k] = z[k] * inv;  // z / (||z|| + 1e-8), representative_query.py:108
    ss = fma(z[k], z[k], ss);
  }
  inv = (A)1 / (sqrt(ss) + (A)1e-8);  // normalised again inside FPS, :63
#pragma unroll
  for (int k = 0; k < DPP; ++k) s.normed[i * DPP + k] = (double)(z[k] * inv);
}

// Argmax keys: a double maps to a uint64 that orders like the double (larger
// key = larger value; -0 is folded into +0 first so that equal values get
// equal keys), and ties go to the lower index, as torch.argmax does.
__device__ __forceinline__ unsigned long long order_key(double v) {
  const long long b = __double_as_longlong(v + 0.0);
  return b >= 0 ? (unsigned long long)b | 0x8000000000000000ull : ~(unsigned long long)b;
}
// Warp-wide argmax of (key, idx) with three redux instructions; every lane
// returns the winning key and index.
__device__ __forceinline__ void warp_argmax_key(unsigned long long& key, int& idx, unsigned mask = 0xffffffffu) {
  const unsigned hi = __reduce_max_sync(mask, (unsigned)(key >> 32));
  const bool m1 = (unsigned)(key >> 32) == hi;
  const unsigned lo = __reduce_max_sync(mask, m1 ? (unsigned)key : 0u);
  const bool m2 = m1 && (unsigned)key == lo;
  idx = (int)__reduce_min_sync(mask, m2 ? (unsigned)idx : 0x7fffffffu);
  key = ((unsigned long long)hi << 32) | lo;
}

struct Cand {
  double v;
  int i;
};
__device__ __forceinline__ bool better(double va, int ia, double vb, int ib) {
  return va > vb || (va == vb && ia < ib);
}
__device__ __forceinline__ void warp_argmax(double& v, int& i) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const double v2 = __shfl_xor_sync(0xffffffffu, v, o);
    const int i2 = __shfl_xor_sync(0xffffffffu, i, o);
    if (better(v2, i2, v, i)) { v = v2; i = i2; }
  }
}

template <int DPP>
struct ClusterSlot {
  unsigned long long key;
  int i;
  int pad;
  double coords[DPP];
};

// ---- FPS, register-resident: one cluster of CL CTAs x T threads per set -------
// A step: warp argmax (redux) -> per-warp winners in shared memory -> warp 0
// takes the CTA winner and stores it (key, index, coordinates) into slot
// [step parity][own rank] of every CTA of the cluster -> one cluster barrier
// -> every warp reduces the cluster's slots from its own shared memory and
// reads the winner's coordinates there.  Slots are double-buffered by step
// parity: a CTA overwrites a parity only after the next barrier, which every
// CTA reaches after its reads of that parity.
template <typename T, int DPP, int TPB>
__global__ void __launch_bounds__(TPB) fps_cluster_kernel(const __grid_constant__ SetBatch b, int M,
                                                          int d) {
  cg::cluster_group cluster = cg::this_cluster();
  const int cl = (int)cluster.num_blocks();
  const int rank = (int)cluster.block_rank();
  const SetDesc& s = b.p[blockIdx.x / cl];
  constexpr int NW = TPB / 32;
  __shared__ unsigned long long wkey[NW];
  __shared__ int widx[NW];
  __shared__ double wcoords[NW][DPP];
  __shared__ ClusterSlot<DPP> cslot[2][16];
  __shared__ double ystart[DPP];
  __shared__ int sel[256];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int me = rank * TPB + threadIdx.x;
  const bool valid = me < s.n;
  double x[DPP];
#pragma unroll
  for (int k = 0; k < DPP; ++k) x[k] = valid ? s.normed[(int64_t)me * DPP + k] : 0.0;
  if (threadIdx.x < DPP) ystart[threadIdx.x] = s.normed[s.start * DPP + threadIdx.x];
  if (threadIdx.x == 0) sel[0] = (int)s.start;
  __syncthreads();
  double mind;
  {
    double dp4[4] = {0.0, 0.0, 0.0, 0.0};
#pragma unroll
    for (int k = 0; k < DPP; ++k) dp4[k & 3] = fma(x[k], ystart[k], dp4[k & 3]);
    mind = valid ? 1.0 - ((dp4[0] + dp4[1]) + (dp4[2] + dp4[3])) : -INFINITY;
  }
  for (int t = 1; t < M; ++t) {
    const int par = t & 1;
    unsigned long long key = order_key(mind);
    int bi = valid ? me : 0x7fffffff;
    warp_argmax_key(key, bi);
    if (valid && bi == me) {
#pragma unroll
      for (int k = 0; k < DPP; ++k) wcoords[warp][k] = x[k];
    }
    if (lane == 0) {
      wkey[warp] = key;
      widx[warp] = bi;
    }
    __syncthreads();
    if (warp == 0) {
      unsigned long long ck = lane < NW ? wkey[lane] : 0ull;
      int ci = lane < NW ? widx[lane] : 0x7fffffff;
      const int my_i = ci;
      warp_argmax_key(ck, ci);
      const int bw = __ffs(__ballot_sync(0xffffffffu, lane < NW && my_i == ci)) - 1;
      for (int dst = 0; dst < cl; ++dst) {
        ClusterSlot<DPP>* rs = cluster.map_shared_rank(&cslot[par][rank], dst);
        if (lane < DPP) rs->coords[lane] = wcoords[bw][lane];
        if (DPP > 32 && lane + 32 < DPP) rs->coords[lane + 32] = wcoords[bw][lane + 32];
        if (lane == 0) {
          rs->key = ck;
          rs->i = ci;
        }
      }
    }
    if (cl > 1) cluster.sync(); else __syncthreads();
    unsigned long long gk = lane < cl ? cslot[par][lane].key : 0ull;
    int gi = lane < cl ? cslot[par][lane].i : 0x7fffffff;
    const int my_gi = gi;
    warp_argmax_key(gk, gi);
    const int gw = __ffs(__ballot_sync(0xffffffffu, lane < cl && my_gi == gi)) - 1;
    if (threadIdx.x == 0) sel[t] = gi;
    const double* y = cslot[par][gw].coords;
    double dp4[4] = {0.0, 0.0, 0.0, 0.0};  // four independent FMA chains
#pragma unroll
    for (int k = 0; k < DPP; ++k) dp4[k & 3] = fma(x[k], y[k], dp4[k & 3]);
    const double dot = (dp4[0] + dp4[1]) + (dp4[2] + dp4[3]);
    if (valid) mind = fmin(mind, 1.0 - dot);
  }
  // keep this CTA's shared memory alive until every remote access finished
  if (cl > 1) cluster.sync();
  if (rank == 0) {
    for (int t = threadIdx.x; t < M; t += TPB) s.out_idx[t] = sel[t];
    if (s.out_repr == nullptr) return;
    const T* q = static_cast<const T*>(s.q);
    T* out = static_cast<T*>(s.out_repr);
    for (int e = threadIdx.x; e < M * d; e += TPB) {
      const int t = e / d, c = e - t * d;
      out[e] = q[set_row_offset(s, sel[t]) + c];
    }
  }
}

// ---- FPS for bf16 query sets: fp32 points, PPT per thread ------------------------
// The same step as fps_cluster_kernel with the projected points rounded to
// fp32 (the FP64 projection and normalisation are unchanged): half the
// registers per point, so a set of 8192 points needs a cluster of 8 CTAs
// instead of 16 and twice as many sets run at once.  Distances are fp32, so
// two candidates closer than fp32 resolution may be ordered differently from
// the FP64 oracle; the bf16 path is held to its output tolerance, not to
// index equality.
__device__ __forceinline__ unsigned order_key32(float v) {
  const int b = __float_as_int(v + 0.f);
  return b >= 0 ? (unsigned)b | 0x80000000u : ~(unsigned)b;
}
__device__ __forceinline__ void warp_argmax_key32(unsigned& key, int& idx) {
  const unsigned hi = __reduce_max_sync(0xffffffffu, key);
  idx = (int)__reduce_min_sync(0xffffffffu, key == hi ? (unsigned)idx : 0x7fffffffu);
  key = hi;
}

template <int DPP>
struct ClusterSlot32 {
  unsigned key;
  int i;
  float coords[DPP];
};

template <typename T, int DPP, int TPB, int PPT>
__global__ void __launch_bounds__(TPB) fps_cluster32_kernel(const __grid_constant__ SetBatch b, int M, int d) {
  cg::cluster_group cluster = cg::this_cluster();
  const int cl = (int)cluster.num_blocks();
  const int rank = (int)cluster.block_rank();
  const SetDesc& s = b.p[blockIdx.x / cl];
  constexpr int NW = TPB / 32;
  __shared__ unsigned wkey[NW];
  __shared__ int widx[NW];
  __shared__ float wcoords[NW][DPP];
  __shared__ ClusterSlot32<DPP> cslot[2][16];
  __shared__ float ystart[DPP];
  __shared__ int sel[256];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float x[PPT][DPP];
  float mind[PPT];
  int pid[PPT];
#pragma unroll
  for (int q = 0; q < PPT; ++q) {
    pid[q] = rank * TPB * PPT + q * TPB + threadIdx.x;  // consecutive threads, consecutive points
    const bool valid = pid[q] < s.n;
#pragma unroll
    for (int k = 0; k < DPP; ++k) x[q][k] = valid ? (float)s.normed[(int64_t)pid[q] * DPP + k] : 0.f;
  }
  if (threadIdx.x < DPP) ystart[threadIdx.x] = (float)s.normed[s.start * DPP + threadIdx.x];
  if (threadIdx.x == 0) sel[0] = (int)s.start;
  __syncthreads();
  auto dist_to = [&](int q, const float* y) {
    float dp4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int k = 0; k < DPP; ++k) dp4[k & 3] = fmaf(x[q][k], y[k], dp4[k & 3]);
    return 1.f - ((dp4[0] + dp4[1]) + (dp4[2] + dp4[3]));
  };
#pragma unroll
  for (int q = 0; q < PPT; ++q) mind[q] = pid[q] < s.n ? dist_to(q, ystart) : -INFINITY;
  for (int t = 1; t < M; ++t) {
    const int par = t & 1;
    // this thread's best point (larger distance, then lower index)
    unsigned key = order_key32(mind[0]);
    int bi = pid[0] < s.n ? pid[0] : 0x7fffffff;
    int bq = 0;
#pragma unroll
    for (int q = 1; q < PPT; ++q) {
      const unsigned kq = order_key32(mind[q]);
      if (pid[q] < s.n && kq > key) {
        key = kq;
        bi = pid[q];
        bq = q;
      }
    }
    const int my_i = bi;
    warp_argmax_key32(key, bi);
    if (my_i == bi && bi != 0x7fffffff) {
#pragma unroll
      for (int q = 0; q < PPT; ++q)
        if (q == bq) {
#pragma unroll
          for (int k = 0; k < DPP; ++k) wcoords[warp][k] = x[q][k];
        }
    }
    if (lane == 0) {
      wkey[warp] = key;
      widx[warp] = bi;
    }
    __syncthreads();
    if (warp == 0) {
      unsigned ck = lane < NW ? wkey[lane] : 0u;
      int ci = lane < NW ? widx[lane] : 0x7fffffff;
      const int mine = ci;
      warp_argmax_key32(ck, ci);
      const int bw = __ffs(__ballot_sync(0xffffffffu, lane < NW && mine == ci)) - 1;
      for (int dst = 0; dst < cl; ++dst) {
        ClusterSlot32<DPP>* rs = cluster.map_shared_rank(&cslot[par][rank], dst);
        if (lane < DPP) rs->coords[lane] = wcoords[bw][lane];
        if (DPP > 32 && lane + 32 < DPP) rs->coords[lane + 32] = wcoords[bw][lane + 32];
        if (lane == 0) {
          rs->key = ck;
          rs->i = ci;
        }
      }
    }
    if (cl > 1) cluster.sync(); else __syncthreads();
    unsigned gk = lane < cl ? cslot[par][lane].key : 0u;
    int gi = lane < cl ? cslot[par][lane].i : 0x7fffffff;
    const int my_gi = gi;
    warp_argmax_key32(gk, gi);
    const int gw = __ffs(__ballot_sync(0xffffffffu, lane < cl && my_gi == gi)) - 1;
    if (threadIdx.x == 0) sel[t] = gi;
    const float* y = cslot[par][gw].coords;
#pragma unroll
    for (int q = 0; q < PPT; ++q)
      if (pid[q] < s.n) mind[q] = fminf(mind[q], dist_to(q, y));
  }
  // keep this CTA's shared memory alive until every remote access finished
  if (cl > 1) cluster.sync();
  if (rank == 0) {
    for (int t = threadIdx.x; t < M; t += TPB) s.out_idx[t] = sel[t];
    if (s.out_repr == nullptr) return;
    const T* q = static_cast<const T*>(s.q);
    T* out = static_cast<T*>(s.out_repr);
    for (int e = threadIdx.x; e < M * d; e += TPB) {
      const int t = e / d, c = e - t * d;
      out[e] = q[set_row_offset(s, sel[t]) + c];
    }
  }
}

// ---- FPS from global memory: any N (one CTA per set) --------------------------
template <typename T, int DPP>
__global__ void __launch_bounds__(1024) fps_global_kernel(const __grid_constant__ SetBatch b, int M,
                                                          int d) {
  const SetDesc& s = b.p[blockIdx.x];
  __shared__ double ynew[DPP];
  __shared__ Cand wbest[32];
  __shared__ int sel[256];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x < DPP) ynew[threadIdx.x] = s.normed[s.start * DPP + threadIdx.x];
  if (threadIdx.x == 0) sel[0] = (int)s.start;
  __syncthreads();
  for (int t = 0; t < M; ++t) {
    double v = -INFINITY;
    int bi = 0x7fffffff;
    for (int i = threadIdx.x; i < s.n; i += blockDim.x) {
      double dot = 0.0;
#pragma unroll
      for (int k = 0; k < DPP; ++k) dot = fma(s.normed[(int64_t)i * DPP + k], ynew[k], dot);
      const double dist = 1.0 - dot;
      const double md = t == 0 ? dist : fmin(s.mind[i], dist);
      s.mind[i] = md;
      if (better(md, i, v, bi)) { v = md; bi = i; }
    }
    if (t == M - 1) break;
    warp_argmax(v, bi);
    if (lane == 0) wbest[warp] = Cand{v, bi};
    __syncthreads();
    if (warp == 0) {
      double bv = lane < (int)(blockDim.x >> 5) ? wbest[lane].v : -INFINITY;
      int bb = lane < (int)(blockDim.x >> 5) ? wbest[lane].i : 0x7fffffff;
      warp_argmax(bv, bb);
      if (lane == 0) sel[t + 1] = bb;
    }
    __syncthreads();
    if (threadIdx.x < DPP) ynew[threadIdx.x] = s.normed[(int64_t)sel[t + 1] * DPP + threadIdx.x];
    __syncthreads();
  }
  __syncthreads();
  for (int t = threadIdx.x; t < M; t += blockDim.x) s.out_idx[t] = sel[t];
  if (s.out_repr == nullptr) return;
  const T* q = static_cast<const T*>(s.q);
  T* out = static_cast<T*>(s.out_repr);
  for (int e = threadIdx.x; e < M * d; e += blockDim.x) {
    const int t = e / d, c = e - t * d;
    out[e] = q[set_row_offset(s, sel[t]) + c];
  }
}

// M >= N: FPS returns arange(N) (representative_query.py:56-57)
template <typename T>
__global__ void gather_all_kernel(const __grid_constant__ SetBatch b, int d) {
  const SetDesc& s = b.p[blockIdx.x];
  for (int t = threadIdx.x; t < s.n; t += blockDim.x) s.out_idx[t] = t;
  if (s.out_repr == nullptr) return;
  const T* q = static_cast<const T*>(s.q);
  T* out = static_cast<T*>(s.out_repr);
  for (int64_t e = threadIdx.x; e < (int64_t)s.n * d; e += blockDim.x) {
    const int64_t t = e / d, c = e - t * d;
    out[e] = q[set_row_offset(s, t) + c];
  }
}

// features / (||features|| + 1e-8), zero-padded to DPP columns (FPS input).
template <typename T, int DPP>
__global__ void normalise_kernel(const T* f, int64_t n, int dim, double* out) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    double ss = 0.0;
    for (int k = 0; k < dim; ++k) {
      const double v = to_f64<T>(f[i * dim + k]);
      ss = fma(v, v, ss);
    }
    const double inv = 1.0 / (sqrt(ss) + 1e-8);
    for (int k = 0; k < DPP; ++k) out[i * DPP + k] = k < dim ? to_f64<T>(f[i * dim + k]) * inv : 0.0;
  }
}

static int dpp_for(int dp) { return dp <= 8 ? 8 : dp <= 16 ? 16 : dp <= 32 ? 32 : 64; }

template <typename T, int DPP>
static int run_fps(SetBatch& b, int M, int d, int max_n, cudaStream_t st) {
  // register path: T threads per CTA, up to 16 CTAs per cluster; bf16 sets
  // keep fp32 points, two per thread
  constexpr int TPB = DPP <= 32 ? 512 : 256;
  constexpr int PPT = std::is_same<T, __nv_bfloat16>::value ? 2 : 1;
  const int cl = (max_n + TPB * PPT - 1) / (TPB * PPT);
  if (cl <= 16) {
    int clp = 1;
    while (clp < cl) clp <<= 1;  // power-of-two cluster
    auto kern = PPT == 2 ? fps_cluster32_kernel<T, DPP, TPB, 2> : fps_cluster_kernel<T, DPP, TPB>;
    if (clp > 8) {
      DCC_CHECK(check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1),
                           "fps: allow cluster 16"));
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(b.n * clp, 1, 1);
    cfg.blockDim = dim3(TPB, 1, 1);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = clp;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return check_cuda(cudaLaunchKernelEx(&cfg, kern, b, M, d), "fps_cluster launch");
  }
  fps_global_kernel<T, DPP><<<b.n, 1024, 0, st>>>(b, M, d);
  return check_launch("fps_global");
}

template <typename T>
static int run_pooling(SetBatch& b, int d, int M, int dp, const ProjBits& proj, int max_n,
                       cudaStream_t st) {
  const int dpp = dpp_for(dp);
  // projection
  const int blocks_x = (max_n + 127) / 128;
  dim3 grid(blocks_x, b.n);
  const size_t pm_bytes = (size_t)d * dpp * sizeof(typename ProjAcc<T>::A);
  auto launch = [&](auto kern) -> int {
    DCC_CHECK(check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pm_bytes),
                         "project smem"));
    kern<<<grid, 128, pm_bytes, st>>>(b, proj, d, dp);
    return check_launch("project");
  };
  switch (dpp) {
    case 8: DCC_CHECK(launch(project_kernel<T, 8>)); break;
    case 16: DCC_CHECK(launch(project_kernel<T, 16>)); break;
    case 32: DCC_CHECK(launch(project_kernel<T, 32>)); break;
    default: DCC_CHECK(launch(project_kernel<T, 64>)); break;
  }
  switch (dpp) {
    case 8: return run_fps<T, 8>(b, M, d, max_n, st);
    case 16: return run_fps<T, 16>(b, M, d, max_n, st);
    case 32: return run_fps<T, 32>(b, M, d, max_n, st);
    default: return run_fps<T, 64>(b, M, d, max_n, st);
  }
}

}  // namespace dcc

using namespace dcc;

static int64_t set_rows(const dcc_query_set& s) { return (int64_t)s.n_seg * s.seg_rows; }

extern "C" size_t dcc_select_representative_queries_workspace_bytes(const dcc_query_set* sets,
                                                                    int n_sets, int head_dim,
                                                                    int projection_dim) {
  (void)head_dim;
  Workspace ws(nullptr, 0);
  const int dpp = dpp_for(projection_dim);
  for (int i = 0; i < n_sets; ++i) {
    const int64_t n = set_rows(sets[i]);
    ws.take<double>((size_t)n * dpp);
    ws.take<double>((size_t)n);
  }
  return ws.used + 256;
}

extern "C" int dcc_select_representative_queries(const dcc_query_set* sets, int n_sets, int head_dim,
                                                 int num_samples, int projection_dim, uint64_t seed,
                                                 int dtype, void* workspace, size_t workspace_bytes,
                                                 void* stream) {
  if (n_sets < 0 || head_dim <= 0 || num_samples <= 0 || projection_dim <= 0)
    return fail(DCC_ERR_INVALID_ARGUMENT, "select_representative_queries: bad sizes");
  if (projection_dim > 64 || head_dim > 256)
    return fail(DCC_ERR_UNSUPPORTED,
                "select_representative_queries: projection_dim > 64 or head_dim > 256");
  if (num_samples > 256)
    return fail(DCC_ERR_UNSUPPORTED, "select_representative_queries: num_samples > 256");
  if (n_sets == 0) return DCC_OK;
  for (int i = 0; i < n_sets; ++i) {
    const dcc_query_set& s = sets[i];
    if (!s.queries || !s.out_repr || !s.out_idx || s.n_seg <= 0 || s.seg_rows <= 0 ||
        s.row_stride < head_dim)
      return fail(DCC_ERR_INVALID_ARGUMENT, "select_representative_queries: bad query set");
    if (set_rows(s) > 0x7fffffff)
      return fail(DCC_ERR_UNSUPPORTED, "select_representative_queries: more than 2^31 queries");
  }
  const size_t need = dcc_select_representative_queries_workspace_bytes(sets, n_sets, head_dim,
                                                                        projection_dim);
  if (workspace == nullptr || workspace_bytes < need)
    return fail(DCC_ERR_WORKSPACE, "select_representative_queries: workspace too small (need " +
                                       std::to_string(need) + " bytes)");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  Workspace ws(workspace, workspace_bytes);
  const int dpp = dpp_for(projection_dim);
  // the projection matrix is the same for every set: draw it once on the host
  std::vector<float> pm((size_t)projection_dim * head_dim);
  DCC_CHECK(dcc_rademacher_projection(head_dim, projection_dim, seed, pm.data()));
  ProjBits proj{};
  proj.mag = pm[0] < 0 ? -pm[0] : pm[0];
  for (size_t e = 0; e < pm.size(); ++e)
    if (pm[e] > 0) proj.bits[e >> 5] |= 1u << (e & 31);
  SetBatch fps{}, all{};
  int max_n_fps = 0;
  auto flush = [&](SetBatch& b, bool gather) -> int {
    if (b.n == 0) return DCC_OK;
    int rc = DCC_OK;
    if (gather) {
      switch (dtype) {
        case DCC_BF16: gather_all_kernel<__nv_bfloat16><<<b.n, 256, 0, st>>>(b, head_dim); break;
        case DCC_F32: gather_all_kernel<float><<<b.n, 256, 0, st>>>(b, head_dim); break;
        default: gather_all_kernel<double><<<b.n, 256, 0, st>>>(b, head_dim); break;
      }
      rc = check_launch("gather_all");
    } else {
      switch (dtype) {
        case DCC_BF16: rc = run_pooling<__nv_bfloat16>(b, head_dim, num_samples, projection_dim, proj, max_n_fps, st); break;
        case DCC_F32: rc = run_pooling<float>(b, head_dim, num_samples, projection_dim, proj, max_n_fps, st); break;
        default: rc = run_pooling<double>(b, head_dim, num_samples, projection_dim, proj, max_n_fps, st); break;
      }
      max_n_fps = 0;
    }
    b.n = 0;
    return rc;
  };
  if (dtype != DCC_BF16 && dtype != DCC_F32 && dtype != DCC_F64)
    return fail(DCC_ERR_DTYPE, "select_representative_queries: unsupported dtype");
  for (int i = 0; i < n_sets; ++i) {
    const dcc_query_set& s = sets[i];
    const int64_t n = set_rows(s);
    SetDesc d{};
    d.q = s.queries;
    d.seg_rows = s.seg_rows;
    d.seg_stride = s.seg_stride;
    d.row_stride = s.row_stride;
    d.n_seg = s.n_seg;
    d.n = (int32_t)n;
    d.start = dcc_fps_start_index(n, seed);
    d.normed = ws.take<double>((size_t)n * dpp);
    d.mind = ws.take<double>((size_t)n);
    d.out_repr = s.out_repr;
    d.out_idx = s.out_idx;
    if (num_samples >= n) {
      all.p[all.n++] = d;
      if (all.n == kSetCap) DCC_CHECK(flush(all, true));
    } else {
      fps.p[fps.n++] = d;
      if (n > max_n_fps) max_n_fps = (int)n;
      if (fps.n == kSetCap) DCC_CHECK(flush(fps, false));
    }
  }
  DCC_CHECK(flush(all, true));
  DCC_CHECK(flush(fps, false));
  return DCC_OK;
}

extern "C" size_t dcc_farthest_point_sampling_workspace_bytes(int64_t N, int dim) {
  Workspace ws(nullptr, 0);
  ws.take<double>((size_t)N * dpp_for(dim));
  ws.take<double>((size_t)N);
  return ws.used + 256;
}

extern "C" int dcc_farthest_point_sampling(const void* features, int64_t N, int dim, int num_samples,
                                           uint64_t seed, int dtype, int64_t* out_idx, void* workspace,
                                           size_t workspace_bytes, void* stream) {
  if (!features || !out_idx || N <= 0 || dim <= 0 || num_samples <= 0)
    return fail(DCC_ERR_INVALID_ARGUMENT, "farthest_point_sampling: bad arguments");
  if (dim > 64 || num_samples > 256 || N > 0x7fffffff)
    return fail(DCC_ERR_UNSUPPORTED, "farthest_point_sampling: need dim <= 64, num_samples <= 256");
  if (!workspace || workspace_bytes < dcc_farthest_point_sampling_workspace_bytes(N, dim))
    return fail(DCC_ERR_WORKSPACE, "farthest_point_sampling: workspace too small");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  Workspace ws(workspace, workspace_bytes);
  const int dpp = dpp_for(dim);
  SetBatch b{};
  SetDesc& d = b.p[0];
  d.q = features;
  d.seg_rows = N;
  d.seg_stride = 0;
  d.row_stride = dim;
  d.n_seg = 1;
  d.n = (int32_t)N;
  d.start = dcc_fps_start_index(N, seed);
  d.normed = ws.take<double>((size_t)N * dpp);
  d.mind = ws.take<double>((size_t)N);
  d.out_repr = nullptr;
  d.out_idx = out_idx;
  b.n = 1;
  const int grid = (int)((N + 255) / 256 < 4096 ? (N + 255) / 256 : 4096);
  auto go = [&](auto* tag) -> int {
    using T = std::remove_pointer_t<decltype(tag)>;
    if (num_samples >= N) {
      gather_all_kernel<T><<<1, 256, 0, st>>>(b, dim);
      return check_launch("fps gather_all");
    }
    switch (dpp) {
      case 8: normalise_kernel<T, 8><<<grid, 256, 0, st>>>((const T*)features, N, dim, d.normed); break;
      case 16: normalise_kernel<T, 16><<<grid, 256, 0, st>>>((const T*)features, N, dim, d.normed); break;
      case 32: normalise_kernel<T, 32><<<grid, 256, 0, st>>>((const T*)features, N, dim, d.normed); break;
      default: normalise_kernel<T, 64><<<grid, 256, 0, st>>>((const T*)features, N, dim, d.normed); break;
    }
    DCC_CHECK(check_launch("fps normalise"));
    switch (dpp) {
      case 8: return run_fps<T, 8>(b, num_samples, dim, (int)N, st);
      case 16: return run_fps<T, 16>(b, num_samples, dim, (int)N, st);
      case 32: return run_fps<T, 32>(b, num_samples, dim, (int)N, st);
      default: return run_fps<T, 64>(b, num_samples, dim, (int)N, st);
    }
  };
  switch (dtype) {
    case DCC_BF16: return go((__nv_bfloat16*)nullptr);
    case DCC_F32: return go((float*)nullptr);
    case DCC_F64: return go((double*)nullptr);
    default: return fail(DCC_ERR_DTYPE, "farthest_point_sampling: unsupported dtype");
  }
}
