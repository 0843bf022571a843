// Scoring passes of the compact-KV build for bf16 inputs on the tcgen05
// tensor cores (head_dim = value_dim = 128, M <= 64 representative queries).
//
// Same outputs as scoring.cu (per key chunk: row max / sum of exp; then RMS
// scores u, block mass and Y = A V partials).  Internally the row statistics
// are kept in log2 units: stats = (m2, l) with m2 = max_j s_aj * scale * log2(e)
// and l = sum_j 2^(s_aj * scale * log2(e) - m2); only the two passes below
// read or write them.
//
// Pass 1 (row statistics), queries in TMEM lanes:
//   S = Q^ K^T        M = 128 (the M query rows, zero-padded), N = 128 keys
//   warps 0, 1, 4, 5: query rows 0-63, each warp half of the 128 key columns
//   (a warp reaches TMEM lanes 32 * (warp % 4) ..); warp 2 TMA, warp 3 MMA.
//
// Pass 2 (probabilities), keys in TMEM lanes -- the transposed problem, so a
// thread owns one key and every per-key quantity stays in its registers:
//   S^T = K Q^T       M = 128 keys, N = 64 queries, both operands K-major
//   p_aj = 2^(s_ja * scale * log2(e) - (m2_a + log2 l_a))    one thread per key
//   u_j  = sqrt(sum_a p_aj^2 / M)                            in-thread
//   P^T  -> shared memory as bf16 hi + lo parts (p = hi + lo to 16 mantissa
//           bits), 128-byte swizzled rows of 64 queries (MN-major operand)
//   Y^T += V^T P^T    M = 128 (head dim, V tile read MN-major), N = 64 queries
//   block mass of the chunk = l_c 2^(m2_c - m2) / l from the statistics
//   warps 0-3: keys / head-dim rows; warp 4 TMA; warp 5 MMA + TMEM owner.
// All waits are bounded and warp-uniform; every tcgen05 ld/st runs on whole
// warps.
#include <memory>
#include <string>

#include "build_common.cuh"
#include "tc05.cuh"

namespace dcc {

using namespace tc05;

constexpr int kScoreTcCap = 56;

struct ScoreTcDesc {
  CUtensorMap k;   // {128, L_s, 1}, box {64, 128, 1}
  CUtensorMap v;
  CUtensorMap q;   // {128, M, 1}: rows >= M read as zero
  int64_t L_s;
  int32_t M, n_chunks, chunk_len, pad;
  float* stats;    // [n_chunks, M, 2]  (m2, l) in log2 units
  float* massp;    // [n_chunks, M]
  float* yp;       // [n_chunks, M, 128]
  float* u;        // [L_s]
};

struct ScoreTcBatch {
  int n;
  float scale;
  ScoreTcDesc p[kScoreTcCap];
};

static __device__ unsigned int g_score_error;

namespace sc {

constexpr int kTile = 128;
constexpr int kTileBytes = 32768;
constexpr int kThreads = 192;
constexpr int kStages1 = 4;     // K tiles in flight, pass 1
constexpr float kLog2e = 1.4426950408889634f;

struct Smem1 {
  unsigned char q[kTileBytes];
  unsigned char k[kStages1][kTileBytes];
  float xm[64], xl[64];  // second column half's (m2, l) per row
  uint64_t bar_q, bar_k[kStages1], bar_empty[kStages1], bar_s[2], bar_sfree[2];
  uint32_t tmem;
};

struct Smem2 {
  unsigned char q[kTileBytes];
  unsigned char k[2][kTileBytes];
  unsigned char v[2][kTileBytes];
  unsigned char ph[2][kTileBytes / 2];  // P^T hi: 128 keys x 64 queries bf16
  unsigned char pl[2][kTileBytes / 2];  // P^T lo
  float mb[64];                          // m2_a + log2 l_a (+inf for padding rows)
  uint64_t bar_q, bar_k[2], bar_v[2], bar_empty[2], bar_s[2], bar_p[2], bar_pfree[2], bar_y;
  uint32_t tmem;
};

__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity) {
  return __all_sync(0xffffffffu, mbar_wait(bar, parity)) != 0;
}
// K-major operand of 128 rows x 128 (two 64-wide halves 16 KB apart), step kk of 16
__device__ __forceinline__ uint64_t kdesc(const unsigned char* tile, int kk) {
  return sdesc_sw128(smem_u32(tile) + (uint32_t)((kk >> 2) * 16384 + (kk & 3) * 32), 16, 1024);
}
// MN-major operand, rows along K: 16 rows (2048 B) per step; 64-wide MN halves 16 KB apart
__device__ __forceinline__ uint64_t mndesc(const unsigned char* tile, int kk) {
  return sdesc_sw128(smem_u32(tile) + (uint32_t)(kk * 2048), 16384, 1024);
}
__device__ __forceinline__ void rows_sync() { asm volatile("bar.sync 1, 128;\n" ::: "memory"); }
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

}  // namespace sc

using namespace sc;

__global__ void __launch_bounds__(kThreads, 1) score_stats_tc05_kernel(const __grid_constant__ ScoreTcBatch b) {
  extern __shared__ unsigned char smem_raw[];
  Smem1& sm = *reinterpret_cast<Smem1*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  const ScoreTcDesc& p = b.p[blockIdx.y];
  const int chunk = blockIdx.x;
  if (chunk >= p.n_chunks) return;
  const int64_t k0 = (int64_t)chunk * p.chunk_len;
  const int64_t k1 = (k0 + p.chunk_len < p.L_s) ? k0 + p.chunk_len : p.L_s;
  const int n_tiles = (int)((k1 - k0 + kTile - 1) / kTile);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(&sm.bar_q, 1);
    for (int i = 0; i < kStages1; ++i) {
      mbar_init(&sm.bar_k[i], 1);
      mbar_init(&sm.bar_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sm.bar_s[i], 1);
      mbar_init(&sm.bar_sfree[i], 128);
    }
    fence_mbar_init();
  }
  if (warp == 3) {
    tmem_alloc(&sm.tmem, 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tm = sm.tmem;

  if (warp == 2) {
    // ---- producer ----
    bool ok = true;
    int issued = 0;
    if (lane == 0) {
      mbar_expect_tx(&sm.bar_q, kTileBytes);
      tma_load_3d(sm.q, &p.q, &sm.bar_q, 0, 0, 0);
      tma_load_3d(sm.q + 16384, &p.q, &sm.bar_q, 64, 0, 0);
    }
    for (int j = 0; j < n_tiles; ++j) {
      const int st = j % kStages1;
      if (j >= kStages1 && !warp_wait(&sm.bar_empty[st], ((j / kStages1) - 1) & 1)) {
        ok = false;
        break;
      }
      if (lane == 0) {
        const int row = (int)(k0 + (int64_t)j * kTile);
        mbar_expect_tx(&sm.bar_k[st], kTileBytes);
        tma_load_3d(sm.k[st], &p.k, &sm.bar_k[st], 0, row, 0);
        tma_load_3d(sm.k[st] + 16384, &p.k, &sm.bar_k[st], 64, row, 0);
      }
      __syncwarp();
      issued = j + 1;
    }
    if (!ok) atomicOr(&g_score_error, 1u);
    if (lane == 0) {
      // loads still in flight when the consumers gave up must land before exit
      for (int j = issued - kStages1 < 0 ? 0 : issued - kStages1; j < issued; ++j)
        mbar_wait(&sm.bar_k[j % kStages1], (j / kStages1) & 1);
      mbar_wait(&sm.bar_q, 0);
    }
  } else if (warp == 3) {
    // ---- MMA issuer ----
    const uint32_t id_s = idesc_bf16_f32(128, 128, 0, 0);
    bool ok = warp_wait(&sm.bar_q, 0);
    int done = 0;
    for (int j = 0; j < n_tiles && ok; ++j) {
      const int st = j % kStages1, sb = j & 1;
      if (!warp_wait(&sm.bar_k[st], (j / kStages1) & 1)) { ok = false; break; }
      if (j >= 2 && !warp_wait(&sm.bar_sfree[sb], ((j >> 1) - 1) & 1)) { ok = false; break; }
      tc_fence_after();
      if (lane == 0) {
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_ss(tm + 128 * sb, kdesc(sm.q, kk), kdesc(sm.k[st], kk), id_s, kk > 0);
        umma_commit(&sm.bar_s[sb]);
        umma_commit(&sm.bar_empty[st]);
      }
      __syncwarp();
      done = j + 1;
    }
    if (!ok) atomicOr(&g_score_error, 2u);
    if (done > 0 && lane == 0) mbar_wait(&sm.bar_empty[(done - 1) % kStages1], ((done - 1) / kStages1) & 1);
  } else {
    // ---- rows: warps 0, 1 (columns 0-63) and 4, 5 (columns 64-127) ----
    const int r = 32 * (warp & 3) + lane;
    const int col0 = warp >= 4 ? 64 : 0;
    const uint32_t lane_off = (uint32_t)(32 * (warp & 3)) << 16;
    const float cs = b.scale * kLog2e;
    bool ok = true;
    float m = -INFINITY, l = 0.f;
    for (int j = 0; j < n_tiles && ok; ++j) {
      const int sb = j & 1;
      if (!warp_wait(&sm.bar_s[sb], (j >> 1) & 1)) { ok = false; break; }
      tc_fence_after();
      float s[64];
      tmem_ld32(tm + lane_off + 128 * sb + col0, reinterpret_cast<uint32_t*>(s));
      tmem_ld32(tm + lane_off + 128 * sb + col0 + 32, reinterpret_cast<uint32_t*>(s) + 32);
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(&sm.bar_sfree[sb]);  // S buffer read; the next S may overwrite it
      const int64_t t0 = k0 + (int64_t)j * kTile;
      const int nvalid = (int)((k1 - t0) < kTile ? (k1 - t0) : kTile) - col0;
      float mt = -INFINITY;
      if (nvalid >= 64) {
#pragma unroll
        for (int c = 0; c < 64; ++c) {
          s[c] *= cs;
          mt = fmaxf(mt, s[c]);
        }
      } else {
#pragma unroll
        for (int c = 0; c < 64; ++c) {
          s[c] = c < nvalid ? s[c] * cs : -INFINITY;
          mt = fmaxf(mt, s[c]);
        }
      }
      const float mn = fmaxf(m, mt);
      if (mn != -INFINITY) {
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int c = 0; c < 64; ++c) acc[c & 3] += fast_exp2(s[c] - mn);
        l = l * fast_exp2(m - mn) + ((acc[0] + acc[1]) + (acc[2] + acc[3]));
        m = mn;
      }
    }
    if (!ok) atomicOr(&g_score_error, 4u);
    // merge the two column halves of each row
    if (col0) {
      sm.xm[r] = m;
      sm.xl[r] = l;
    }
    rows_sync();
    if (!col0 && r < p.M) {
      const float m1 = sm.xm[r], l1 = sm.xl[r];
      const float mm = fmaxf(m, m1);
      float lt = 0.f;
      if (mm != -INFINITY) lt = (m != -INFINITY ? l * fast_exp2(m - mm) : 0.f) + (m1 != -INFINITY ? l1 * fast_exp2(m1 - mm) : 0.f);
      p.stats[((int64_t)chunk * p.M + r) * 2] = mm;
      p.stats[((int64_t)chunk * p.M + r) * 2 + 1] = lt;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 3) tmem_dealloc(tm, 256);
}

__global__ void __launch_bounds__(kThreads, 1) score_probs_tc05_kernel(const __grid_constant__ ScoreTcBatch b) {
  extern __shared__ unsigned char smem_raw[];
  Smem2& sm = *reinterpret_cast<Smem2*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  const ScoreTcDesc& p = b.p[blockIdx.y];
  const int chunk = blockIdx.x;
  if (chunk >= p.n_chunks) return;
  const int64_t k0 = (int64_t)chunk * p.chunk_len;
  const int64_t k1 = (k0 + p.chunk_len < p.L_s) ? k0 + p.chunk_len : p.L_s;
  const int n_tiles = (int)((k1 - k0 + kTile - 1) / kTile);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr uint32_t kColS = 0, kColY = 128;  // S^T double buffer [0, 128), Y^T [128, 192)

  if (threadIdx.x == 0) {
    mbar_init(&sm.bar_q, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sm.bar_k[i], 1);
      mbar_init(&sm.bar_v[i], 1);
      mbar_init(&sm.bar_empty[i], 1);
      mbar_init(&sm.bar_s[i], 1);
      mbar_init(&sm.bar_p[i], 128);
      mbar_init(&sm.bar_pfree[i], 1);
    }
    mbar_init(&sm.bar_y, 1);
    fence_mbar_init();
  }
  if (warp == 5) {
    tmem_alloc(&sm.tmem, 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tm = sm.tmem;

  if (warp == 4) {
    // ---- producer ----
    bool ok = true;
    int issued = 0;
    if (lane == 0) {
      mbar_expect_tx(&sm.bar_q, kTileBytes);
      tma_load_3d(sm.q, &p.q, &sm.bar_q, 0, 0, 0);
      tma_load_3d(sm.q + 16384, &p.q, &sm.bar_q, 64, 0, 0);
    }
    for (int j = 0; j < n_tiles; ++j) {
      const int st = j & 1;
      if (j >= 2 && !warp_wait(&sm.bar_empty[st], ((j >> 1) - 1) & 1)) {
        ok = false;
        break;
      }
      if (lane == 0) {
        const int row = (int)(k0 + (int64_t)j * kTile);
        mbar_expect_tx(&sm.bar_k[st], kTileBytes);
        tma_load_3d(sm.k[st], &p.k, &sm.bar_k[st], 0, row, 0);
        tma_load_3d(sm.k[st] + 16384, &p.k, &sm.bar_k[st], 64, row, 0);
        mbar_expect_tx(&sm.bar_v[st], kTileBytes);
        tma_load_3d(sm.v[st], &p.v, &sm.bar_v[st], 0, row, 0);
        tma_load_3d(sm.v[st] + 16384, &p.v, &sm.bar_v[st], 64, row, 0);
      }
      __syncwarp();
      issued = j + 1;
    }
    if (!ok) atomicOr(&g_score_error, 1u);
    if (lane == 0) {
      for (int j = issued - 2 < 0 ? 0 : issued - 2; j < issued; ++j) {
        mbar_wait(&sm.bar_k[j & 1], (j >> 1) & 1);
        mbar_wait(&sm.bar_v[j & 1], (j >> 1) & 1);
      }
      mbar_wait(&sm.bar_q, 0);
    }
  } else if (warp == 5) {
    // ---- MMA issuer: S^T(j), then Y^T += V^T P^T(j - 1) ----
    const uint32_t id_s = idesc_bf16_f32(128, 64, 0, 0);
    const uint32_t id_y = idesc_bf16_f32(128, 64, 1, 1);
    bool ok = warp_wait(&sm.bar_q, 0);
    int pv_done = 0;
    for (int j = 0; j <= n_tiles && ok; ++j) {
      if (j < n_tiles) {
        const int st = j & 1;
        // S^T buffer st was last read by the softmax of tile j - 2, whose
        // P-ready barrier this warp waited for before issuing PV(j - 2)
        if (!warp_wait(&sm.bar_k[st], (j >> 1) & 1)) { ok = false; break; }
        tc_fence_after();
        if (lane == 0) {
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            umma_ss(tm + kColS + 64 * st, kdesc(sm.k[st], kk), kdesc(sm.q, kk), id_s, kk > 0);
          umma_commit(&sm.bar_s[st]);
        }
        __syncwarp();
      }
      if (j >= 1) {
        const int t = j - 1, st = t & 1;
        const uint32_t ph = (t >> 1) & 1;
        if (!warp_wait(&sm.bar_v[st], ph)) { ok = false; break; }
        if (!warp_wait(&sm.bar_p[st], ph)) { ok = false; break; }
        tc_fence_after();
        if (lane == 0) {
#pragma unroll
          for (int part = 0; part < 2; ++part) {
            const unsigned char* pt = part ? sm.pl[st] : sm.ph[st];
#pragma unroll
            for (int kk = 0; kk < 8; ++kk)
              umma_ss(tm + kColY, mndesc(sm.v[st], kk), mndesc(pt, kk), id_y, (t > 0 || part > 0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(&sm.bar_pfree[st]);
          umma_commit(&sm.bar_empty[st]);
          if (t == n_tiles - 1) umma_commit(&sm.bar_y);
        }
        __syncwarp();
        pv_done = j;
      }
    }
    if (!ok) atomicOr(&g_score_error, 2u);
    if (pv_done > 0 && lane == 0) mbar_wait(&sm.bar_empty[(pv_done - 1) & 1], ((pv_done - 1) >> 1) & 1);
  } else {
    // ---- warps 0-3: thread t = key t of each tile (TMEM lane t), then head-dim row t of Y^T ----
    const int t = threadIdx.x;
    const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
    if (t < 64) {
      float mb = INFINITY;  // padding query rows get p = 2^-inf = 0
      if (t < p.M) {
        float m = -INFINITY, l = 0.f;
        for (int c = 0; c < p.n_chunks; ++c) m = fmaxf(m, p.stats[((int64_t)c * p.M + t) * 2]);
        for (int c = 0; c < p.n_chunks; ++c) {
          const float mc = p.stats[((int64_t)c * p.M + t) * 2];
          if (mc != -INFINITY) l += p.stats[((int64_t)c * p.M + t) * 2 + 1] * exp2f(mc - m);
        }
        mb = m + log2f(l);
        const float mc = p.stats[((int64_t)chunk * p.M + t) * 2];
        p.massp[(int64_t)chunk * p.M + t] =
            mc != -INFINITY ? p.stats[((int64_t)chunk * p.M + t) * 2 + 1] * exp2f(mc - m) / l : 0.f;
      }
      sm.mb[t] = mb;
    }
    rows_sync();
    float mbr[64];
#pragma unroll
    for (int a = 0; a < 64; ++a) mbr[a] = sm.mb[a];
    const float cs = b.scale * kLog2e;
    const float inv_m = 1.f / (float)p.M;
    const uint32_t row_off = (uint32_t)((t >> 3) * 1024 + (t & 7) * 128);
    bool ok = true;
    for (int j = 0; j < n_tiles; ++j) {
      const int sb = j & 1;
      if (!warp_wait(&sm.bar_s[sb], (j >> 1) & 1)) { ok = false; break; }
      if (j >= 2 && !warp_wait(&sm.bar_pfree[sb], ((j >> 1) - 1) & 1)) { ok = false; break; }
      tc_fence_after();
      float s[64];
      tmem_ld32(tm + lane_off + kColS + 64 * sb, reinterpret_cast<uint32_t*>(s));
      tmem_ld32(tm + lane_off + kColS + 64 * sb + 32, reinterpret_cast<uint32_t*>(s) + 32);
      tmem_wait_ld();
      const int64_t key = k0 + (int64_t)j * kTile + t;
      const bool valid = key < k1;
      const uint32_t hi_base = smem_u32(sm.ph[sb]) + row_off, lo_base = smem_u32(sm.pl[sb]) + row_off;
      float acc[2] = {0.f, 0.f};
#pragma unroll
      for (int c = 0; c < 8; ++c) {  // 16-byte chunk c: queries 8c .. 8c + 7
        uint32_t hi[4], lo[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int a = 8 * c + 2 * i;
          const float p0 = valid ? fast_exp2(fmaf(s[a], cs, -mbr[a])) : 0.f;
          const float p1 = valid ? fast_exp2(fmaf(s[a + 1], cs, -mbr[a + 1])) : 0.f;
          acc[0] = fmaf(p0, p0, acc[0]);
          acc[1] = fmaf(p1, p1, acc[1]);
          __nv_bfloat162 h2 = __floats2bfloat162_rn(p0, p1);
          const float2 hf = __bfloat1622float2(h2);
          __nv_bfloat162 l2 = __floats2bfloat162_rn(p0 - hf.x, p1 - hf.y);
          hi[i] = *reinterpret_cast<uint32_t*>(&h2);
          lo[i] = *reinterpret_cast<uint32_t*>(&l2);
        }
        const uint32_t off = (uint32_t)((c ^ (t & 7)) << 4);  // 128-byte swizzle
        st_shared_v4(hi_base + off, hi[0], hi[1], hi[2], hi[3]);
        st_shared_v4(lo_base + off, lo[0], lo[1], lo[2], lo[3]);
      }
      if (valid) p.u[key] = sqrtf((acc[0] + acc[1]) * inv_m);  // sqrt(sum / M), key_selection.py:26
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&sm.bar_p[sb]);
    }
    if (!ok) atomicOr(&g_score_error, 4u);
    const bool have = ok && n_tiles > 0 && warp_wait(&sm.bar_y, 0);
    if (!have && n_tiles > 0) atomicOr(&g_score_error, 8u);
    tc_fence_after();
    // Y^T: thread t holds head-dim row t for the 64 query columns
#pragma unroll 1
    for (int c = 0; c < 2; ++c) {
      uint32_t r[32];
      tmem_ld32(tm + lane_off + kColY + 32 * c, r);
      tmem_wait_ld();
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const int a = 32 * c + i;
        if (a < p.M) p.yp[((int64_t)chunk * p.M + a) * 128 + t] = have ? __uint_as_float(r[i]) : 0.f;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 5) tmem_dealloc(tm, 256);
}

static size_t score_stats_smem() { return sizeof(Smem1) + 1024; }
static size_t score_probs_smem() { return sizeof(Smem2) + 1024; }

bool scoring_tc05_supported(const BuildBatch<float>& b, const BuildParams& prm) {
  if (prm.d != 128 || prm.dv != 128) return false;
  for (int i = 0; i < b.n; ++i) {
    const BuildDesc<float>& p = b.p[i];
    if (p.M > 64 || p.ld_k % 8 || p.ld_v % 8 || (reinterpret_cast<uintptr_t>(p.keys) & 15) ||
        (reinterpret_cast<uintptr_t>(p.values) & 15) || (reinterpret_cast<uintptr_t>(p.repr) & 15) ||
        p.L_s > 0x7fffffff)
      return false;
  }
  return true;
}

int launch_scoring_tc05(const BuildBatch<float>& bb, const BuildParams& prm, int max_chunks, cudaStream_t st) {
  auto k1 = score_stats_tc05_kernel;
  auto k2 = score_probs_tc05_kernel;
  DCC_CHECK(check_cuda(cudaFuncSetAttribute(k1, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)score_stats_smem()),
                       "score_stats_tc05 smem"));
  DCC_CHECK(check_cuda(cudaFuncSetAttribute(k2, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)score_probs_smem()),
                       "score_probs_tc05 smem"));
  std::unique_ptr<ScoreTcBatch> own(new ScoreTcBatch());
  ScoreTcBatch& b = *own;
  b.scale = (float)prm.scale;
  for (int i0 = 0; i0 < bb.n; i0 += kScoreTcCap) {
    b.n = 0;
    int mc = 0;
    for (int i = i0; i < bb.n && b.n < kScoreTcCap; ++i) {
      const BuildDesc<float>& p = bb.p[i];
      ScoreTcDesc& t = b.p[b.n++];
      t = ScoreTcDesc{};
      DCC_CHECK(make_tmap_bf16_3d(&t.k, p.keys, 128, p.L_s, 1, p.ld_k, p.ld_k * p.L_s, 128));
      DCC_CHECK(make_tmap_bf16_3d(&t.v, p.values, 128, p.L_s, 1, p.ld_v, p.ld_v * p.L_s, 128));
      DCC_CHECK(make_tmap_bf16_3d(&t.q, p.repr, 128, p.M, 1, 128, 128 * p.M, 128));
      t.L_s = p.L_s;
      t.M = p.M;
      t.n_chunks = p.n_chunks;
      t.chunk_len = p.chunk_len;
      t.stats = p.stats;
      t.massp = p.massp;
      t.yp = p.yp;
      t.u = p.u;
      if (p.n_chunks > mc) mc = p.n_chunks;
    }
    dim3 grid(mc, b.n);
    k1<<<grid, kThreads, score_stats_smem(), st>>>(b);
    DCC_CHECK(check_launch("score_stats_tc05"));
    k2<<<grid, kThreads, score_probs_smem(), st>>>(b);
    DCC_CHECK(check_launch("score_probs_tc05"));
  }
  (void)max_chunks;
  return DCC_OK;
}

// Device address of the scoring passes' bounded-wait error word on the
// current device (the symbol lives in this translation unit).
int score_error_flag_address(unsigned int** out) {
  return check_cuda(cudaGetSymbolAddress(reinterpret_cast<void**>(out), g_score_error),
                    "device_error_flags_async: scoring flag address");
}

}  // namespace dcc

extern "C" int dcc_build_error_status(int clear) {
  using namespace dcc;
  DCC_CHECK(check_cuda(cudaDeviceSynchronize(), "build_error_status: synchronize"));
  unsigned int v = 0;
  DCC_CHECK(check_cuda(cudaMemcpyFromSymbol(&v, g_score_error, sizeof(v)), "build_error_status: read"));
  if (clear && v) {
    unsigned int z = 0;
    DCC_CHECK(check_cuda(cudaMemcpyToSymbol(g_score_error, &z, sizeof(z)), "build_error_status: clear"));
  }
  if (v) return fail(DCC_ERR_TIMEOUT, "scoring: a bounded device wait expired (flags " + std::to_string(v) + ")");
  return DCC_OK;
}
