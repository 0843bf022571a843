// Scoring passes of the compact-KV build for bf16 inputs on the tcgen05
// tensor cores (head_dim = value_dim = 128, M <= 64 representative queries).
//
// Same outputs as scoring.cu (per key chunk: row max / sum of exp; then RMS
// scores u, block mass and Y = A V partials), computed as
//   S = Q^ K^T      M=128 (the M query rows, zero-padded), N=128 keys, SS MMA
//   P = exp(S*scale - m) / l                 fp32, one thread per query row
//   Y += P V        TS MMA with P split into bf16 hi + lo parts (P = hi + lo
//                   to 16 mantissa bits), so Y keeps ~1e-5 relative accuracy
//   u_j = sqrt(sum_a P_aj^2 / M)             column sums through shared memory
// CTA: warps 0-3 rows / columns (rows >= 64 are padding), warp 4 TMA
// producer, warp 5 TMEM owner + MMA issuer.  TMEM: S double buffer
// [0,256), Y [256,384).  All waits are bounded and warp-uniform; every
// tcgen05 ld/st runs on whole warps.
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
  float* stats;    // [n_chunks, M, 2]
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
constexpr uint32_t kColS = 0, kColY = 256;

struct Smem {
  unsigned char q[kTileBytes];
  unsigned char k[2][kTileBytes];
  unsigned char v[2][kTileBytes];
  float tb[64][kTile + 1];  // p^2 rows, read back by columns
  uint64_t bar_q, bar_k[2], bar_v[2], bar_empty[2], bar_s[2], bar_sfree[2], bar_p[2], bar_y;
  uint32_t tmem;
};

__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity) {
  return __all_sync(0xffffffffu, mbar_wait(bar, parity)) != 0;
}
__device__ __forceinline__ uint64_t kdesc(const unsigned char* tile, int kk) {
  return sdesc_sw128(smem_u32(tile) + (uint32_t)((kk >> 2) * 16384 + (kk & 3) * 32), 16, 1024);
}
__device__ __forceinline__ uint64_t vdesc(const unsigned char* tile, int kk) {
  return sdesc_sw128(smem_u32(tile) + (uint32_t)(kk * 2048), 16384, 1024);
}
__device__ __forceinline__ void rows_sync() { asm volatile("bar.sync 1, 128;\n" ::: "memory"); }

}  // namespace sc

using namespace sc;

template <bool PASS2>
__global__ void __launch_bounds__(kThreads, 1) score_tc05_kernel(const __grid_constant__ ScoreTcBatch b) {
  extern __shared__ unsigned char smem_raw[];
  Smem& sm = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  const ScoreTcDesc& p = b.p[blockIdx.y];
  const int chunk = blockIdx.x;
  if (chunk >= p.n_chunks) return;
  const int64_t k0 = (int64_t)chunk * p.chunk_len;
  const int64_t k1 = (k0 + p.chunk_len < p.L_s) ? k0 + p.chunk_len : p.L_s;
  const int n_tiles = (int)((k1 - k0 + kTile - 1) / kTile);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(&sm.bar_q, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sm.bar_k[i], 1);
      mbar_init(&sm.bar_v[i], 1);
      mbar_init(&sm.bar_empty[i], 1);
      mbar_init(&sm.bar_s[i], 1);
      mbar_init(&sm.bar_sfree[i], PASS2 ? 1 : 64);
      mbar_init(&sm.bar_p[i], 64);
    }
    mbar_init(&sm.bar_y, 1);
    fence_mbar_init();
  }
  if (warp == 5) {
    tmem_alloc(&sm.tmem, 512);
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
        if (PASS2) {
          mbar_expect_tx(&sm.bar_v[st], kTileBytes);
          tma_load_3d(sm.v[st], &p.v, &sm.bar_v[st], 0, row, 0);
          tma_load_3d(sm.v[st] + 16384, &p.v, &sm.bar_v[st], 64, row, 0);
        }
      }
      __syncwarp();
      issued = j + 1;
    }
    if (!ok) atomicOr(&g_score_error, 1u);
    if (lane == 0) {
      for (int j = issued - 2 < 0 ? 0 : issued - 2; j < issued; ++j) {
        mbar_wait(&sm.bar_k[j & 1], (j >> 1) & 1);
        if (PASS2) mbar_wait(&sm.bar_v[j & 1], (j >> 1) & 1);
      }
      mbar_wait(&sm.bar_q, 0);
    }
  } else if (warp == 5) {
    // ---- MMA issuer ----
    const uint32_t id_s = idesc_bf16_f32(128, 128, 0, 0);
    const uint32_t id_pv = idesc_bf16_f32(128, 128, 0, 1);
    bool ok = warp_wait(&sm.bar_q, 0);
    int done = 0;
    for (int j = 0; j < n_tiles && ok; ++j) {
      const int st = j & 1, sb = j & 1;
      const uint32_t ph = (j >> 1) & 1;
      if (!warp_wait(&sm.bar_k[st], ph)) { ok = false; break; }
      if (j >= 2 && !warp_wait(&sm.bar_sfree[sb], ((j >> 1) - 1) & 1)) { ok = false; break; }
      tc_fence_after();
      const uint32_t s_col = kColS + 128 * sb;
      if (lane == 0) {
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) umma_ss(tm + s_col, kdesc(sm.q, kk), kdesc(sm.k[st], kk), id_s, kk > 0);
        umma_commit(&sm.bar_s[sb]);
        if (!PASS2) umma_commit(&sm.bar_empty[st]);
      }
      __syncwarp();
      if (PASS2) {
        if (!warp_wait(&sm.bar_v[st], ph)) { ok = false; break; }
        if (!warp_wait(&sm.bar_p[sb], ph)) { ok = false; break; }
        tc_fence_after();
        if (lane == 0) {
#pragma unroll
          for (int half = 0; half < 2; ++half)
#pragma unroll
            for (int kk = 0; kk < 8; ++kk)
              umma_ts(tm + kColY, tm + s_col + 64 * half + kk * 8, vdesc(sm.v[st], kk), id_pv,
                      (j > 0 || half > 0 || kk > 0) ? 1u : 0u);
          umma_commit(&sm.bar_sfree[sb]);
          umma_commit(&sm.bar_empty[st]);
          if (j == n_tiles - 1) umma_commit(&sm.bar_y);
        }
        __syncwarp();
      }
      done = j + 1;
    }
    if (!ok) atomicOr(&g_score_error, 2u);
    if (done > 0 && lane == 0) mbar_wait(&sm.bar_empty[(done - 1) & 1], ((done - 1) >> 1) & 1);
  } else {
    // ---- rows (warps 0-1: query a = thread) and columns (warps 0-3: key = thread) ----
    const bool row_warp = warp < 2;
    const int a = warp * 32 + lane;
    const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
    bool ok = true;
    float m = -INFINITY, l = 0.f, mass = 0.f, inv_l = 0.f;
    if (PASS2 && row_warp && a < p.M) {
      for (int c = 0; c < p.n_chunks; ++c) m = fmaxf(m, p.stats[((int64_t)c * p.M + a) * 2]);
      for (int c = 0; c < p.n_chunks; ++c) {
        const float mc = p.stats[((int64_t)c * p.M + a) * 2];
        if (mc != -INFINITY) l += p.stats[((int64_t)c * p.M + a) * 2 + 1] * expf(mc - m);
      }
      inv_l = 1.f / l;
    }
    for (int j = 0; j < n_tiles; ++j) {
      const int sb = j & 1;
      const uint32_t ph = (j >> 1) & 1;
      const int64_t t0 = k0 + (int64_t)j * kTile;
      const int nvalid = (int)((k1 - t0) < kTile ? (k1 - t0) : kTile);
      const uint32_t s_col = kColS + 128 * sb;
      if (row_warp) {
        if (!warp_wait(&sm.bar_s[sb], ph)) { ok = false; }
        if (ok) {
          tc_fence_after();
          float s[128];
#pragma unroll
          for (int c = 0; c < 4; ++c) tmem_ld32(tm + lane_off + s_col + 32 * c, reinterpret_cast<uint32_t*>(s) + 32 * c);
          tmem_wait_ld();
          if (!PASS2) {
            tc_fence_before();
            mbar_arrive(&sm.bar_sfree[sb]);  // S buffer read; the next S may overwrite it
            float mt = -INFINITY;
#pragma unroll
            for (int c = 0; c < 128; ++c) {
              s[c] = c < nvalid ? s[c] * b.scale : -INFINITY;
              mt = fmaxf(mt, s[c]);
            }
            const float mn = fmaxf(m, mt);
            if (mn != -INFINITY) {
              float acc = 0.f;
#pragma unroll
              for (int c = 0; c < 128; ++c) acc += expf(s[c] - mn);
              l = l * expf(m - mn) + acc;
              m = mn;
            }
          } else {
            float* trow = sm.tb[a & 63];
#pragma unroll
            for (int c4 = 0; c4 < 4; ++c4) {
              uint32_t hi[16], lo[16];
#pragma unroll
              for (int i = 0; i < 16; ++i) {
                float pr[2];
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                  const int c = 32 * c4 + 2 * i + e;
                  pr[e] = (c < nvalid && a < p.M) ? expf(s[c] * b.scale - m) * inv_l : 0.f;
                  mass += pr[e];
                  trow[c] = pr[e] * pr[e];
                }
                __nv_bfloat162 h2 = __floats2bfloat162_rn(pr[0], pr[1]);
                const float2 hf = __bfloat1622float2(h2);
                __nv_bfloat162 l2 = __floats2bfloat162_rn(pr[0] - hf.x, pr[1] - hf.y);
                hi[i] = *reinterpret_cast<uint32_t*>(&h2);
                lo[i] = *reinterpret_cast<uint32_t*>(&l2);
              }
              tmem_st16(tm + lane_off + s_col + 16 * c4, hi);
              tmem_st16(tm + lane_off + s_col + 64 + 16 * c4, lo);
            }
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(&sm.bar_p[sb]);
          }
        }
      }
      if (PASS2) {
        // every warp of the row group reaches both barriers each tile, timeouts included
        rows_sync();
        const int t = threadIdx.x;  // key of the tile
        if (t < nvalid) {
          float acc = 0.f;
          for (int r = 0; r < p.M; ++r) acc += sm.tb[r][t];
          p.u[t0 + t] = sqrtf(acc / (float)p.M);  // sqrt(sum / M), key_selection.py:26
        }
        rows_sync();
      }
      if (!__all_sync(0xffffffffu, ok)) ok = false;
    }
    if (!ok) atomicOr(&g_score_error, 4u);
    if (row_warp) {
      if (!PASS2) {
        if (a < p.M) {
          p.stats[((int64_t)chunk * p.M + a) * 2] = m;
          p.stats[((int64_t)chunk * p.M + a) * 2 + 1] = l;
        }
      } else {
        const bool have = ok && n_tiles > 0 && warp_wait(&sm.bar_y, 0);
        if (!have && n_tiles > 0) atomicOr(&g_score_error, 8u);
        tc_fence_after();
        float* yrow = p.yp + ((int64_t)chunk * p.M + (a < p.M ? a : 0)) * 128;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t r[32];
          if (n_tiles > 0) {
            tmem_ld32(tm + lane_off + kColY + 32 * c, r);
            tmem_wait_ld();
          }
          if (a < p.M) {
#pragma unroll
            for (int i = 0; i < 32; ++i) yrow[32 * c + i] = (have ? __uint_as_float(r[i]) : 0.f);
          }
        }
        if (a < p.M) p.massp[(int64_t)chunk * p.M + a] = mass;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 5) tmem_dealloc(tm, 512);
}

static size_t score_tc05_smem() { return sizeof(Smem) + 1024; }

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
  auto k1 = score_tc05_kernel<false>;
  auto k2 = score_tc05_kernel<true>;
  DCC_CHECK(check_cuda(cudaFuncSetAttribute(k1, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)score_tc05_smem()),
                       "score_tc05 smem"));
  DCC_CHECK(check_cuda(cudaFuncSetAttribute(k2, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)score_tc05_smem()),
                       "score_tc05 smem"));
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
    k1<<<grid, kThreads, score_tc05_smem(), st>>>(b);
    DCC_CHECK(check_launch("score_tc05 pass 1"));
    k2<<<grid, kThreads, score_tc05_smem(), st>>>(b);
    DCC_CHECK(check_launch("score_tc05 pass 2"));
  }
  (void)max_chunks;
  return DCC_OK;
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
