// bf16 attention over KV segments with per-key logit bias on the 5th-gen
// tensor cores (tcgen05 + TMEM + TMA), head_dim 128.
//
// One CTA = 128 query rows of two query heads that share a KV head (GQA), so
// every K/V tile is loaded once for 256 rows.  Warp roles (384 threads):
//   warps 0-3  softmax for head A (thread = query row = TMEM lane)
//   warps 4-7  softmax for head B
//   warp  8    TMA producer (Q once; K, V tiles of 128 keys, 2-stage ring;
//              the per-key bias tile through shared memory)
//   warp  9    TMEM owner and MMA issuer (one elected thread)
//   warps 10-11 idle
// Registers: launched at 168 per thread (3 warps per SM sub-partition), the
// third warpgroup hands registers to the softmax warpgroups with setmaxnreg:
// 2 x 128 x 216 + 128 x 64 = 63488 <= 384 x 168 = 64512.
// TMEM (512 columns): O_A [0,128) O_B [128,256) S_A [256,384) S_B [384,512);
// P (bf16, two per column) overwrites the first 64 columns of its S.
// Per KV tile j:  S_A = Q_A K_j^T, S_B = Q_B K_j^T      (SS MMA, K-major)
//                 softmax A/B: S -> P in TMEM (base-2, lazily rescaled max)
//                 O_A += P_A V_j, O_B += P_B V_j        (TS MMA, V MN-major)
// so softmax of one head overlaps the MMAs of the other.  The running max is
// only moved (and O rescaled in TMEM) when it grows by more than 2^8, so P
// stays below 256 and the rescale is rare.
//
// Every mbarrier wait is bounded (2 s); a timeout sets g_attn_error, the
// roles unwind, in-flight copies and MMAs are waited for, TMEM is freed.
#include <memory>
#include <mutex>
#include <string>

#include "attention.cuh"
#include "tc05.cuh"

namespace dcc {

using namespace tc05;

constexpr int kTcMaxSeg = 8;
constexpr int kTcCap = 8;

struct Tc05Seg {
  CUtensorMap k;  // {128, len, n_kv_heads}, box {64, 128, 1}, 128B swizzle
  CUtensorMap v;
  const float* bias;
  int64_t bias_head_stride;
  int64_t len;
};

struct Tc05Problem {
  CUtensorMap q;  // {128, Lq, n_q_heads}
  void* o;
  float* lse;
  int64_t o_head_stride, o_row_stride, lse_head_stride;
  int64_t Lq;
  int32_t n_seg, causal;
  int64_t causal_offset;
  const void* o_init;  // optional initial state (o's strides), may alias o
  const float* lse_init;
  int64_t lse_init_head_stride;
  Tc05Seg seg[kTcMaxSeg];
};

struct Tc05Batch {
  int n;
  int group;   // query heads per KV head
  float scale_log2;
  Tc05Problem p[kTcCap];
};

static __device__ unsigned int g_attn_error;

namespace fa {

constexpr int kRows = 128;       // query rows per head tile
constexpr int kKeys = 128;       // keys per KV tile
constexpr int kTileBytes = 32768;  // [128 rows x 128 bf16] as two 16 KB 128B-swizzled column blocks
constexpr int kThreads = 384;
constexpr int kRegsLaunch = 168, kRegsSoftmax = 216, kRegsOther = 64;
static_assert(2 * 128 * kRegsSoftmax + 128 * kRegsOther <= kThreads * kRegsLaunch, "register split");
constexpr uint32_t kColOA = 0, kColOB = 128, kColSA = 256, kColSB = 384;

struct Smem {
  unsigned char q[2][kTileBytes];    // head A, head B
  unsigned char k[2][kTileBytes];    // stages
  unsigned char v[2][kTileBytes];
  __align__(16) float bias[2][kKeys];
  uint64_t bar_q, bar_k[2], bar_v[2], bar_bias[2], bar_empty[2], bar_s[2], bar_p[2], bar_o[2];
  uint32_t tmem;
};

struct Tile {
  int seg;
  int64_t t0;
  int64_t kend;
};

// The j-th KV tile of this CTA (segments in order, 128 keys per tile).
__device__ __forceinline__ Tile tile_at(const Tc05Problem& p, const int64_t* kend, int j) {
  for (int s = 0; s < p.n_seg; ++s) {
    const int nt = (int)((kend[s] + kKeys - 1) / kKeys);
    if (j < nt) return Tile{s, (int64_t)j * kKeys, kend[s]};
    j -= nt;
  }
  return Tile{0, 0, 0};
}

__device__ __forceinline__ uint64_t kdesc(const unsigned char* tile, int kk) {
  // K-major operand: 16-column step kk inside column block kk / 4
  return sdesc_sw128(smem_u32(tile) + (uint32_t)((kk >> 2) * 16384 + (kk & 3) * 32), 16, 1024);
}
__device__ __forceinline__ uint64_t vdesc(const unsigned char* tile, int kk) {
  // MN-major operand: 16 keys (rows) per step, the two 64-column blocks 16 KB apart
  return sdesc_sw128(smem_u32(tile) + (uint32_t)(kk * 2048), 16384, 1024);
}

// Every lane waits; the warp agrees on the outcome, so no lane runs ahead into a
// warp-collective tcgen05 instruction while another has given up.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity) {
  return __all_sync(0xffffffffu, mbar_wait(bar, parity)) != 0;
}
__device__ __forceinline__ bool warp_wait_limited(uint64_t* bar, uint32_t parity, uint64_t limit_ns) {
  return __all_sync(0xffffffffu, mbar_wait(bar, parity, limit_ns)) != 0;
}

// 2^x on the SFU (ex2.approx.ftz: ~2 ulp, 2^-inf = 0).
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

}  // namespace fa

using namespace fa;

// ---- TMA producer (warp 8) --------------------------------------------------------
__device__ __forceinline__ void producer_role(const Tc05Problem& p, Smem& sm, const int64_t* kend, int n_tiles,
                                              int64_t q0, int hA, int hB, int hk, int lane) {
  bool ok = true;
  if (lane == 0) {
    prefetch_tmap(&p.q);
    mbar_expect_tx(&sm.bar_q, 2 * kTileBytes);
    tma_load_3d(sm.q[0], &p.q, &sm.bar_q, 0, (int)q0, hA);
    tma_load_3d(sm.q[0] + 16384, &p.q, &sm.bar_q, 64, (int)q0, hA);
    tma_load_3d(sm.q[1], &p.q, &sm.bar_q, 0, (int)q0, hB);
    tma_load_3d(sm.q[1] + 16384, &p.q, &sm.bar_q, 64, (int)q0, hB);
  }
  int issued = 0;
  for (int j = 0; j < n_tiles; ++j) {
    const int st = j & 1;
    if (j >= 2 && !warp_wait(&sm.bar_empty[st], ((j >> 1) - 1) & 1)) {
      ok = false;
      break;
    }
    const Tile t = tile_at(p, kend, j);
    const Tc05Seg& sg = p.seg[t.seg];
    if (lane == 0) {
      mbar_expect_tx(&sm.bar_k[st], kTileBytes);
      tma_load_3d(sm.k[st], &sg.k, &sm.bar_k[st], 0, (int)t.t0, hk);
      tma_load_3d(sm.k[st] + 16384, &sg.k, &sm.bar_k[st], 64, (int)t.t0, hk);
      mbar_expect_tx(&sm.bar_v[st], kTileBytes);
      tma_load_3d(sm.v[st], &sg.v, &sm.bar_v[st], 0, (int)t.t0, hk);
      tma_load_3d(sm.v[st] + 16384, &sg.v, &sm.bar_v[st], 64, (int)t.t0, hk);
    }
    const float* bg = sg.bias ? sg.bias + hk * sg.bias_head_stride : nullptr;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int c = lane * 4 + i;
      const int64_t key = t.t0 + c;
      sm.bias[st][c] = (bg && key < t.kend) ? __ldg(bg + key) * 1.4426950408889634f : 0.f;  // log2 units
    }
    mbar_arrive(&sm.bar_bias[st]);
    issued = j + 1;
  }
  if (!ok) atomicOr(&g_attn_error, 1u);
  // copies still in flight land before the CTA can exit
  if (lane == 0) {
    for (int j = issued - 2 < 0 ? 0 : issued - 2; j < issued; ++j) {
      mbar_wait(&sm.bar_k[j & 1], (j >> 1) & 1);
      mbar_wait(&sm.bar_v[j & 1], (j >> 1) & 1);
    }
    mbar_wait(&sm.bar_q, 0);
  }
}

// ---- MMA issuer (warp 9) -----------------------------------------------------------
// Issue order per tile j:  PV_A(j), S_A(j+1), PV_B(j), S_B(j+1)  (S_A(0), S_B(0) first),
// so head A's next scores are ready while head B's softmax still runs.  S(j+1)
// overwrites P(j) in TMEM only after PV(j), issued earlier from this thread.
template <bool kInit>
__device__ __forceinline__ void mma_role(Smem& sm, int n_tiles, uint32_t tm, int lane) {
  const uint32_t id_s = idesc_bf16_f32(128, 128, 0, 0);
  const uint32_t id_pv = idesc_bf16_f32(128, 128, 0, 1);
  bool ok = warp_wait(&sm.bar_q, 0);
  int done = 0;
  auto issue_s = [&](int h, int st) {
    if (lane == 0) {
      const uint32_t s_col = h ? kColSB : kColSA;
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) umma_ss(tm + s_col, kdesc(sm.q[h], kk), kdesc(sm.k[st], kk), id_s, kk > 0);
      umma_commit(&sm.bar_s[h]);
    }
    __syncwarp();
  };
  auto issue_pv = [&](int h, int st, int j) {
    if (lane == 0) {
      const uint32_t o_col = h ? kColOB : kColOA, p_col = h ? kColSB : kColSA;
#pragma unroll
      for (int kk = 0; kk < 8; ++kk)
        umma_ts(tm + o_col, tm + p_col + kk * 8, vdesc(sm.v[st], kk), id_pv, (kInit || j > 0 || kk > 0) ? 1u : 0u);
      umma_commit(&sm.bar_o[h]);
    }
    __syncwarp();
  };
  if (ok && n_tiles > 0) {
    ok = warp_wait(&sm.bar_k[0], 0);
    if (ok) {
      tc_fence_after();
      issue_s(0, 0);
      issue_s(1, 0);
    }
  }
  for (int j = 0; j < n_tiles && ok; ++j) {
    const int st = j & 1, st1 = (j + 1) & 1;
    const bool more = j + 1 < n_tiles;
    if (!warp_wait(&sm.bar_v[st], (j >> 1) & 1) || !warp_wait(&sm.bar_p[0], j & 1)) {
      ok = false;
      break;
    }
    tc_fence_after();
    issue_pv(0, st, j);
    if (more) {
      if (!warp_wait(&sm.bar_k[st1], ((j + 1) >> 1) & 1)) {
        ok = false;
        break;
      }
      tc_fence_after();
      issue_s(0, st1);
    }
    if (!warp_wait(&sm.bar_p[1], j & 1)) {
      ok = false;
      break;
    }
    tc_fence_after();
    issue_pv(1, st, j);
    if (lane == 0) umma_commit(&sm.bar_empty[st]);
    __syncwarp();
    if (more) issue_s(1, st1);
    done = j + 1;
  }
  if (!ok) atomicOr(&g_attn_error, 2u);
  // every MMA issued so far has finished before TMEM can be released
  if (done > 0 && lane == 0) mbar_wait(&sm.bar_empty[(done - 1) & 1], ((done - 1) >> 1) & 1);
}

// ---- softmax + epilogue (warps 0-3: head A, 4-7: head B) ------------------------
template <bool kInit>
__device__ __forceinline__ void softmax_role(const Tc05Batch& b, const Tc05Problem& p, Smem& sm,
                                             const int64_t* kend, int n_tiles, int64_t q0, int hA, int hB,
                                             uint32_t tm, int warp, int lane) {
  const int role = warp >> 2;
  const int row = (warp & 3) * 32 + lane;
  const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
  const uint32_t s_col = role ? kColSB : kColSA, o_col = role ? kColOB : kColOA;
  const int64_t q_row = q0 + row;
  float m_use = -INFINITY, l = 0.f;
  bool ok = true;
  // Optional initial state (m = lse_init, l = 1, O = o_init): O goes to TMEM
  // before the first P hand-off (whose tcgen05.wait::st covers these stores);
  // rows past Lq or without keys so far start empty.
  if (kInit) {
    const int h = role ? hB : hA;
    const bool real = q_row < p.Lq;
    const float lse0 = real ? p.lse_init[h * p.lse_init_head_stride + q_row] : -INFINITY;
    const bool have = lse0 > -INFINITY;
    if (have) {
      m_use = lse0 * 1.4426950408889634f;
      l = 1.f;
    }
    const uint4* oi = reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(p.o_init) +
                                                     h * p.o_head_stride + (real ? q_row : 0) * p.o_row_stride);
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {
      uint32_t r[32];
#pragma unroll
      for (int v = 0; v < 4; ++v) {
        const uint4 w = have ? oi[4 * c + v] : make_uint4(0u, 0u, 0u, 0u);
        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {  // bf16 pair -> two fp32 (a bf16 is the top half of its fp32)
          r[8 * v + 2 * i] = ws[i] << 16;
          r[8 * v + 2 * i + 1] = ws[i] & 0xffff0000u;
        }
      }
      tmem_st32(tm + lane_off + o_col + 32 * c, r);
    }
    tmem_wait_st();
  }
  for (int j = 0; j < n_tiles; ++j) {
    const int st = j & 1;
    const Tile t = tile_at(p, kend, j);
    const int64_t t_end = t.kend;
    const bool causal = p.causal && t.seg == 0;
    if (!warp_wait(&sm.bar_s[role], j & 1)) {
      ok = false;
      break;
    }
    tc_fence_after();
    float s[128];
#pragma unroll
    for (int c = 0; c < 4; ++c) tmem_ld32(tm + lane_off + s_col + 32 * c, reinterpret_cast<uint32_t*>(s) + 32 * c);
    tmem_wait_ld();
    if (!warp_wait(&sm.bar_bias[st], (j >> 1) & 1)) {
      ok = false;
      break;
    }
    // visible keys of this row in the tile: [t0, t0 + nvis)
    const int64_t lim = causal ? q_row + p.causal_offset : t_end - 1;  // last visible key
    const int64_t lim2 = lim < t_end - 1 ? lim : t_end - 1;
    const int nvis = (int)(lim2 - t.t0 + 1 < 0 ? 0 : (lim2 - t.t0 + 1 > 128 ? 128 : lim2 - t.t0 + 1));
    const bool full = __all_sync(0xffffffffu, nvis == 128) != 0;
    const bool biased = p.seg[t.seg].bias != nullptr;
    const bool plain = full && !biased;
    // row max over 8 independent chains (a single 128-long chain stalls on latency)
    float mx[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) mx[i] = -INFINITY;
    if (plain) {
      // whole tile visible, no bias: max of the raw scores, scaled once
#pragma unroll
      for (int c = 0; c < 128; ++c) mx[c & 7] = fmaxf(mx[c & 7], s[c]);
    } else if (full) {
      // whole tile visible with a per-key bias (log2 units, 16-byte shared loads)
      const float4* bv = reinterpret_cast<const float4*>(sm.bias[st]);
#pragma unroll
      for (int c4 = 0; c4 < 32; ++c4) {
        const float4 bb = bv[c4];
        s[4 * c4 + 0] = fmaf(s[4 * c4 + 0], b.scale_log2, bb.x);
        s[4 * c4 + 1] = fmaf(s[4 * c4 + 1], b.scale_log2, bb.y);
        s[4 * c4 + 2] = fmaf(s[4 * c4 + 2], b.scale_log2, bb.z);
        s[4 * c4 + 3] = fmaf(s[4 * c4 + 3], b.scale_log2, bb.w);
      }
#pragma unroll
      for (int c = 0; c < 128; ++c) mx[c & 7] = fmaxf(mx[c & 7], s[c]);
    } else {
#pragma unroll
      for (int c = 0; c < 128; ++c) {
        s[c] = c < nvis ? fmaf(s[c], b.scale_log2, sm.bias[st][c]) : -INFINITY;
        mx[c & 7] = fmaxf(mx[c & 7], s[c]);
      }
    }
    float mt = fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])), fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7])));
    if (plain) mt *= b.scale_log2;
    // Move the running max when it grows by more than 2^8 (always on the first
    // visible tile).  tcgen05.ld/st are warp-collective, so the O rescale runs
    // for the whole warp when any of its rows needs it (others scale by 1).
    const bool need = mt > m_use + 8.f;
    if (__any_sync(0xffffffffu, need)) {
      const float corr = !need ? 1.f : (m_use == -INFINITY ? 0.f : exp2f(m_use - mt));
      if (j > 0 || kInit) {
        if (j > 0 && !warp_wait(&sm.bar_o[role], (j - 1) & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t r[32];
          tmem_ld32(tm + lane_off + o_col + 32 * c, r);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * corr);
          tmem_st32(tm + lane_off + o_col + 32 * c, r);
        }
      }
      if (need) {
        l *= corr;
        m_use = mt;
      }
    }
    const float msub = m_use == -INFINITY ? 0.f : m_use;
    // p = 2^(x - m): one FFMA into the exponent for plain tiles, one FADD otherwise
    const float sa = plain ? b.scale_log2 : 1.f;
    float ls[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) ls[i] = 0.f;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      uint32_t pk[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float p0 = fast_exp2(fmaf(s[32 * c + 2 * i], sa, -msub));
        const float p1 = fast_exp2(fmaf(s[32 * c + 2 * i + 1], sa, -msub));
        ls[(2 * i) & 7] += p0;
        ls[(2 * i + 1) & 7] += p1;
        pk[i] = pack_bf16x2(p0, p1);
      }
      tmem_st16(tm + lane_off + s_col + 16 * c, pk);
    }
    l += ((ls[0] + ls[1]) + (ls[2] + ls[3])) + ((ls[4] + ls[5]) + (ls[6] + ls[7]));
    tmem_wait_st();
    tc_fence_before();
    mbar_arrive(&sm.bar_p[role]);
  }
  if (!ok) atomicOr(&g_attn_error, 4u);
  const int h = role ? hB : hA;
  if (ok && n_tiles > 0 && !warp_wait(&sm.bar_o[role], (n_tiles - 1) & 1)) {
    ok = false;
    atomicOr(&g_attn_error, 8u);
  }
  tc_fence_after();
  // the TMEM reads run on every lane (warp-collective); only real rows store
  const bool store = q_row < p.Lq;
  const float inv = (ok && l > 0.f) ? 1.f / l : 0.f;
  __nv_bfloat16* orow = static_cast<__nv_bfloat16*>(p.o) + h * p.o_head_stride + (store ? q_row : 0) * p.o_row_stride;
#pragma unroll 1
  for (int c = 0; c < 4; ++c) {
    uint32_t r[32];
    if (n_tiles > 0 || kInit) {
      tmem_ld32(tm + lane_off + o_col + 32 * c, r);
      tmem_wait_ld();
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i) r[i] = 0u;
    }
    if (store) {
#pragma unroll
      for (int v = 0; v < 4; ++v) {
        uint4 w;
        w.x = pack_bf16x2(__uint_as_float(r[8 * v + 0]) * inv, __uint_as_float(r[8 * v + 1]) * inv);
        w.y = pack_bf16x2(__uint_as_float(r[8 * v + 2]) * inv, __uint_as_float(r[8 * v + 3]) * inv);
        w.z = pack_bf16x2(__uint_as_float(r[8 * v + 4]) * inv, __uint_as_float(r[8 * v + 5]) * inv);
        w.w = pack_bf16x2(__uint_as_float(r[8 * v + 6]) * inv, __uint_as_float(r[8 * v + 7]) * inv);
        *reinterpret_cast<uint4*>(orow + 32 * c + 8 * v) = w;
      }
    }
  }
  if (store && p.lse)
    p.lse[h * p.lse_head_stride + q_row] = (ok && l > 0.f) ? (m_use + log2f(l)) * 0.6931471805599453f : -INFINITY;
}

// kInit: every problem of the batch carries an initial state (a separate
// instantiation, so the plain launch carries no code for it)
template <bool kInit>
__global__ void __launch_bounds__(kThreads, 1) attn_tc05_kernel(const __grid_constant__ Tc05Batch b) {
  extern __shared__ unsigned char smem_raw[];
  Smem& sm = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  const Tc05Problem& p = b.p[blockIdx.z];
  const int n_qt = (int)((p.Lq + kRows - 1) / kRows);
  const int qt = n_qt - 1 - (int)blockIdx.x;  // heaviest (causal) tiles first
  if (qt < 0) return;
  const int64_t q0 = (int64_t)qt * kRows;
  const int hA = 2 * blockIdx.y, hB = hA + 1, hk = hA / b.group;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  int64_t kend[kTcMaxSeg];
  int n_tiles = 0;
  for (int s = 0; s < kTcMaxSeg; ++s) {
    int64_t e = s < p.n_seg ? p.seg[s].len : 0;
    if (p.causal && s == 0) {
      const int64_t last = (q0 + kRows - 1 < p.Lq - 1 ? q0 + kRows - 1 : p.Lq - 1) + p.causal_offset + 1;
      e = e < last ? e : last;
    }
    kend[s] = e > 0 ? e : 0;
    n_tiles += (int)((kend[s] + kKeys - 1) / kKeys);
  }

  if (threadIdx.x == 0) {
    mbar_init(&sm.bar_q, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sm.bar_k[i], 1);
      mbar_init(&sm.bar_v[i], 1);
      mbar_init(&sm.bar_bias[i], 32);
      mbar_init(&sm.bar_empty[i], 1);
      mbar_init(&sm.bar_s[i], 1);
      mbar_init(&sm.bar_p[i], 128);
      mbar_init(&sm.bar_o[i], 1);
    }
    fence_mbar_init();
  }
  if (warp == 9) {
    tmem_alloc(&sm.tmem, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tm = sm.tmem;
  if (warp >= 8) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;\n" ::"n"(kRegsOther));
    if (warp == 8) producer_role(p, sm, kend, n_tiles, q0, hA, hB, hk, lane);
    else if (warp == 9) mma_role<kInit>(sm, n_tiles, tm, lane);
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;\n" ::"n"(kRegsSoftmax));
    softmax_role<kInit>(b, p, sm, kend, n_tiles, q0, hA, hB, tm, warp, lane);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 9) tmem_dealloc(tm, 512);
}

static size_t tc05_smem_bytes() { return sizeof(Smem) + 1024; }

// Host: build the batch (tensor maps per problem and segment) and launch.
// Problems with and without an initial state go to separate launches of the
// two kernel instantiations.
template <bool kInit>
static int tc05_prepare() {
  DCC_CHECK(check_cuda(cudaFuncSetAttribute(attn_tc05_kernel<kInit>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            (int)tc05_smem_bytes()),
                       "attn_tc05 smem"));
  // The setmaxnreg split assumes the kernel launches with kRegsLaunch registers
  // per thread; a smaller launch allocation would make setmaxnreg.inc wait forever.
  cudaFuncAttributes fa{};
  DCC_CHECK(check_cuda(cudaFuncGetAttributes(&fa, attn_tc05_kernel<kInit>), "attn_tc05 attributes"));
  if (fa.numRegs < kRegsLaunch)
    return fail(DCC_ERR_UNSUPPORTED, "attn_tc05: compiled with " + std::to_string(fa.numRegs) +
                                         " registers per thread, the register split needs " +
                                         std::to_string(kRegsLaunch));
  return DCC_OK;
}

template <bool kInit>
static int tc05_launch(const Tc05Batch& b, int64_t max_lq, const AttnParams& prm, cudaStream_t st) {
  dim3 grid((unsigned)((max_lq + 127) / 128), prm.n_q_heads / 2, b.n);
  attn_tc05_kernel<kInit><<<grid, kThreads, tc05_smem_bytes(), st>>>(b);
  const cudaError_t le = cudaGetLastError();
  if (le != cudaSuccess) {
    cudaFuncAttributes fa{};
    cudaFuncGetAttributes(&fa, attn_tc05_kernel<kInit>);
    return fail(DCC_ERR_CUDA, std::string("attn_tc05 launch: ") + cudaGetErrorString(le) + " (" +
                                  std::to_string(fa.numRegs) + " registers, max " +
                                  std::to_string(fa.maxThreadsPerBlock) + " threads, " +
                                  std::to_string(tc05_smem_bytes()) + " B dynamic shared memory)");
  }
  return DCC_OK;
}

int launch_attn_tc05(const dcc_attn_problem* probs, int n, const AttnParams& prm, cudaStream_t st) {
  bool any_init = false, any_plain = false;
  for (int i = 0; i < n; ++i) (probs[i].o_init ? any_init : any_plain) = true;
  if (any_plain) DCC_CHECK(tc05_prepare<false>());
  if (any_init) DCC_CHECK(tc05_prepare<true>());
  Tc05Batch* bp = new Tc05Batch();
  std::unique_ptr<Tc05Batch> own(bp);
  Tc05Batch& b = *bp;
  b.group = prm.group;
  b.scale_log2 = (float)(prm.scale * 1.4426950408889634);
  int64_t max_lq = 0;
  bool batch_init = false;
  auto flush = [&]() -> int {
    if (b.n == 0) return DCC_OK;
    if (max_lq > 0) DCC_CHECK(batch_init ? tc05_launch<true>(b, max_lq, prm, st) : tc05_launch<false>(b, max_lq, prm, st));
    b.n = 0;
    max_lq = 0;
    return DCC_OK;
  };
  for (int i = 0; i < n; ++i) {
    const dcc_attn_problem& q = probs[i];
    const bool init = q.o_init != nullptr;
    if (b.n > 0 && init != batch_init) DCC_CHECK(flush());
    batch_init = init;
    Tc05Problem& t = b.p[b.n];
    t = Tc05Problem{};
    if (q.Lq > 0)  // an empty problem launches no CTA and needs no map
      DCC_CHECK(make_tmap_bf16_3d(&t.q, q.q, 128, q.Lq, prm.n_q_heads, q.q_row_stride, q.q_head_stride, 128));
    t.o = q.o;
    t.lse = q.lse;
    t.o_head_stride = q.o_head_stride;
    t.o_row_stride = q.o_row_stride;
    t.lse_head_stride = q.lse_head_stride;
    t.Lq = q.Lq;
    t.n_seg = q.n_seg;
    t.causal = q.causal;
    t.causal_offset = q.causal_offset;
    t.o_init = q.o_init;
    t.lse_init = q.lse_init;
    t.lse_init_head_stride = q.lse_init_head_stride;
    for (int s = 0; s < q.n_seg; ++s) {
      const dcc_kv_segment& g = q.seg[s];
      Tc05Seg& ts = t.seg[s];
      if (g.len > 0) {  // an empty segment contributes no tile and needs no map
        DCC_CHECK(make_tmap_bf16_3d(&ts.k, g.k, 128, g.len, prm.n_kv_heads, g.row_stride, g.k_head_stride, 128));
        DCC_CHECK(make_tmap_bf16_3d(&ts.v, g.v, 128, g.len, prm.n_kv_heads, g.row_stride, g.v_head_stride, 128));
      }
      ts.bias = g.bias;
      ts.bias_head_stride = g.bias_head_stride;
      ts.len = g.len;
    }
    if (q.Lq > max_lq) max_lq = q.Lq;
    ++b.n;
    if (b.n == kTcCap) DCC_CHECK(flush());
  }
  return flush();
}

bool attn_tc05_supported(const dcc_attn_problem& p, const AttnParams& prm) {
  if (prm.d != 128 || prm.group % 2 != 0 || prm.n_q_heads % 2 != 0 || p.n_seg > kTcMaxSeg) return false;
  if (p.Lq > 0x7fffffff) return false;
  for (int s = 0; s < p.n_seg; ++s)
    if (p.seg[s].len > 0x7fffffff) return false;
  return true;
}

int score_error_flag_address(unsigned int** out);

// Both error words to host memory by a posted write from the device (pinned
// host memory is device-accessible under unified addressing), so reading
// them needs neither a copy engine nor a synchronisation.
__global__ void flags_to_host_kernel(const unsigned int* score_flag, unsigned int* host) {
  host[0] = *reinterpret_cast<volatile unsigned int*>(&g_attn_error);
  host[1] = *reinterpret_cast<const volatile unsigned int*>(score_flag);
  __threadfence_system();
}

// One warp waits, with the same bounded wait as the kernels above, on an
// mbarrier that nothing arrives at; when the limit passes it records the
// timeout in the attention error word (bit 16).  It has no asynchronous
// copy or MMA in flight, so it simply returns.
__global__ void expire_wait_kernel(uint64_t limit_ns) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncwarp();
  if (!warp_wait_limited(&bar, 0, limit_ns) && threadIdx.x == 0) atomicOr(&g_attn_error, 16u);
}

}  // namespace dcc

using namespace dcc;

extern "C" int dcc_device_error_flags_async(unsigned int* host_flags, void* stream) {
  if (host_flags == nullptr) return fail(DCC_ERR_INVALID_ARGUMENT, "device_error_flags_async: null destination");
  static std::mutex mu;
  static unsigned int* score_flag[64] = {};
  int dev = 0;
  DCC_CHECK(check_cuda(cudaGetDevice(&dev), "device_error_flags_async: cudaGetDevice"));
  if (dev < 0 || dev >= 64) return fail(DCC_ERR_UNSUPPORTED, "device_error_flags_async: device ordinal above 63");
  {
    std::lock_guard<std::mutex> lock(mu);
    if (score_flag[dev] == nullptr) DCC_CHECK(score_error_flag_address(&score_flag[dev]));
  }
  cudaPointerAttributes pa{};
  DCC_CHECK(check_cuda(cudaPointerGetAttributes(&pa, host_flags), "device_error_flags_async: pointer attributes"));
  if (pa.type != cudaMemoryTypeHost || pa.devicePointer == nullptr)
    return fail(DCC_ERR_INVALID_ARGUMENT, "device_error_flags_async: destination must be pinned host memory");
  flags_to_host_kernel<<<1, 1, 0, static_cast<cudaStream_t>(stream)>>>(
      score_flag[dev], static_cast<unsigned int*>(pa.devicePointer));
  return check_cuda(cudaGetLastError(), "device_error_flags_async launch");
}

extern "C" int dcc_debug_expire_wait(uint64_t limit_ns, void* stream) {
  if (limit_ns > 100000000ull) return fail(DCC_ERR_INVALID_ARGUMENT, "debug_expire_wait: limit above 100 ms");
  expire_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(limit_ns);
  return check_cuda(cudaGetLastError(), "debug_expire_wait launch");
}

extern "C" int dcc_device_error_status(int clear) {
  DCC_CHECK(check_cuda(cudaDeviceSynchronize(), "device_error_status: synchronize"));
  unsigned int v = 0;
  DCC_CHECK(check_cuda(cudaMemcpyFromSymbol(&v, g_attn_error, sizeof(v)), "device_error_status: read"));
  if (clear && v) {
    unsigned int z = 0;
    DCC_CHECK(check_cuda(cudaMemcpyToSymbol(g_attn_error, &z, sizeof(z)), "device_error_status: clear"));
  }
  if (v) return fail(DCC_ERR_TIMEOUT, "attention: a bounded device wait expired (flags " + std::to_string(v) + ")");
  return DCC_OK;
}
