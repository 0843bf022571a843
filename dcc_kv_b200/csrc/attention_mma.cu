// bf16 attention over KV segments with per-key logit bias, warp-level MMA
// (m16n8k16, fp32 accumulate), head_dim 128.
//
// CTA = 4 warps x 16 query rows; K/V tiles of 64 keys double-buffered with
// cp.async into XOR-swizzled shared memory (16-byte chunk c of row r sits at
// chunk c ^ (r & 7), so ldmatrix rows never collide).  S = Q K^T stays in
// registers, the online softmax runs in base 2, and P is re-used as the A
// operand of P V straight from the S accumulators.
#include "attention.cuh"

namespace dcc {

namespace mma_attn {

constexpr int kD = 128;
constexpr int kBM = 64;   // query rows per CTA
constexpr int kBN = 64;   // keys per tile
constexpr int kThreads = 128;
constexpr int kTileBytes = kBN * kD * 2;  // 16 KB

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ uint32_t swz(int row, int chunk) {
  return (uint32_t)(row * 256 + ((chunk ^ (row & 7)) << 4));
}
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  const int n = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(n));
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
__device__ __forceinline__ void mma16816(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Load rows [r0, r0 + 64) of a [len, 128] bf16 matrix (row stride `ld`) into a
// swizzled tile; rows at or beyond `len` are zero-filled.
__device__ __forceinline__ void load_tile(uint32_t sbase, const __nv_bfloat16* g, int64_t ld, int64_t r0,
                                          int64_t len) {
#pragma unroll
  for (int i = 0; i < (kBN * 16) / kThreads; ++i) {
    const int e = threadIdx.x + i * kThreads;
    const int r = e >> 4, c = e & 15;
    const int64_t gr = r0 + r;
    const bool ok = gr < len;
    const __nv_bfloat16* src = g + (ok ? gr : 0) * ld + c * 8;
    cp_async16(sbase + swz(r, c), src, ok);
  }
}

struct TileCursor {
  int seg;
  int64_t t0;
};

}  // namespace mma_attn

using namespace mma_attn;

__global__ void __launch_bounds__(kThreads) attn_mma_bf16_kernel(const __grid_constant__ AttnBatch b,
                                                                 const AttnParams prm) {
  const dcc_attn_problem& p = b.p[blockIdx.z];
  const int h = blockIdx.y, hk = h / prm.group;
  const int64_t q0 = (int64_t)blockIdx.x * kBM;
  if (q0 >= p.Lq) return;
  extern __shared__ __align__(1024) unsigned char smem[];
  unsigned char* qs = smem;                       // [64][128]
  unsigned char* ks = smem + kTileBytes;          // [2][64][128]
  unsigned char* vs = ks + 2 * kTileBytes;        // [2][64][128]
  float* bsm = reinterpret_cast<float*>(vs + 2 * kTileBytes);  // [2][64]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  // key range of each segment visible to this CTA
  int64_t kend[DCC_MAX_SEGMENTS];
  for (int s = 0; s < p.n_seg; ++s) {
    kend[s] = p.seg[s].len;
    if (p.causal && s == 0) kend[s] = min(kend[s], min(p.Lq - 1, q0 + kBM - 1) + p.causal_offset + 1);
  }
  auto advance = [&](TileCursor& c) {
    c.t0 += kBN;
    while (c.seg < p.n_seg && c.t0 >= kend[c.seg]) {
      ++c.seg;
      c.t0 = 0;
    }
  };
  TileCursor cur{0, -kBN};
  advance(cur);

  const __nv_bfloat16* qg = static_cast<const __nv_bfloat16*>(p.q) + h * p.q_head_stride;
  load_tile(smem_u32(qs), qg, p.q_row_stride, q0, p.Lq);
  auto issue = [&](const TileCursor& c, int buf) {
    const dcc_kv_segment& s = p.seg[c.seg];
    const __nv_bfloat16* kg = static_cast<const __nv_bfloat16*>(s.k) + hk * s.k_head_stride;
    const __nv_bfloat16* vg = static_cast<const __nv_bfloat16*>(s.v) + hk * s.v_head_stride;
    load_tile(smem_u32(ks + buf * kTileBytes), kg, s.row_stride, c.t0, kend[c.seg]);
    load_tile(smem_u32(vs + buf * kTileBytes), vg, s.row_stride, c.t0, kend[c.seg]);
    if (threadIdx.x < kBN) {
      const int64_t j = c.t0 + threadIdx.x;
      const float* bg = s.bias ? s.bias + hk * s.bias_head_stride : nullptr;
      bsm[buf * kBN + threadIdx.x] = (bg && j < kend[c.seg]) ? bg[j] : 0.f;
    }
  };
  if (cur.seg < p.n_seg) issue(cur, 0);
  cp_commit();
  cp_wait<0>();
  __syncthreads();

  // Q fragments, 8 k-steps
  uint32_t qf[8][4];
  {
    const int r = warp * 16 + (lane & 15);
#pragma unroll
    for (int kk = 0; kk < 8; ++kk)
      ldsm_x4(smem_u32(qs) + swz(r, 2 * kk + (lane >> 4)), qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3]);
  }
  float o[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  const float kLog2e = 1.4426950408889634f;
  const float sl2 = (float)prm.scale * kLog2e;
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
  const int64_t row_a = q0 + warp * 16 + (lane >> 2);  // this thread's rows: row_a, row_a + 8
  if (p.o_init) {  // continue from (m = lse, l = 1, o = normalised partial); l summed over the quad
    const __nv_bfloat16* oi = static_cast<const __nv_bfloat16*>(p.o_init) + h * p.o_head_stride;
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const int64_t row = row_a + 8 * r;
      if (row >= p.Lq) continue;
      const float lse0 = p.lse_init[h * p.lse_init_head_stride + row];
      if (!(lse0 > -INFINITY)) continue;
      m_run[r] = lse0 * kLog2e;
      l_run[r] = (lane & 3) == 0 ? 1.f : 0.f;
#pragma unroll
      for (int nd = 0; nd < 16; ++nd) {
        const int col = nd * 8 + 2 * (lane & 3);
        const __nv_bfloat162 v2 = *reinterpret_cast<const __nv_bfloat162*>(oi + row * p.o_row_stride + col);
        o[nd][2 * r] = __bfloat162float(v2.x);
        o[nd][2 * r + 1] = __bfloat162float(v2.y);
      }
    }
  }

  int buf = 0;
  while (cur.seg < p.n_seg) {
    TileCursor nxt = cur;
    advance(nxt);
    if (nxt.seg < p.n_seg) issue(nxt, buf ^ 1);
    cp_commit();
    cp_wait<1>();
    __syncthreads();
    const uint32_t kb = smem_u32(ks + buf * kTileBytes), vb = smem_u32(vs + buf * kTileBytes);
    float s[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
#pragma unroll
      for (int nt = 0; nt < 8; nt += 2) {
        const int j = lane >> 3;
        const int key = 8 * (nt + (j >> 1)) + (lane & 7);
        uint32_t b0, b1, b2, b3;
        ldsm_x4(kb + swz(key, 2 * kk + (j & 1)), b0, b1, b2, b3);
        mma16816(s[nt], qf[kk], b0, b1);
        mma16816(s[nt + 1], qf[kk], b2, b3);
      }
    }
    // scale, bias, mask (base-2 logits)
    const bool causal = p.causal && cur.seg == 0;
    const int64_t klen = kend[cur.seg];
    float tmax[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int col = nt * 8 + 2 * (lane & 3) + (e & 1);
        const int64_t key = cur.t0 + col;
        const int64_t row = row_a + ((e >> 1) << 3);
        float x = s[nt][e] * sl2 + bsm[buf * kBN + col] * kLog2e;
        const bool masked = key >= klen || (causal && key > row + p.causal_offset);
        x = masked ? -INFINITY : x;
        s[nt][e] = x;
        tmax[e >> 1] = fmaxf(tmax[e >> 1], x);
      }
    }
    float corr[2], muse[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      tmax[r] = fmaxf(tmax[r], __shfl_xor_sync(0xffffffffu, tmax[r], 1));
      tmax[r] = fmaxf(tmax[r], __shfl_xor_sync(0xffffffffu, tmax[r], 2));
      const float mn = fmaxf(m_run[r], tmax[r]);
      muse[r] = mn == -INFINITY ? 0.f : mn;
      corr[r] = exp2f(m_run[r] - muse[r]);
      m_run[r] = mn;
      l_run[r] *= corr[r];
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      o[i][0] *= corr[0];
      o[i][1] *= corr[0];
      o[i][2] *= corr[1];
      o[i][3] *= corr[1];
    }
    uint32_t pa[4][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      const float p0 = exp2f(s[nt][0] - muse[0]), p1 = exp2f(s[nt][1] - muse[0]);
      const float p2 = exp2f(s[nt][2] - muse[1]), p3 = exp2f(s[nt][3] - muse[1]);
      l_run[0] += p0 + p1;
      l_run[1] += p2 + p3;
      const int kk = nt >> 1, hi = nt & 1;
      pa[kk][hi * 2 + 0] = pack_bf16(p0, p1);
      pa[kk][hi * 2 + 1] = pack_bf16(p2, p3);
    }
    // O += P V
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
      for (int nd = 0; nd < 16; nd += 2) {
        const int j = lane >> 3;
        const int key = 16 * kk + (lane & 7) + 8 * (j & 1);
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(vb + swz(key, nd + (j >> 1)), b0, b1, b2, b3);
        mma16816(o[nd], pa[kk], b0, b1);
        mma16816(o[nd + 1], pa[kk], b2, b3);
      }
    }
    __syncthreads();
    cur = nxt;
    buf ^= 1;
  }
  // finalize
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    l_run[r] += __shfl_xor_sync(0xffffffffu, l_run[r], 1);
    l_run[r] += __shfl_xor_sync(0xffffffffu, l_run[r], 2);
  }
  __nv_bfloat16* og = static_cast<__nv_bfloat16*>(p.o) + h * p.o_head_stride;
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int64_t row = row_a + 8 * r;
    if (row >= p.Lq) continue;
    const float inv = l_run[r] > 0.f ? 1.f / l_run[r] : 0.f;
#pragma unroll
    for (int nd = 0; nd < 16; ++nd) {
      const int col = nd * 8 + 2 * (lane & 3);
      *reinterpret_cast<uint32_t*>(og + row * p.o_row_stride + col) =
          pack_bf16(o[nd][2 * r] * inv, o[nd][2 * r + 1] * inv);
    }
    if (p.lse && (lane & 3) == 0)
      p.lse[h * p.lse_head_stride + row] =
          l_run[r] > 0.f ? (m_run[r] + log2f(l_run[r])) * 0.6931471805599453f : -INFINITY;
  }
}

int launch_attn_mma_bf16(const AttnBatch& b, const AttnParams& prm, int64_t max_lq, cudaStream_t st) {
  const size_t smem = 5 * (size_t)kTileBytes + 2 * kBN * sizeof(float);
  DCC_CHECK(check_cuda(cudaFuncSetAttribute(attn_mma_bf16_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            (int)smem),
                       "attn_mma smem"));
  dim3 grid((unsigned)((max_lq + kBM - 1) / kBM), prm.n_q_heads, b.n);
  attn_mma_bf16_kernel<<<grid, kThreads, smem, st>>>(b, prm);
  return check_launch("attn_mma_bf16");
}

}  // namespace dcc
