// Attention over KV segments with per-key logit bias, CUDA-core version:
// the FP64-accumulating parity path for DCC_F32 / DCC_F64 inputs and any
// head_dim <= 128 (dcc_kv_sync_cpu.py:52-55 local, :71-74 compact).
//
// 8 threads share one query row (each owns head_dim/8 output columns), 16
// rows per CTA; K/V tiles of 32 keys are staged in shared memory and every
// key updates the running (max, sum, output) online-softmax state.
#include "attention.cuh"

namespace dcc {

template <typename TIn, typename Acc>
__global__ void __launch_bounds__(128) attn_simt_kernel(const __grid_constant__ AttnBatch b,
                                                        const AttnParams prm) {
  const dcc_attn_problem& p = b.p[blockIdx.z];
  const int h = blockIdx.y;
  const int hk = h / prm.group;
  const int row_in = threadIdx.x >> 3, part = threadIdx.x & 7;
  const int64_t row = (int64_t)blockIdx.x * 16 + row_in;
  if ((int64_t)blockIdx.x * 16 >= p.Lq) return;
  const bool valid = row < p.Lq;
  const int D = prm.d;
  const int per = (D + 7) / 8;
  constexpr int kMaxPer = 16;
  extern __shared__ unsigned char smem_raw[];
  Acc* ks = reinterpret_cast<Acc*>(smem_raw);  // [32][D]
  Acc* vs = ks + 32 * D;                        // [32][D]
  __shared__ float bs[32];
  Acc q[kMaxPer], o[kMaxPer];
  const TIn* qp = static_cast<const TIn*>(p.q) + h * p.q_head_stride + (valid ? row : 0) * p.q_row_stride;
#pragma unroll
  for (int i = 0; i < kMaxPer; ++i) {
    const int c = part * per + i;
    q[i] = (i < per && c < D) ? to_acc<Acc, TIn>(qp[c]) : Acc(0);
    o[i] = Acc(0);
  }
  Acc m = NegInf<Acc>::v(), l = Acc(0);
  if (p.o_init && valid) {  // continue from (m = lse, l = 1, o = normalised partial)
    const float lse0 = p.lse_init[h * p.lse_init_head_stride + row];
    if (lse0 > -INFINITY) {
      m = Acc(lse0);
      l = Acc(1);
      const TIn* oi = static_cast<const TIn*>(p.o_init) + h * p.o_head_stride + row * p.o_row_stride;
#pragma unroll
      for (int i = 0; i < kMaxPer; ++i) {
        const int c = part * per + i;
        if (i < per && c < D) o[i] = to_acc<Acc, TIn>(oi[c]);
      }
    }
  }
  const Acc scale = Acc(prm.scale);
  for (int sg = 0; sg < p.n_seg; ++sg) {
    const dcc_kv_segment& s = p.seg[sg];
    const bool causal = p.causal && sg == 0;
    int64_t kend = s.len;
    if (causal) {  // keys this CTA's last row can see
      const int64_t last = min(p.Lq - 1, (int64_t)blockIdx.x * 16 + 15);
      kend = min(kend, last + p.causal_offset + 1);
    }
    const TIn* kp = static_cast<const TIn*>(s.k) + hk * s.k_head_stride;
    const TIn* vp = static_cast<const TIn*>(s.v) + hk * s.v_head_stride;
    const float* bp = s.bias ? s.bias + hk * s.bias_head_stride : nullptr;
    for (int64_t t0 = 0; t0 < kend; t0 += 32) {
      __syncthreads();
      for (int e = threadIdx.x; e < 32 * D; e += blockDim.x) {
        const int r = e / D, c = e - r * D;
        const int64_t j = t0 + r;
        ks[e] = j < kend ? to_acc<Acc, TIn>(kp[j * s.row_stride + c]) : Acc(0);
        vs[e] = j < kend ? to_acc<Acc, TIn>(vp[j * s.row_stride + c]) : Acc(0);
      }
      if (threadIdx.x < 32) bs[threadIdx.x] = (bp && t0 + threadIdx.x < kend) ? bp[t0 + threadIdx.x] : 0.f;
      __syncthreads();
      const int jn = (int)((kend - t0) < 32 ? (kend - t0) : 32);
      for (int jj = 0; jj < jn; ++jj) {
        Acc dot = 0;
#pragma unroll
        for (int i = 0; i < kMaxPer; ++i) {
          const int c = part * per + i;
          if (i < per && c < D) dot = fma(q[i], ks[jj * D + c], dot);
        }
        dot += __shfl_xor_sync(0xffffffffu, dot, 1);
        dot += __shfl_xor_sync(0xffffffffu, dot, 2);
        dot += __shfl_xor_sync(0xffffffffu, dot, 4);
        const int64_t j = t0 + jj;
        if (!valid || (causal && j > row + p.causal_offset)) continue;
        const Acc x = dot * scale + Acc(bs[jj]);
        const Acc mn = max(m, x);
        const Acc corr = acc_exp(m - mn);
        const Acc e = acc_exp(x - mn);
        l = l * corr + e;
#pragma unroll
        for (int i = 0; i < kMaxPer; ++i) {
          const int c = part * per + i;
          if (i < per && c < D) o[i] = o[i] * corr + e * vs[jj * D + c];
        }
        m = mn;
      }
    }
  }
  if (!valid) return;
  TIn* op = static_cast<TIn*>(p.o) + h * p.o_head_stride + row * p.o_row_stride;
  const Acc inv = l > Acc(0) ? Acc(1) / l : Acc(0);
#pragma unroll
  for (int i = 0; i < kMaxPer; ++i) {
    const int c = part * per + i;
    if (i < per && c < D) op[c] = from_f64<TIn>((double)(o[i] * inv));
  }
  if (p.lse && part == 0)
    p.lse[h * p.lse_head_stride + row] = l > Acc(0) ? (float)(m + acc_log(l)) : -INFINITY;
}

template <typename TIn, typename Acc>
int launch_attn_simt(const AttnBatch& b, const AttnParams& prm, int64_t max_lq, cudaStream_t st) {
  const size_t smem = 2 * 32 * (size_t)prm.d * sizeof(Acc);
  auto k = attn_simt_kernel<TIn, Acc>;
  DCC_CHECK(check_cuda(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                       "attn_simt smem"));
  dim3 grid((unsigned)((max_lq + 15) / 16), prm.n_q_heads, b.n);
  k<<<grid, 128, smem, st>>>(b, prm);
  return check_launch("attn_simt");
}

template int launch_attn_simt<float, double>(const AttnBatch&, const AttnParams&, int64_t, cudaStream_t);
template int launch_attn_simt<double, double>(const AttnBatch&, const AttnParams&, int64_t, cudaStream_t);
template int launch_attn_simt<__nv_bfloat16, float>(const AttnBatch&, const AttnParams&, int64_t, cudaStream_t);

}  // namespace dcc
