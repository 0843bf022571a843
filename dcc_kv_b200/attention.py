"""Attention over KV segments with per-key logit bias (GPU).

The destination side of the reference layer (dcc_kv_sync_cpu.py:52-84):
the local block attended causally, each compact block attended with its
logit bias added at full weight, each producing a normalised output and its
log-sum-exp for the online-softmax merge.  Query head h reads KV head
h // (n_q_heads // n_kv_heads) (GQA).
"""
from __future__ import annotations

import math
from typing import Optional, Sequence, Tuple

import torch

from . import _lib as L


def kv_segment(k: torch.Tensor, v: torch.Tensor, bias: Optional[torch.Tensor] = None,
               length: Optional[int] = None) -> L.dcc_kv_segment:
    """k, v: [H_kv, len, d] views (unit column stride); bias [H_kv, len] float32."""
    assert k.stride(-1) == 1 and v.stride(-1) == 1 and k.stride(1) == v.stride(1)
    s = L.dcc_kv_segment()
    s.k = k.data_ptr()
    s.v = v.data_ptr()
    s.bias = None if bias is None else bias.data_ptr()
    s.k_head_stride = k.stride(0)
    s.v_head_stride = v.stride(0)
    s.row_stride = k.stride(1)
    s.bias_head_stride = 0 if bias is None else bias.stride(0)
    s.len = k.shape[1] if length is None else length
    return s


def attn_problem(q: torch.Tensor, o: torch.Tensor, lse: Optional[torch.Tensor],
                 segments: Sequence[L.dcc_kv_segment], causal: bool = False,
                 causal_offset: int = 0, o_init: Optional[torch.Tensor] = None,
                 lse_init: Optional[torch.Tensor] = None) -> L.dcc_attn_problem:
    """q, o: [H_q, Lq, d] views (unit column stride); lse [H_q, Lq] float32.
    ``o_init`` (o's strides, may be o itself) and ``lse_init`` [H_q, Lq]: an
    initial online-softmax state the rows continue from (merge_softmax_states
    of that state with the attention over the segments)."""
    if len(segments) > L.MAX_SEGMENTS:
        raise ValueError(f"at most {L.MAX_SEGMENTS} KV segments per problem")
    p = L.dcc_attn_problem()
    p.q = q.data_ptr()
    p.q_head_stride = q.stride(0)
    p.q_row_stride = q.stride(1)
    p.o = o.data_ptr()
    p.o_head_stride = o.stride(0)
    p.o_row_stride = o.stride(1)
    p.lse = None if lse is None else lse.data_ptr()
    p.lse_head_stride = 0 if lse is None else lse.stride(0)
    p.Lq = q.shape[1]
    p.n_seg = len(segments)
    p.causal = 1 if causal else 0
    p.causal_offset = causal_offset
    for i, s in enumerate(segments):
        p.seg[i] = s
    if (o_init is None) != (lse_init is None):
        raise ValueError("o_init and lse_init come together")
    if o_init is not None:
        if o_init.stride() != o.stride() or o_init.shape != o.shape or o_init.dtype != o.dtype:
            raise ValueError("o_init must have o's shape, strides and dtype")
        if lse_init.dtype != torch.float32 or lse_init.shape != o.shape[:2] or lse_init.stride(1) != 1:
            raise ValueError("lse_init must be float32 [H_q, Lq] with unit row stride")
        p.o_init = o_init.data_ptr()
        p.lse_init = lse_init.data_ptr()
        p.lse_init_head_stride = lse_init.stride(0)
    return p


def run_attention(problems: Sequence[L.dcc_attn_problem], n_q_heads: int, n_kv_heads: int, head_dim: int,
                  scale: float, dtype_code: int, device: torch.device) -> None:
    n = len(problems)
    if n == 0:
        return
    arr = (L.dcc_attn_problem * n)(*problems)
    L.check(L.lib().dcc_attention_fwd(arr, n, n_q_heads, n_kv_heads, head_dim, scale, dtype_code,
                                      L.stream_ptr(device)), "attention_fwd")


def attention(q: torch.Tensor, segments: Sequence[Tuple[torch.Tensor, torch.Tensor, Optional[torch.Tensor]]],
              causal: bool = False, causal_offset: int = 0,
              scale: Optional[float] = None,
              init: Optional[Tuple[torch.Tensor, torch.Tensor]] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """q [H_q, Lq, d]; segments: (k [H_kv, len, d], v, bias [H_kv, len] or None).
    Returns (O [H_q, Lq, d] in q's dtype, LSE [H_q, Lq] float32).  ``init`` =
    (O0, LSE0) from an earlier call continues that online softmax: the result
    is merge_softmax_states of the earlier state with these segments."""
    assert q.dim() == 3
    L.require_cuda(q)
    q = q.contiguous() if q.stride(-1) != 1 else q
    hq, lq, d = q.shape
    segs = []
    hkv = None
    for k, v, b in segments:
        L.require_cuda(k, v, b)
        k = k.to(q.dtype).contiguous()
        v = v.to(q.dtype).contiguous()
        b = None if b is None else b.to(torch.float32).contiguous()
        hkv = k.shape[0]
        segs.append((k, v, b))
    if hkv is None:
        raise ValueError("need at least one KV segment")
    o = torch.empty_like(q)
    lse = torch.empty(hq, lq, dtype=torch.float32, device=q.device)
    o0 = lse0 = None
    if init is not None:
        o0, lse0 = init
        L.require_cuda(o0, lse0)
        o0 = o0.to(q.dtype).contiguous()
        lse0 = lse0.to(torch.float32).contiguous()
        if o0.shape != q.shape or lse0.shape != (hq, lq):
            raise ValueError(f"init must be O {tuple(q.shape)} and LSE {(hq, lq)}")
    prob = attn_problem(q, o, lse, [kv_segment(k, v, b) for k, v, b in segs], causal, causal_offset,
                        o_init=o0, lse_init=lse0)
    run_attention([prob], hq, hkv, d, scale if scale is not None else 1.0 / math.sqrt(d), L.dtype_code(q), q.device)
    return o, lse
