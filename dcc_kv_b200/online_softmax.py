"""Online-softmax states and merges on the GPU.

Mirrors ``src/dcc_kv_ref/online_softmax.py`` (lfei7199-star/dcc-kv): the
same names, argument meaning and assertions, batched over leading
dimensions.  Every computation runs in ``libdcckv.so`` kernels.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional, Sequence, Tuple

import torch

from . import _lib as L


@dataclass
class OnlineSoftmaxState:
    """(m, l, o) of one block: m = max logit, l = sum exp(logit - m),
    o = sum exp(logit - m) V (unnormalised); output = o / l.
    online_softmax.py:20-49.  Batched: m, l [...], o [..., d]."""
    m: torch.Tensor
    l: torch.Tensor
    o: torch.Tensor

    def __post_init__(self):
        if not isinstance(self.m, torch.Tensor):
            self.m = torch.tensor(self.m, dtype=torch.float64)
        if not isinstance(self.l, torch.Tensor):
            self.l = torch.tensor(self.l, dtype=torch.float64)
        if not isinstance(self.o, torch.Tensor):
            self.o = torch.tensor(self.o, dtype=torch.float64)


def online_softmax_from_attention(logits: torch.Tensor, values: torch.Tensor,
                                  logit_bias: Optional[torch.Tensor] = None) -> OnlineSoftmaxState:
    """online_softmax.py:52-89.  ``logits`` [L] (or [R, L]), ``values`` [L, d]
    (shared by every row) or [R, L, d]; ``logit_bias`` [L] is added first."""
    assert logits.dim() in (1, 2), f"logits must be 1D, got {logits.dim()}D"
    assert values.dim() in (2, 3), f"values must be 2D, got {values.dim()}D"
    assert logits.shape[-1] == values.shape[-2], "logits/values length mismatch"
    if logit_bias is not None:
        assert logit_bias.shape == logits.shape[-1:], "logit_bias shape mismatch"
    L.require_cuda(logits, values, logit_bias)
    single = logits.dim() == 1
    x = logits.reshape(-1, logits.shape[-1]).contiguous()
    R, n = x.shape
    v = values.to(x.dtype).contiguous()
    d = v.shape[-1]
    vstride = 0 if v.dim() == 2 else n * d
    if v.dim() == 3:
        assert v.shape[0] == R, "per-row values need one [L, d] block per logits row"
    b = None if logit_bias is None else logit_bias.to(x.dtype).contiguous()
    m = torch.empty(R, dtype=x.dtype, device=x.device)
    l = torch.empty_like(m)
    o = torch.empty(R, d, dtype=x.dtype, device=x.device)
    L.check(L.lib().dcc_online_softmax_from_attention(
        x.data_ptr(), v.data_ptr(), L.ptr(b), R, n, d, vstride, L.dtype_code(x), m.data_ptr(),
        l.data_ptr(), o.data_ptr(), L.stream_ptr(x.device)), "online_softmax_from_attention")
    if single:
        return OnlineSoftmaxState(m=m[0], l=l[0], o=o[0])
    return OnlineSoftmaxState(m=m, l=l, o=o)


def merge_softmax_states(state_a: OnlineSoftmaxState, state_b: OnlineSoftmaxState) -> OnlineSoftmaxState:
    """online_softmax.py:92-111: m = max, l and o rescaled and summed."""
    L.require_cuda(state_a.o, state_b.o)
    dtype = state_a.o.dtype
    ma = state_a.m.to(dtype).reshape(-1).contiguous()
    la = state_a.l.to(dtype).reshape(-1).contiguous()
    mb = state_b.m.to(dtype).reshape(-1).contiguous()
    lb = state_b.l.to(dtype).reshape(-1).contiguous()
    d = state_a.o.shape[-1]
    oa = state_a.o.reshape(-1, d).contiguous()
    ob = state_b.o.to(dtype).reshape(-1, d).contiguous()
    R = oa.shape[0]
    assert ma.numel() == R and mb.numel() == R and ob.shape[0] == R, "state shapes differ"
    m = torch.empty_like(ma)
    l = torch.empty_like(la)
    o = torch.empty_like(oa)
    L.check(L.lib().dcc_merge_softmax_states(
        ma.data_ptr(), la.data_ptr(), oa.data_ptr(), mb.data_ptr(), lb.data_ptr(), ob.data_ptr(), R, d,
        L.dtype_code(oa), m.data_ptr(), l.data_ptr(), o.data_ptr(), L.stream_ptr(oa.device)),
        "merge_softmax_states")
    shape = state_a.m.shape
    return OnlineSoftmaxState(m=m.reshape(shape), l=l.reshape(shape), o=o.reshape(state_a.o.shape))


def merge_softmax_states_list(states: List[OnlineSoftmaxState]) -> OnlineSoftmaxState:
    """online_softmax.py:114-123 (left fold)."""
    if len(states) == 0:
        raise ValueError("Empty state list")
    result = states[0]
    for s in states[1:]:
        result = merge_softmax_states(result, s)
    return result


def attention_output_from_state(state: OnlineSoftmaxState) -> torch.Tensor:
    """online_softmax.py:164-166: o / l."""
    return state.o / state.l.unsqueeze(-1) if state.o.dim() > state.l.dim() else state.o / state.l


def verify_order_invariance(states: List[OnlineSoftmaxState], n_trials: int = 10, seed: int = 42) -> bool:
    """online_softmax.py:126-161: merge under random permutations (host
    torch.Generator, as the reference) and compare o / l."""
    if len(states) < 2:
        return True
    g = torch.Generator().manual_seed(seed)
    ref = attention_output_from_state(merge_softmax_states_list(states))
    for _ in range(n_trials):
        perm = torch.randperm(len(states), generator=g).tolist()
        out = attention_output_from_state(merge_softmax_states_list([states[i] for i in perm]))
        if not torch.allclose(ref, out, atol=1e-5, rtol=1e-5):
            return False
    return True


def merge_lse(outputs: Sequence[torch.Tensor], lses: Sequence[torch.Tensor],
              out: Optional[torch.Tensor] = None, lse_out: Optional[torch.Tensor] = None,
              want_lse: bool = True) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
    """P-way merge of normalised partial attention outputs ``outputs[p]``
    [..., D] with log-sum-exp ``lses[p]`` [...] (float32): the (m=lse, l=1,
    o=O) form of merge_softmax_states folded over P states.  Returns (O, LSE)."""
    if len(outputs) != len(lses) or len(outputs) == 0:
        raise ValueError("need one LSE per partial output")
    L.require_cuda(*outputs, *lses)
    o0 = outputs[0]
    D = o0.shape[-1]
    R = o0.numel() // D
    parts = [o.contiguous() for o in outputs]
    ls = [x.to(torch.float32).contiguous() for x in lses]
    for o, x in zip(parts, ls):
        if o.shape != o0.shape or x.numel() != R or o.dtype != o0.dtype:
            raise ValueError("partial outputs must share shape and dtype")
    if out is None:
        out = torch.empty_like(parts[0])
    if want_lse and lse_out is None:
        lse_out = torch.empty(o0.shape[:-1], dtype=torch.float32, device=o0.device)
    n = len(parts)
    optrs = (L.C.c_void_p * n)(*[o.data_ptr() for o in parts])
    lptrs = (L.C.c_void_p * n)(*[x.data_ptr() for x in ls])
    L.check(L.lib().dcc_merge_lse(optrs, lptrs, n, R, D, L.dtype_code(o0), out.data_ptr(),
                                  L.ptr(lse_out) if want_lse else None, L.stream_ptr(o0.device)), "merge_lse")
    return out, (lse_out if want_lse else None)
