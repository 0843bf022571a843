"""CompactKV and the compact-KV build on the GPU (``src/dcc_kv_ref/compact_kv.py``).

``build_compact_kv`` keeps the reference signature and runs the four stages
as one stream-ordered kernel sequence: FP64 FPS pooling, two streaming
scoring passes (row statistics; probabilities -> RMS scores, block mass and
Y = A V), radix top-k + C_K gather, and the FP64 beta / value solves.

dtype modes: float32 / float64 inputs compute every reduction in FP64 (the
parity path); bfloat16 inputs score with fp32 accumulation and keep the
solves in FP64.  ``logit_bias`` is float64 for float64 inputs and float32
otherwise; keys and values keep the input dtype.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional, Sequence

import torch

from . import _lib as L
from .calibration import side_dtype


@dataclass(frozen=True)
class CompactKV:
    """A destination-conditioned compact representation of one source KV block
    (compact_kv.py:24-47): keys [B, d_h], logit_bias [B], values [B, d_v],
    selected_indices [B] (int64, into the source block)."""
    keys: torch.Tensor
    logit_bias: torch.Tensor
    values: torch.Tensor
    selected_indices: torch.Tensor

    def __post_init__(self):
        assert self.keys.dim() == 2, f"keys must be 2D [budget, head_dim], got {self.keys.dim()}D"
        assert self.logit_bias.dim() == 1, f"logit_bias must be 1D, got {self.logit_bias.dim()}D"
        assert self.values.dim() == 2, f"values must be 2D, got {self.values.dim()}D"
        assert self.selected_indices.dim() == 1, \
            f"selected_indices must be 1D, got {self.selected_indices.dim()}D"
        B = self.keys.shape[0]
        assert self.logit_bias.shape[0] == B
        assert self.values.shape[0] == B
        assert self.selected_indices.shape[0] == B


def build_compact_kv(source_keys: torch.Tensor, source_values: torch.Tensor,
                     destination_queries: torch.Tensor, budget: int,
                     num_representative_queries: int = 64, projection_dim: int = 32,
                     lambda_beta: float = 1e-3, lambda_value: float = 1e-3,
                     seed: int = 42) -> CompactKV:
    """compact_kv.py:50-118 on one head: source_keys [L_s, d_h],
    source_values [L_s, d_v], destination_queries [L_r, d_h]."""
    assert source_keys.dim() == 2 and source_values.dim() == 2 and destination_queries.dim() == 2
    assert source_keys.shape[0] == source_values.shape[0], "keys/values length mismatch"
    assert destination_queries.shape[1] == source_keys.shape[1], "query/key head_dim mismatch"
    L.require_cuda(source_keys, source_values, destination_queries)
    k = source_keys.contiguous()
    v = source_values.to(k.dtype).contiguous()
    q = destination_queries.to(k.dtype).contiguous()
    ls, d = k.shape
    dv = v.shape[1]
    lr = q.shape[0]
    if budget <= 0:
        raise ValueError("budget must be positive")
    bp = min(budget, ls)
    dev = k.device
    out_k = torch.empty(bp, d, dtype=k.dtype, device=dev)
    out_v = torch.empty(bp, dv, dtype=k.dtype, device=dev)
    out_b = torch.empty(bp, dtype=side_dtype(k), device=dev)
    out_i = torch.empty(bp, dtype=torch.int64, device=dev)
    code = L.dtype_code(k)
    nbytes = L.lib().dcc_build_compact_kv_workspace(ls, lr, d, dv, budget, num_representative_queries,
                                                    projection_dim, code)
    ws = L.workspace(nbytes, dev)
    L.check(L.lib().dcc_build_compact_kv(
        k.data_ptr(), v.data_ptr(), q.data_ptr(), ls, lr, d, dv, budget, num_representative_queries,
        projection_dim, lambda_beta, lambda_value, seed, code, out_k.data_ptr(), out_b.data_ptr(),
        out_v.data_ptr(), out_i.data_ptr(), None, ws.data_ptr(), ws.numel(), L.stream_ptr(dev)),
        "build_compact_kv")
    return CompactKV(keys=out_k, logit_bias=out_b, values=out_v, selected_indices=out_i)


def build_problem(keys: torch.Tensor, values: torch.Tensor, repr_q: torch.Tensor, budget: int,
                  out_keys: torch.Tensor, out_values: torch.Tensor, out_bias: torch.Tensor,
                  out_idx: torch.Tensor, num_repr: Optional[int] = None,
                  out_mass: Optional[torch.Tensor] = None) -> L.dcc_build_problem:
    """Descriptor of one (source, destination, KV head) edge.  ``keys`` /
    ``values`` are [L_s, d] views with unit column stride; outputs may be
    views into larger buffers (rows contiguous)."""
    p = L.dcc_build_problem()
    p.keys = keys.data_ptr()
    p.values = values.data_ptr()
    p.repr = repr_q.data_ptr()
    p.L_s = keys.shape[0]
    p.ld_k = keys.stride(0)
    p.ld_v = values.stride(0)
    p.budget = budget
    p.num_repr = num_repr if num_repr is not None else repr_q.shape[0]
    p.out_keys = out_keys.data_ptr()
    p.out_values = out_values.data_ptr()
    p.out_bias = out_bias.data_ptr()
    p.out_idx = out_idx.data_ptr()
    p.out_mass = None if out_mass is None else out_mass.data_ptr()
    return p


def build_launch_count(n_problems: int, dtype_code: int, head_dim: int) -> int:
    """Kernel launches of one batched build (C-library batch caps: 128 edges per
    flush; tcgen05 scoring 56 edges per launch; 3 calibration launches)."""
    n, total = n_problems, 0
    while n > 0:
        k = min(n, 128)
        scoring = 2 * -(-k // 56) if (dtype_code == L.DCC_BF16 and head_dim == 128) else 2
        total += scoring + 1 + 3
        n -= k
    return total


def run_build_problems(problems: Sequence[L.dcc_build_problem], head_dim: int, value_dim: int,
                       lambda_beta: float, lambda_value: float, dtype_code: int, device: torch.device,
                       workspace: Optional[torch.Tensor] = None) -> None:
    """One batched build launch sequence over edge descriptors."""
    n = len(problems)
    if n == 0:
        return
    arr = (L.dcc_build_problem * n)(*problems)
    need = L.lib().dcc_build_compact_kv_workspace_bytes(arr, n, head_dim, value_dim, dtype_code)
    if workspace is None or workspace.numel() < need:
        workspace = L.workspace(need, device)
    L.check(L.lib().dcc_build_compact_kv_batched(arr, n, head_dim, value_dim, lambda_beta, lambda_value, dtype_code,
                                                 workspace.data_ptr(), workspace.numel(), L.stream_ptr(device)),
            "build_compact_kv_batched")


def build_compact_kv_batched(source_keys: torch.Tensor, source_values: torch.Tensor,
                             repr_queries: torch.Tensor, budget: int, lambda_beta: float = 1e-3,
                             lambda_value: float = 1e-3) -> List[CompactKV]:
    """GQA batch: source_keys/values [H_kv, L_s, d], repr_queries [H_kv, M, d]
    (one set per KV head) -> one CompactKV per KV head."""
    assert source_keys.dim() == 3 and repr_queries.dim() == 3
    L.require_cuda(source_keys, source_values, repr_queries)
    k = source_keys.contiguous()
    v = source_values.to(k.dtype).contiguous()
    rq = repr_queries.to(k.dtype).contiguous()
    h, ls, d = k.shape
    dv = v.shape[2]
    bp = min(budget, ls)
    dev = k.device
    ok = torch.empty(h, bp, d, dtype=k.dtype, device=dev)
    ov = torch.empty(h, bp, dv, dtype=k.dtype, device=dev)
    ob = torch.empty(h, bp, dtype=side_dtype(k), device=dev)
    oi = torch.empty(h, bp, dtype=torch.int64, device=dev)
    probs = [build_problem(k[i], v[i], rq[i], budget, ok[i], ov[i], ob[i], oi[i]) for i in range(h)]
    run_build_problems(probs, d, dv, lambda_beta, lambda_value, L.dtype_code(k), dev)
    return [CompactKV(ok[i], ob[i], ov[i], oi[i]) for i in range(h)]
