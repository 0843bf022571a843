"""The DCC-KV sync layer on one GPU (all logical blocks resident).

Semantics (dcc_kv_sync_cpu.py:22-84 and compact_kv.py:50-118, in the
north-star direction): the context is split into ``n_blocks`` contiguous
blocks; block r attends causally to its own keys and, for every earlier
block s < r, to the compact KV C_{s->r} built from s's keys and values and
r's destination queries (per KV head: the first ``window`` queries of each
of its query heads, concatenated head by head), with the compact logit bias
added at full weight; the partial outputs are merged by online softmax.

Layout (HBM): block-major, head-major, contiguous --
    q [n_blocks, H_q, L, d], k / v [n_blocks, H_kv, L, d], out like q.
All buffers and kernel descriptors are built once per shape; ``forward``
only enqueues kernels on the current stream:
    1 projection + 1 FPS launch       (all (destination, KV head) sets)
    4 build launches per <=128 edges  (score stats, score probs, top-k, solves)
    1 attention launch: per block its causal local segment followed by its
      compact segment with the logit bias, one online softmax over both (the
      merge of dcc_kv_sync_cpu.py:81-84 happens inside the kernel)
"""
from __future__ import annotations

import math
from typing import Dict, Optional, Tuple, Union

import torch

from . import _lib as L
from .attention import attn_problem, kv_segment, run_attention
from .calibration import side_dtype
from .compact_kv import build_launch_count, build_problem, run_build_problems
from .representative_query import query_set, select_query_sets

Budgets = Union[int, Dict[Tuple[int, int], int]]


def budget_table(n_blocks: int, budgets: Budgets) -> Dict[Tuple[int, int], int]:
    if isinstance(budgets, int):
        return {(s, r): budgets for r in range(n_blocks) for s in range(r)}
    return {(s, r): int(budgets[(s, r)]) for r in range(n_blocks) for s in range(r)}


class DccKvSyncLayer:
    """One DCC-KV layer over ``n_blocks`` logical blocks on a single device."""

    def __init__(self, n_blocks: int, block_len: int, n_q_heads: int, n_kv_heads: int, head_dim: int,
                 budgets: Budgets, window: int, num_representative_queries: int = 64,
                 projection_dim: int = 32, lambda_beta: float = 1e-3, lambda_value: float = 1e-3,
                 seed: int = 42, dtype: torch.dtype = torch.bfloat16,
                 device: Union[str, torch.device] = "cuda"):
        if n_q_heads % n_kv_heads:
            raise ValueError("n_q_heads must be a multiple of n_kv_heads")
        if dtype not in (torch.float32, torch.bfloat16):
            raise ValueError("the layer runs in float32 (parity path) or bfloat16")
        self.nb, self.L, self.hq, self.hkv, self.d = n_blocks, block_len, n_q_heads, n_kv_heads, head_dim
        self.group = n_q_heads // n_kv_heads
        self.window = min(window, block_len)
        self.M = num_representative_queries
        self.m_eff = min(self.M, self.group * self.window)
        self.dp = projection_dim
        self.lb, self.lv, self.seed = lambda_beta, lambda_value, seed
        self.dtype = dtype
        self.code = L.dtype_code(torch.empty(0, dtype=dtype))
        self.device = torch.device(device)
        self.budgets = budget_table(n_blocks, budgets)
        dev, d = self.device, head_dim
        self.repr = torch.empty(n_blocks, n_kv_heads, self.m_eff, d, dtype=dtype, device=dev)
        self.repr_idx = torch.empty(n_blocks, n_kv_heads, self.m_eff, dtype=torch.int64, device=dev)
        # compact KV per destination r: the sources s < r concatenated, B' = min(B, L) rows each
        self.offsets: Dict[Tuple[int, int], int] = {}
        self.total = [0] * n_blocks
        for r in range(n_blocks):
            off = 0
            for s in range(r):
                self.offsets[(s, r)] = off
                off += min(self.budgets[(s, r)], block_len)
            self.total[r] = off
        sd = side_dtype(torch.empty(0, dtype=dtype))
        self.ck = [torch.empty(n_kv_heads, t, d, dtype=dtype, device=dev) for t in self.total]
        self.cv = [torch.empty(n_kv_heads, t, d, dtype=dtype, device=dev) for t in self.total]
        self.cb = [torch.empty(n_kv_heads, t, dtype=sd, device=dev) for t in self.total]
        self.ci = [torch.empty(n_kv_heads, t, dtype=torch.int64, device=dev) for t in self.total]
        self.out = torch.empty(n_blocks, n_q_heads, block_len, d, dtype=dtype, device=dev)
        self._bound = None
        self._ws = None
        # optional (start, end) CUDA events per step around the local-attention launch
        self.timing_events = None
        self.timing_index = 0

    # -- descriptors (rebuilt only when the input tensors change) ------------
    def _bind(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> None:
        key = (q.data_ptr(), k.data_ptr(), v.data_ptr())
        if self._bound == key:
            return
        g = self.group
        self.sets = []
        for r in range(1, self.nb):
            for h in range(self.hkv):
                self.sets.append(query_set(q[r, h * g], self.repr[r, h], self.repr_idx[r, h], n_seg=g,
                                           seg_rows=self.window, seg_stride=q.stride(1), row_stride=q.stride(2)))
        self.build = []
        for r in range(1, self.nb):
            for s in range(r):
                b = self.budgets[(s, r)]
                bp = min(b, self.L)
                o = self.offsets[(s, r)]
                for h in range(self.hkv):
                    self.build.append(build_problem(
                        k[s, h], v[s, h], self.repr[r, h], b, self.ck[r][h, o:o + bp], self.cv[r][h, o:o + bp],
                        self.cb[r][h, o:o + bp], self.ci[r][h, o:o + bp], num_repr=self.m_eff))
        n = len(self.build)
        if n:
            arr = (L.dcc_build_problem * n)(*self.build)
            need = L.lib().dcc_build_compact_kv_workspace_bytes(arr, n, self.d, self.d, self.code)
            self._ws = L.workspace(need, self.device)
        # one attention problem per block: its causal local segment, then (for r >= 1)
        # the concatenated compact blocks with their logit bias -- the online softmax
        # runs over both in one pass, so no separate merge is needed
        self.attn_problems = []
        for b in range(self.nb):
            segs = [kv_segment(k[b], v[b])]
            if b > 0 and self.total[b] > 0:
                segs.append(kv_segment(self.ck[b], self.cv[b], self.cb[b]))
            self.attn_problems.append(attn_problem(q[b], self.out[b], None, segs, causal=True))
        self._bound = key

    def check_inputs(self, q, k, v):
        L.require_cuda(q, k, v)
        exp_q = (self.nb, self.hq, self.L, self.d)
        exp_kv = (self.nb, self.hkv, self.L, self.d)
        if tuple(q.shape) != exp_q or tuple(k.shape) != exp_kv or tuple(v.shape) != exp_kv:
            raise ValueError(f"expected q {exp_q}, k/v {exp_kv}; got {tuple(q.shape)}, {tuple(k.shape)}, {tuple(v.shape)}")
        for t in (q, k, v):
            if t.dtype != self.dtype or not t.is_contiguous():
                raise ValueError(f"inputs must be contiguous {self.dtype}")

    def forward(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
        """q [nb, H_q, L, d], k / v [nb, H_kv, L, d] -> out [nb, H_q, L, d]
        (the returned tensor is an internal buffer, reused by the next call)."""
        self.check_inputs(q, k, v)
        self._bind(q, k, v)
        dev = self.device
        select_query_sets(self.sets, self.d, self.M, self.dp, self.seed, self.code, dev)
        run_build_problems(self.build, self.d, self.d, self.lb, self.lv, self.code, dev, self._ws)
        scale = 1.0 / math.sqrt(self.d)
        ev = self.timing_events[self.timing_index] if self.timing_events else None
        if ev is not None:
            ev[0].record(torch.cuda.current_stream(dev))
        run_attention(self.attn_problems, self.hq, self.hkv, self.d, scale, self.code, dev)
        if ev is not None:
            ev[1].record(torch.cuda.current_stream(dev))
        return self.out

    __call__ = forward

    def launches_per_forward(self) -> int:
        """Kernel launches one forward enqueues (batch caps of the C library:
        64 query sets, 96 build edges, 8 tcgen05 attention problems per launch)."""
        sets = len(self.sets)
        pool = 0 if sets == 0 else (2 if self.m_eff < self.group * self.window else 1) * -(-sets // 64)
        build = build_launch_count(len(self.build), self.code, self.d)
        attn = -(-len(self.attn_problems) // 8)
        return pool + build + attn

    def compact(self, s: int, r: int, h: int):
        """The CompactKV C_{s->r} of KV head h from the last forward."""
        from .compact_kv import CompactKV
        o = self.offsets[(s, r)]
        bp = min(self.budgets[(s, r)], self.L)
        return CompactKV(self.ck[r][h, o:o + bp], self.cb[r][h, o:o + bp], self.cv[r][h, o:o + bp],
                         self.ci[r][h, o:o + bp])
