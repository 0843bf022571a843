"""Shared-compaction baselines on the GPU (src/baselines/fast_kv_cpu.py,
src/baselines/apb_cpu.py): the comparison points of the DCC-KV paper, built
from the same kernels as the DCC-KV path.

* FastKV: every source chunk is compacted once (``build_compact_kv`` with ALL
  queries as destination queries), and every later query attends to the
  same compacts with their logit bias.
* APB: every source chunk keeps the ``anchor_budget`` keys with the largest
  attention mass from the queries at and after the chunk (no bias).

Both then run "ring attention" over the per-chunk compacts with the
reference's causal rule: query r sees the first r + 1 - offset_s entries of
chunk s's compact (fast_kv_cpu.py:96-104, apb_cpu.py:121-128), and the
per-chunk partials are merged by online softmax.  On the GPU that rule is a
causal KV segment over the queries from offset_s on; the merge is the P-way
LSE merge.  Single head, [L, d] tensors on one device, as the reference.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional, Sequence, Tuple

import torch

from . import _lib as L
from .attention import attention
from .compact_kv import build_compact_kv
from .online_softmax import merge_lse


@dataclass
class FastKVConfig:
    """fast_kv_cpu.py:24-32."""
    budget: int = 256
    num_repr_queries: int = 64
    projection_dim: int = 32
    lambda_beta: float = 1e-3
    lambda_value: float = 1e-3
    seed: int = 42


@dataclass
class APBConfig:
    """apb_cpu.py:29-33 (num_anchor_queries is kept for the interface; the
    reference does not use it either)."""
    anchor_budget: int = 128
    num_anchor_queries: int = 32


def _chunk_bounds(total: int, chunk_size: int, world_size: int) -> List[Tuple[int, int]]:
    """Chunk s = [s * chunk, (s + 1) * chunk); the last one runs to the end."""
    return [(s * chunk_size, (s + 1) * chunk_size if s < world_size - 1 else total) for s in range(world_size)]


def _ring_over_compacts(queries: torch.Tensor, compacts: Sequence[Tuple[torch.Tensor, torch.Tensor,
                                                                        Optional[torch.Tensor]]],
                        offsets: Sequence[int], causal: bool) -> torch.Tensor:
    """Merge, per query row, one attention state per visible chunk."""
    T, _ = queries.shape
    dv = compacts[0][1].shape[-1]
    outs, lses = [], []
    for (k, v, bias), off in zip(compacts, offsets):
        o = torch.zeros(T, dv, dtype=queries.dtype, device=queries.device)
        lse = torch.full((T,), float("-inf"), dtype=torch.float32, device=queries.device)
        seg = [(k[None], v[None], None if bias is None else bias[None])]
        if causal:
            if off >= T:
                continue
            # row r >= off sees compact entries j <= r - off
            po, pl = attention(queries[off:][None], seg, causal=True, causal_offset=0)
            o[off:] = po[0]
            lse[off:] = pl[0]
        else:
            po, pl = attention(queries[None], seg)
            o, lse = po[0], pl[0]
        outs.append(o)
        lses.append(lse)
    out, _ = merge_lse(outs, lses, want_lse=False)
    return out


def fast_kv(queries: torch.Tensor, keys: torch.Tensor, values: torch.Tensor, chunk_size: int, world_size: int,
            config: Optional[FastKVConfig] = None, causal: bool = True) -> torch.Tensor:
    """fast_kv_cpu.py:35-125 on the GPU: queries / keys / values [L, d]."""
    cfg = config if config is not None else FastKVConfig()
    L.require_cuda(queries, keys, values)
    T = queries.shape[0]
    compacts, offsets = [], []
    for lo, hi in _chunk_bounds(T, chunk_size, world_size):
        c = build_compact_kv(keys[lo:hi], values[lo:hi], queries, min(cfg.budget, hi - lo),
                             num_representative_queries=cfg.num_repr_queries, projection_dim=cfg.projection_dim,
                             lambda_beta=cfg.lambda_beta, lambda_value=cfg.lambda_value, seed=cfg.seed)
        compacts.append((c.keys, c.values, c.logit_bias))
        offsets.append(lo)
    return _ring_over_compacts(queries, compacts, offsets, causal)


def select_anchor_blocks(keys: torch.Tensor, values: torch.Tensor, queries: torch.Tensor,
                         budget: int) -> Tuple[torch.Tensor, torch.Tensor]:
    """apb_cpu.py:36-61: the ``budget`` keys of largest attention mass
    m_j = sum_a softmax(q_a K^T / sqrt(d))_j.  Two attention launches: the
    row log-sum-exps lse_a of the queries over the keys, then the keys over
    the queries with per-key bias -lse_a, whose log-sum-exp is log m_j."""
    L.require_cuda(keys, values, queries)
    _, lse = attention(queries[None], [(keys[None], keys[None], None)])
    _, lmass = attention(keys[None], [(queries[None], queries[None], -lse)])
    idx = torch.topk(lmass[0], budget).indices  # log is monotone: same order as the mass
    return keys[idx], values[idx]


def apb(queries: torch.Tensor, keys: torch.Tensor, values: torch.Tensor, chunk_size: int, world_size: int,
        config: Optional[APBConfig] = None, causal: bool = True) -> torch.Tensor:
    """apb_cpu.py:64-152 on the GPU: queries / keys / values [L, d]."""
    cfg = config if config is not None else APBConfig()
    L.require_cuda(queries, keys, values)
    T = queries.shape[0]
    compacts, offsets = [], []
    for lo, hi in _chunk_bounds(T, chunk_size, world_size):
        fut = queries[lo:] if T - lo > 0 else queries
        ak, av = select_anchor_blocks(keys[lo:hi], values[lo:hi], fut, min(cfg.anchor_budget, hi - lo))
        compacts.append((ak, av, None))
        offsets.append(lo)
    return _ring_over_compacts(queries, compacts, offsets, causal)


# ---------------------------------------------------------------------------
# Ring attention (src/baselines/ring_attention_cpu.py): exact attention over
# the whole context, chunk by chunk, merged by online softmax.
# ---------------------------------------------------------------------------
def ring_attention(queries: torch.Tensor, keys_chunks: Sequence[torch.Tensor],
                   values_chunks: Sequence[torch.Tensor], causal: bool = True) -> torch.Tensor:
    """ring_attention_cpu.py:24-82 on one GPU: queries [L, d_h] see the
    concatenated chunks (row r the keys at positions <= r when causal) -- one
    attention launch over the chunks as KV segments (causal on the
    concatenation), the same online softmax the reference folds per chunk."""
    L.require_cuda(queries, *keys_chunks, *values_chunks)
    k = torch.cat(list(keys_chunks), dim=0)
    v = torch.cat(list(values_chunks), dim=0)
    o, _ = attention(queries[None], [(k[None], v[None], None)], causal=causal)
    return o[0]


def dist_ring_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, group=None,
                        causal: bool = True) -> torch.Tensor:
    """Ring attention over NCCL: rank s holds chunk s (q, k, v [L_s, d] with
    equal L_s on every rank).  Step i attends the local queries to the chunk
    of rank s - i (causal for i = 0, skipped for later chunks when causal)
    while the next chunk travels one hop around the ring (batched isend /
    irecv on a side stream); the partials are merged by one P-way LSE merge.
    Every rank takes the same communication steps."""
    import torch.distributed as dist
    L.require_cuda(q, k, v)
    rank, world = dist.get_rank(group), dist.get_world_size(group)
    dev = q.device
    main = torch.cuda.current_stream(dev)
    comm = torch.cuda.Stream(device=dev)
    cur = torch.cat([k, v], dim=1).contiguous()  # one buffer per hop: [L_s, d_k + d_v]
    nxt = torch.empty_like(cur)
    dk = k.shape[1]
    outs, lses = [], []
    nxt_rank, prv_rank = (rank + 1) % world, (rank - 1) % world
    if group is not None:
        nxt_rank = dist.get_global_rank(group, nxt_rank)
        prv_rank = dist.get_global_rank(group, prv_rank)
    for i in range(world):
        src = (rank - i) % world
        reqs = []
        if i + 1 < world:
            comm.wait_stream(main)  # cur is complete, nxt is free
            with torch.cuda.stream(comm):
                ops = [dist.P2POp(dist.isend, cur, nxt_rank, group), dist.P2POp(dist.irecv, nxt, prv_rank, group)]
                reqs = dist.batch_isend_irecv(ops)
        if not causal or src <= rank:
            seg = [(cur[None, :, :dk], cur[None, :, dk:], None)]
            o, lse = attention(q[None], seg, causal=causal and src == rank)
            outs.append(o[0])
            lses.append(lse[0])
        for r in reqs:
            r.wait()
        if i + 1 < world:
            main.wait_stream(comm)
            cur, nxt = nxt, cur
    out, _ = merge_lse(outs, lses, want_lse=False)
    return out
