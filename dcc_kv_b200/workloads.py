"""Seeded synthetic inputs with the shapes and value distributions of the
benchmark configurations (no dataset is involved).

* merge microbench: 8 partial outputs [32, 4096, 128] ~ N(0,1) (bf16) with
  fp32 LSE ~ N(0,1) * 4;
* GQA build: 32 query / 8 KV heads, d = 128, K and V ~ N(0,1) with 4 outlier
  channels per KV head (randperm(128)[:4]) scaled x8, Q ~ N(0,1)/sqrt(128);
* layer: the context split into blocks of that geometry, block b drawn from
  seed 1000 + b.

``device="cuda"`` draws with a CUDA generator (fast, for the benchmark);
``device="cpu"`` draws with torch's CPU generator (for parity fixtures).
"""
from __future__ import annotations

from typing import Dict, Tuple

import torch


def _gen(seed: int, device: str) -> torch.Generator:
    return torch.Generator(device=device).manual_seed(seed)


def gqa_block(n_q_heads: int, n_kv_heads: int, length: int, head_dim: int, seed: int,
              dtype: torch.dtype = torch.bfloat16, device: str = "cpu", q_len: int = None):
    """One block: Q [H_q, q_len, d], K, V [H_kv, length, d]."""
    g = _gen(seed, device)
    q_len = length if q_len is None else q_len
    k = torch.randn(n_kv_heads, length, head_dim, generator=g, device=device)
    v = torch.randn(n_kv_heads, length, head_dim, generator=g, device=device)
    for h in range(n_kv_heads):
        ch = torch.randperm(head_dim, generator=g, device=device)[:4]
        k[h][:, ch] *= 8
        v[h][:, ch] *= 8
    q = torch.randn(n_q_heads, q_len, head_dim, generator=g, device=device) / head_dim ** 0.5
    return q.to(dtype), k.to(dtype), v.to(dtype)


def layer_inputs(n_blocks: int, block_len: int, n_q_heads: int = 32, n_kv_heads: int = 8,
                 head_dim: int = 128, dtype: torch.dtype = torch.bfloat16, device: str = "cuda",
                 first_seed: int = 1000):
    """q [nb, H_q, L, d], k / v [nb, H_kv, L, d], block b from seed first_seed + b."""
    qs, ks, vs = [], [], []
    for b in range(n_blocks):
        q, k, v = gqa_block(n_q_heads, n_kv_heads, block_len, head_dim, first_seed + b, dtype, device)
        qs.append(q)
        ks.append(k)
        vs.append(v)
    return torch.stack(qs), torch.stack(ks), torch.stack(vs)


def variable_budgets(n_blocks: int, choices=(256, 512, 1024, 2048), seed: int = 1) -> Dict[Tuple[int, int], int]:
    """Per-edge budgets drawn uniformly from ``choices`` in row-major (s, r), s < r."""
    g = torch.Generator().manual_seed(seed)
    out = {}
    for s in range(n_blocks):
        for r in range(s + 1, n_blocks):
            out[(s, r)] = int(choices[int(torch.randint(0, len(choices), (1,), generator=g))])
    return out


def merge_inputs(n_parts: int = 8, heads: int = 32, queries: int = 4096, head_dim: int = 128,
                 seed: int = 0, device: str = "cuda"):
    g = _gen(seed, device)
    outs, lses = [], []
    for _ in range(n_parts):
        outs.append(torch.randn(heads, queries, head_dim, generator=g, device=device).to(torch.bfloat16))
        lses.append(torch.randn(heads, queries, generator=g, device=device) * 4)
    return outs, lses
