"""Representative-query pooling on the GPU.

Mirrors ``src/dcc_kv_ref/representative_query.py``: Rademacher projection
(host mt19937 draw, bit-identical to torch's CPU generator), double
normalisation and FP64 farthest-point sampling in ``libdcckv.so``.
"""
from __future__ import annotations

import ctypes as C
from typing import Tuple

import torch

from . import _lib as L


def rademacher_projection(queries: torch.Tensor, projection_dim: int = 32, seed: int = 42) -> torch.Tensor:
    """representative_query.py:10-31: P [d_p, d] = (2 randint{0,1} - 1) / sqrt(d_p),
    float32, on the queries' device."""
    d = int(queries.shape[-1])
    buf = (C.c_float * (projection_dim * d))()
    L.check(L.lib().dcc_rademacher_projection(d, projection_dim, seed, buf), "rademacher_projection")
    p = torch.frombuffer(bytearray(buf), dtype=torch.float32).reshape(projection_dim, d)
    return p.to(queries.device)


def farthest_point_sampling(features: torch.Tensor, num_samples: int, seed: int = 42) -> torch.Tensor:
    """representative_query.py:34-79 -> int64 indices [min(num_samples, N)]."""
    assert features.dim() == 2, "features must be [N, d]"
    L.require_cuda(features)
    f = features.contiguous()
    n, dim = f.shape
    k = min(num_samples, n)
    idx = torch.empty(k, dtype=torch.int64, device=f.device)
    ws = L.workspace(L.lib().dcc_farthest_point_sampling_workspace_bytes(n, dim), f.device)
    L.check(L.lib().dcc_farthest_point_sampling(f.data_ptr(), n, dim, num_samples, seed, L.dtype_code(f),
                                                idx.data_ptr(), ws.data_ptr(), ws.numel(),
                                                L.stream_ptr(f.device)), "farthest_point_sampling")
    return idx


def query_set(queries: torch.Tensor, out_repr: torch.Tensor, out_idx: torch.Tensor,
              n_seg: int = 1, seg_rows: int = None, seg_stride: int = 0, row_stride: int = None,
              base: torch.Tensor = None) -> L.dcc_query_set:
    """Descriptor of one destination query set (see include/dcc_kv.h)."""
    s = L.dcc_query_set()
    s.queries = (base if base is not None else queries).data_ptr()
    s.seg_rows = seg_rows if seg_rows is not None else queries.shape[0]
    s.seg_stride = seg_stride
    s.row_stride = row_stride if row_stride is not None else queries.shape[-1]
    s.n_seg = n_seg
    s.out_repr = out_repr.data_ptr()
    s.out_idx = out_idx.data_ptr()
    return s


def select_query_sets(sets, head_dim: int, num_samples: int, projection_dim: int, seed: int,
                      dtype_code: int, device: torch.device) -> None:
    """Batched launch over query-set descriptors (one FPS cluster per set)."""
    n = len(sets)
    if n == 0:
        return
    arr = (L.dcc_query_set * n)(*sets)
    nbytes = L.lib().dcc_select_representative_queries_workspace_bytes(arr, n, head_dim, projection_dim)
    ws = L.workspace(nbytes, device)
    L.check(L.lib().dcc_select_representative_queries(arr, n, head_dim, num_samples, projection_dim, seed,
                                                      dtype_code, ws.data_ptr(), ws.numel(),
                                                      L.stream_ptr(device)), "select_representative_queries")


def select_representative_queries(queries: torch.Tensor, num_samples: int = 64, projection_dim: int = 32,
                                  seed: int = 42) -> Tuple[torch.Tensor, torch.Tensor]:
    """representative_query.py:82-110 -> (queries[idx], idx)."""
    assert queries.dim() == 2, "queries must be [N, d]"
    L.require_cuda(queries)
    q = queries.contiguous()
    n, d = q.shape
    k = min(num_samples, n)
    rep = torch.empty(k, d, dtype=q.dtype, device=q.device)
    idx = torch.empty(k, dtype=torch.int64, device=q.device)
    select_query_sets([query_set(q, rep, idx)], d, num_samples, projection_dim, seed, L.dtype_code(q), q.device)
    return rep, idx
