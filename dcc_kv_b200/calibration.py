"""Logit-bias calibration on the GPU (``src/dcc_kv_ref/calibration.py``).

All arithmetic is FP64 inside the kernels: cond(G^T G + lam I) reaches 1e7 at
the production shapes.  Side vectors (block mass, logit bias) are float64 for
float64 inputs and float32 otherwise.
"""
from __future__ import annotations

import torch

from . import _lib as L


def side_dtype(t: torch.Tensor) -> torch.dtype:
    return torch.float64 if t.dtype == torch.float64 else torch.float32


def nonneg_least_squares(G: torch.Tensor, target: torch.Tensor, lambda_reg: float = 1e-3,
                         n_iter: int = 100) -> torch.Tensor:
    """calibration.py:17-60: w = clamp(solve(G^T G + lam I, G^T t), 0); when
    M >= B, ``n_iter`` projected-gradient steps (lr 1e-2, ridge toward 1)."""
    assert G.dim() == 2 and target.dim() == 1 and target.shape[0] == G.shape[0]
    L.require_cuda(G, target)
    g = G.contiguous()
    t = target.to(g.dtype).contiguous()
    m, b = g.shape
    w = torch.empty(b, dtype=g.dtype, device=g.device)
    ws = L.workspace(L.lib().dcc_nnls_workspace_bytes(m, b), g.device)
    L.check(L.lib().dcc_nonneg_least_squares(g.data_ptr(), t.data_ptr(), m, b, lambda_reg, n_iter,
                                             L.dtype_code(g), w.data_ptr(), ws.data_ptr(), ws.numel(),
                                             L.stream_ptr(g.device)), "nonneg_least_squares")
    return w


def fit_logit_bias(representative_queries: torch.Tensor, compact_keys: torch.Tensor,
                   original_block_mass: torch.Tensor, lambda_reg: float = 1e-3) -> torch.Tensor:
    """calibration.py:63-94: beta = log(max(NNLS(exp(Q^ C_K^T / sqrt d), mass), 1e-6))."""
    assert representative_queries.dim() == 2 and compact_keys.dim() == 2
    L.require_cuda(representative_queries, compact_keys, original_block_mass)
    ck = compact_keys.contiguous()
    rq = representative_queries.to(ck.dtype).contiguous()
    m, d = rq.shape
    b = ck.shape[0]
    sd = side_dtype(ck)
    mass = original_block_mass.to(sd).contiguous()
    beta = torch.empty(b, dtype=sd, device=ck.device)
    code = L.dtype_code(ck)
    ws = L.workspace(L.lib().dcc_stage_workspace_bytes(b, m, b, d, d, code), ck.device)
    L.check(L.lib().dcc_fit_logit_bias(rq.data_ptr(), ck.data_ptr(), mass.data_ptr(), m, b, d, lambda_reg, code,
                                       beta.data_ptr(), ws.data_ptr(), ws.numel(), L.stream_ptr(ck.device)),
            "fit_logit_bias")
    return beta
