"""Compact-value ridge regression on the GPU (``src/dcc_kv_ref/value_regression.py``)."""
from __future__ import annotations

import torch

from . import _lib as L
from .calibration import side_dtype


def ridge_regression_value(X: torch.Tensor, Y: torch.Tensor, lambda_reg: float = 1e-3) -> torch.Tensor:
    """value_regression.py:15-35: (X^T X + lam I)^-1 X^T Y, X [M, B], Y [M, D]."""
    assert X.dim() == 2 and Y.dim() == 2 and X.shape[0] == Y.shape[0]
    L.require_cuda(X, Y)
    x = X.contiguous()
    y = Y.to(x.dtype).contiguous()
    m, b = x.shape
    dd = y.shape[1]
    out = torch.empty(b, dd, dtype=x.dtype, device=x.device)
    ws = L.workspace(L.lib().dcc_ridge_workspace_bytes(m, b, dd), x.device)
    L.check(L.lib().dcc_ridge_regression_value(x.data_ptr(), y.data_ptr(), m, b, dd, lambda_reg, L.dtype_code(x),
                                               out.data_ptr(), ws.data_ptr(), ws.numel(), L.stream_ptr(x.device)),
            "ridge_regression_value")
    return out


def fit_compact_value(representative_queries: torch.Tensor, original_keys: torch.Tensor,
                      original_values: torch.Tensor, compact_keys: torch.Tensor, logit_bias: torch.Tensor,
                      lambda_reg: float = 1e-3) -> torch.Tensor:
    """value_regression.py:38-78: Y = softmax(Q^K^T/sqrt d) V,
    X = softmax(Q^C_K^T/sqrt d + beta/M), C_V = ridge(X, Y)."""
    L.require_cuda(representative_queries, original_keys, original_values, compact_keys, logit_bias)
    k = original_keys.contiguous()
    v = original_values.to(k.dtype).contiguous()
    ck = compact_keys.to(k.dtype).contiguous()
    rq = representative_queries.to(k.dtype).contiguous()
    beta = logit_bias.to(side_dtype(k)).contiguous()
    ls, d = k.shape
    dv = v.shape[1]
    m = rq.shape[0]
    b = ck.shape[0]
    out = torch.empty(b, dv, dtype=k.dtype, device=k.device)
    code = L.dtype_code(k)
    ws = L.workspace(L.lib().dcc_stage_workspace_bytes(ls, m, b, d, dv, code), k.device)
    L.check(L.lib().dcc_fit_compact_value(rq.data_ptr(), k.data_ptr(), v.data_ptr(), ck.data_ptr(), beta.data_ptr(),
                                          ls, m, b, d, dv, lambda_reg, code, out.data_ptr(), ws.data_ptr(),
                                          ws.numel(), L.stream_ptr(k.device)), "fit_compact_value")
    return out
