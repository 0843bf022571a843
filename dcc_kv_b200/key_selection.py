"""RMS-of-attention key selection on the GPU (``src/dcc_kv_ref/key_selection.py``)."""
from __future__ import annotations

from typing import Tuple

import torch

from . import _lib as L


def rms_per_token_score(attention_weights: torch.Tensor) -> torch.Tensor:
    """key_selection.py:14-26: u_j = sqrt(sum_a A_aj^2 / M), A [M, L] -> [L]."""
    assert attention_weights.dim() == 2, "attention_weights must be [M, L]"
    L.require_cuda(attention_weights)
    a = attention_weights.contiguous()
    m, n = a.shape
    out = torch.empty(n, dtype=a.dtype, device=a.device)
    L.check(L.lib().dcc_rms_per_token_score(a.data_ptr(), m, n, L.dtype_code(a), out.data_ptr(),
                                            L.stream_ptr(a.device)), "rms_per_token_score")
    return out


def select_topk_keys(keys: torch.Tensor, representative_queries: torch.Tensor,
                     budget: int) -> Tuple[torch.Tensor, torch.Tensor]:
    """key_selection.py:29-62: the budget keys with the largest RMS attention
    over the representative queries, sorted by score (desc); every key in
    original order when budget >= L_s."""
    assert keys.dim() == 2 and representative_queries.dim() == 2
    L.require_cuda(keys, representative_queries)
    ls, d = keys.shape
    if budget >= ls:  # reference early exit (:48-49)
        return keys, torch.arange(ls, device=keys.device)
    k = keys.contiguous()
    rq = representative_queries.to(k.dtype).contiguous()
    m = rq.shape[0]
    out_k = torch.empty(budget, d, dtype=k.dtype, device=k.device)
    out_i = torch.empty(budget, dtype=torch.int64, device=k.device)
    code = L.dtype_code(k)
    ws = L.workspace(L.lib().dcc_stage_workspace_bytes(ls, m, budget, d, d, code), k.device)
    L.check(L.lib().dcc_select_topk_keys(k.data_ptr(), rq.data_ptr(), ls, d, m, budget, code, out_k.data_ptr(),
                                         out_i.data_ptr(), ws.data_ptr(), ws.numel(), L.stream_ptr(k.device)),
            "select_topk_keys")
    return out_k, out_i
