"""The DCC-KV sync layer as an attention backend of Hugging Face transformers.

This is the model-integration step the reference plans for its end-to-end
test (tests/gpu/test_end_to_end_8b.py:33-109, where the DCC-KV case is left
deferred): a Llama prefill whose RoPE'd queries and keys go through DCC-KV
instead of full attention.

    import dcc_kv_b200.hf_attention as ha
    ha.register_dcc_kv_attention(n_blocks=8, budgets=1024, window=2048)
    model = AutoModelForCausalLM.from_pretrained(path, torch_dtype=torch.bfloat16,
                                                 attn_implementation="dcc_kv").cuda()
    logits = model(input_ids, use_cache=False).logits   # input_ids [1, n_blocks * L]

Every attention layer of the prefill then runs ``DccKvSyncLayer``: the
sequence is split into ``n_blocks`` logical blocks of equal length; block r
attends causally to its own keys and to the compact KV C_{s->r} of every
earlier block s, built from r's destination queries (dcc_kv_sync_cpu.py:
52-84).  The layer is causal by construction, so the attention mask that
transformers would build is not needed (it passes none to a registered
backend).  Only a batch-1 prefill is supported: a batch above 1, keys that
include cached earlier tokens, dropout, a scaling other than 1/sqrt(head_dim)
or a length that does not split into ``n_blocks`` equal blocks raise
ValueError -- there is no fallback to another attention.
"""
from __future__ import annotations

import math
from typing import Dict, Optional, Tuple

import torch

from .layer import Budgets, DccKvSyncLayer

NAME = "dcc_kv"

_settings: Optional[dict] = None
_layers: Dict[tuple, "_Backend"] = {}


class _Backend:
    """One DccKvSyncLayer per attention shape, with fixed block-major input
    buffers (so its kernel descriptors are built once and reused by every
    decoder layer of the model)."""

    def __init__(self, nb: int, L: int, hq: int, hkv: int, d: int, dtype: torch.dtype, device: torch.device,
                 settings: dict):
        self.layer = DccKvSyncLayer(nb, L, hq, hkv, d, settings["budgets"], settings["window"],
                                    settings["num_representative_queries"], settings["projection_dim"],
                                    dtype=dtype, device=device)
        self.q = torch.empty(nb, hq, L, d, dtype=dtype, device=device)
        self.k = torch.empty(nb, hkv, L, d, dtype=dtype, device=device)
        self.v = torch.empty(nb, hkv, L, d, dtype=dtype, device=device)


def register_dcc_kv_attention(n_blocks: int, budgets: Budgets, window: int, num_representative_queries: int = 64,
                              projection_dim: int = 32, name: str = NAME) -> str:
    """Register the backend with transformers under ``name`` and set the
    layer's parameters (logical blocks per sequence, compact budget per
    edge -- an int or {(s, r): B} --, destination window).  Returns the name
    to pass as ``attn_implementation``."""
    from transformers import AttentionInterface
    global _settings
    if n_blocks < 1:
        raise ValueError("n_blocks must be positive")
    _settings = dict(n_blocks=n_blocks, budgets=budgets, window=window,
                     num_representative_queries=num_representative_queries, projection_dim=projection_dim)
    _layers.clear()
    AttentionInterface.register(name, dcc_kv_attention_forward)
    return name


def _check(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor, scaling, dropout) -> Tuple[int, ...]:
    if _settings is None:
        raise RuntimeError("call register_dcc_kv_attention() before running a model with the dcc_kv backend")
    if query.dim() != 4 or key.dim() != 4 or value.shape != key.shape:
        raise ValueError("expected query [B, H_q, S, d] and key / value [B, H_kv, S, d]")
    b, hq, s, d = query.shape
    hkv = key.shape[1]
    if b != 1:
        raise ValueError(f"the dcc_kv backend runs a batch-1 prefill; got batch {b}")
    if key.shape[2] != s or key.shape[0] != 1 or key.shape[3] != d:
        raise ValueError("the dcc_kv backend runs a prefill: keys must be the query positions only "
                         "(run the model with use_cache=False)")
    if dropout:
        raise ValueError("the dcc_kv backend has no attention dropout")
    if scaling is not None and not math.isclose(float(scaling), d ** -0.5, rel_tol=1e-6):
        raise ValueError(f"the DCC-KV layer scales logits by 1/sqrt(head_dim); got {scaling}")
    nb = _settings["n_blocks"]
    if s % nb:
        raise ValueError(f"sequence length {s} does not split into {nb} equal blocks")
    if hq % hkv:
        raise ValueError("query heads must be a multiple of the KV heads")
    return nb, s // nb, hq, hkv, d


def dcc_kv_attention_forward(module, query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                             attention_mask: Optional[torch.Tensor], scaling: Optional[float] = None,
                             dropout: float = 0.0, **kwargs) -> Tuple[torch.Tensor, None]:
    """transformers attention-backend signature: query [1, H_q, S, d], key /
    value [1, H_kv, S, d] (RoPE applied) -> ([1, S, H_q, d], None)."""
    nb, L, hq, hkv, d = _check(query, key, value, scaling, dropout)
    dev = query.device
    sig = (nb, L, hq, hkv, d, query.dtype, dev)
    backend = _layers.get(sig)
    if backend is None:
        backend = _layers[sig] = _Backend(nb, L, hq, hkv, d, query.dtype, dev, _settings)
    # sequence-major [H, S, d] -> block-major [nb, H, L, d] in the fixed buffers
    backend.q.copy_(query[0].view(hq, nb, L, d).transpose(0, 1))
    backend.k.copy_(key[0].view(hkv, nb, L, d).transpose(0, 1))
    backend.v.copy_(value[0].view(hkv, nb, L, d).transpose(0, 1))
    out = backend.layer(backend.q, backend.k, backend.v)          # [nb, H_q, L, d]
    return out.permute(0, 2, 1, 3).reshape(1, nb * L, hq, d), None   # [1, S, H_q, d] (a copy)
