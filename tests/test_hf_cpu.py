"""The transformers attention backend on CPU: registration and the argument
checks it makes before touching a GPU (no fallback: unsupported calls raise)."""
from __future__ import annotations

import pytest
import torch

transformers = pytest.importorskip("transformers")

import dcc_kv_b200.hf_attention as ha  # noqa: E402


def test_registration_and_argument_checks():
    from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS
    name = ha.register_dcc_kv_attention(n_blocks=4, budgets=64, window=32)
    assert name == "dcc_kv"
    assert ALL_ATTENTION_FUNCTIONS.get_interface("dcc_kv", None) is ha.dcc_kv_attention_forward
    q = torch.zeros(1, 8, 256, 32)
    kv = torch.zeros(1, 2, 256, 32)
    assert ha._check(q, kv, kv, 32 ** -0.5, 0.0) == (4, 64, 8, 2, 32)
    with pytest.raises(ValueError):  # batch above 1
        ha._check(torch.zeros(2, 8, 256, 32), torch.zeros(2, 2, 256, 32), torch.zeros(2, 2, 256, 32), None, 0.0)
    with pytest.raises(ValueError):  # keys include cached earlier tokens
        ha._check(q[:, :, :64], kv, kv, None, 0.0)
    with pytest.raises(ValueError):  # length does not split into 4 blocks
        ha._check(q[:, :, :250], kv[:, :, :250], kv[:, :, :250], None, 0.0)
    with pytest.raises(ValueError):  # the layer scales by 1/sqrt(d)
        ha._check(q, kv, kv, 0.5, 0.0)
    with pytest.raises(ValueError):
        ha._check(q, kv, kv, None, 0.1)
