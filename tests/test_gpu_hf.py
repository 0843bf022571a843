"""A Llama prefill through the DCC-KV attention backend (the model
integration the reference plans in tests/gpu/test_end_to_end_8b.py:33-109;
its weights are not available here, so the model has random weights with the
Llama-3.1-8B attention geometry: 32 query / 8 KV heads, head_dim 128, RoPE
theta 500000).  Two decoder layers, a 2048-token prefill as 4 blocks of 512:
the logits are finite, and the first layer's attention output -- computed by
the backend from the RoPE'd queries and keys the model produced -- matches
the FP64 oracle of the layer (dcc_kv_sync_cpu.py:52-84) on sampled rows of
every block within the bf16 bar 2e-2."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from gpu_util import assert_no_device_timeouts, dev, rel_err

pytestmark = pytest.mark.gpu
transformers = pytest.importorskip("transformers")


def test_llama_prefill_through_dcc_kv_backend():
    from transformers import AttentionInterface, LlamaConfig, LlamaForCausalLM
    import dcc_kv_b200.hf_attention as ha
    from oracle import dcc_kv_oracle as orc

    nb, L, budget, window = 4, 512, 128, 128
    ha.register_dcc_kv_attention(n_blocks=nb, budgets=budget, window=window)
    captured = []

    def recording(module, query, key, value, attention_mask, **kw):
        out, w = ha.dcc_kv_attention_forward(module, query, key, value, attention_mask, **kw)
        if module.layer_idx == 0:
            captured.append(tuple(t.detach().float().cpu() for t in (query, key, value, out)))
        return out, w

    AttentionInterface.register("dcc_kv_recording", recording)
    cfg = LlamaConfig(hidden_size=4096, intermediate_size=1024, num_hidden_layers=2, num_attention_heads=32,
                      num_key_value_heads=8, head_dim=128, vocab_size=1024, max_position_embeddings=8192,
                      rope_theta=500000.0)
    cfg._attn_implementation = "dcc_kv_recording"
    torch.manual_seed(0)
    model = LlamaForCausalLM(cfg).to(torch.bfloat16).to(dev()).eval()
    ids = torch.randint(0, 1024, (1, nb * L), generator=torch.Generator().manual_seed(1)).to(dev())
    with torch.no_grad():
        logits = model(ids, use_cache=False).logits
    torch.cuda.synchronize()
    assert_no_device_timeouts()
    assert torch.isfinite(logits).all()
    q, k, v, out = captured[0]          # [1, 32, S, d], [1, 8, S, d] x 2, [1, S, 32, d]
    group = 4
    rows = {b: np.array([0, 1, 100, L - 1]) for b in range(nb)}
    budgets = {(s, r): budget for r in range(nb) for s in range(r)}
    for g in (0, 7):
        qb = [q[0, g * group:(g + 1) * group, b * L:(b + 1) * L].numpy() for b in range(nb)]
        kb = [k[0, g:g + 1, b * L:(b + 1) * L].numpy() for b in range(nb)]
        vb = [v[0, g:g + 1, b * L:(b + 1) * L].numpy() for b in range(nb)]
        ref, _ = orc.layer_forward(qb, kb, vb, budgets, window, rows=rows)
        for b in range(nb):
            got = out[0, b * L + rows[b]][:, g * group:(g + 1) * group].permute(1, 0, 2).double().numpy()
            assert rel_err(got, ref[b]) < 2e-2, (g, b)
