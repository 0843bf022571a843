"""GPU parity of the baselines (FastKV, APB, ring attention) against the
reference's own baseline functions (golden vectors) and the oracle.

* float64 inputs: the golden outputs within 1e-4 relative;
* float32 inputs: the oracle on the float32-rounded inputs within 1e-4;
* bfloat16 inputs: the oracle on the bf16-rounded inputs within 2e-2.
Causal (the reference's prefix rule on compact entries) and non-causal.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from dcc_kv_b200 import baselines as bl
from oracle import dcc_kv_oracle as orc

from gpu_util import assert_no_device_timeouts, baseline_inputs, dev, golden, np64, rel_err

pytestmark = pytest.mark.gpu


def _cfgs(f):
    fk = bl.FastKVConfig(budget=int(f["fk_budget"]), num_repr_queries=int(f["fk_M"]), projection_dim=int(f["fk_dp"]))
    ap = bl.APBConfig(anchor_budget=int(f["apb_budget"]))
    return fk, ap


@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("dtype", [torch.float64, torch.float32, torch.bfloat16])
def test_fast_kv_and_apb(dtype, causal):
    f = golden("baselines_small.npz")
    Q, K, V = baseline_inputs(f)
    chunk, world = int(f["chunk"]), int(f["world"])
    fk_cfg, ap_cfg = _cfgs(f)
    tag = "causal" if causal else "full"
    q, k, v = (x.to(dtype).to(dev()) for x in (Q, K, V))
    got_fk = bl.fast_kv(q, k, v, chunk, world, fk_cfg, causal=causal)
    got_ap = bl.apb(q, k, v, chunk, world, ap_cfg, causal=causal)
    torch.cuda.synchronize()
    assert_no_device_timeouts()
    if dtype == torch.float64:
        want_fk, want_ap, tol = f[f"fastkv_{tag}"], f[f"apb_{tag}"], 1e-4
    else:
        Qr, Kr, Vr = (x.to(dtype).double().numpy() for x in (Q, K, V))
        want_fk = orc.fast_kv(Qr, Kr, Vr, chunk, world, fk_cfg.budget, fk_cfg.num_repr_queries,
                              fk_cfg.projection_dim, causal=causal)
        want_ap = orc.apb(Qr, Kr, Vr, chunk, world, ap_cfg.anchor_budget, causal=causal)
        tol = 1e-4 if dtype == torch.float32 else 2e-2
    assert rel_err(np64(got_fk), want_fk) < tol
    assert rel_err(np64(got_ap), want_ap) < tol


def test_anchor_selection_matches_oracle():
    """APB anchors (indices of the top attention mass) for one chunk, float64."""
    f = golden("baselines_small.npz")
    Q, K, V = baseline_inputs(f)
    budget = int(f["apb_budget"])
    ak, _ = bl.select_anchor_blocks(K[:96].to(dev()), V[:96].to(dev()), Q.to(dev()), budget)
    _, _, idx = orc.select_anchor_blocks(K[:96].numpy(), V[:96].numpy(), Q.numpy(), budget)
    np.testing.assert_array_equal(np64(ak), K[:96].numpy()[idx])


@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("dtype", [torch.float64, torch.bfloat16])
def test_ring_attention(dtype, causal):
    f = golden("baselines_small.npz")
    Q, K, V = baseline_inputs(f)
    chunk, world, T = int(f["chunk"]), int(f["world"]), int(f["T"])
    bounds = [(s * chunk, (s + 1) * chunk if s < world - 1 else T) for s in range(world)]
    q, k, v = (x.to(dtype).to(dev()) for x in (Q, K, V))
    got = bl.ring_attention(q, [k[a:b] for a, b in bounds], [v[a:b] for a, b in bounds], causal=causal)
    torch.cuda.synchronize()
    if dtype == torch.float64:
        want, tol = f["ring_causal" if causal else "ring_full"], 1e-4
    else:
        Qr, Kr, Vr = (x.to(dtype).double().numpy() for x in (Q, K, V))
        want = orc.attention_partial(Qr, Kr, Vr, positions=np.arange(T) if causal else None)[0]
        tol = 2e-2
    assert rel_err(np64(got), want) < tol
