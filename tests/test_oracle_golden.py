"""The oracle against the golden vectors produced by the reference itself.

These pin the CPU restatement (oracle/dcc_kv_oracle.py) before it is trusted
as the checker for the CUDA path.
"""
from __future__ import annotations

import glob
import os

import numpy as np
import pytest
import torch

from oracle import dcc_kv_oracle as orc

from conftest import GOLDEN


def _load(name):
    return np.load(os.path.join(GOLDEN, name))


def test_rng_matches_torch_generator():
    rng = _load("rng.npz")
    for key in rng.files:
        parts = key.split("_")
        if parts[0] == "proj":
            seed, dp, d = map(int, parts[1:])
            got = orc.rademacher_projection(d, dp, seed)
            np.testing.assert_array_equal(got, rng[key].astype(np.float64))
        else:
            seed, n = map(int, parts[1:])
            assert orc.fps_start_index(n, seed) == int(rng[key])


def test_rng_matches_live_torch():
    # torch is present on every machine this runs on; compare live as well
    for seed in (3, 99):
        g = torch.Generator().manual_seed(seed)
        t = torch.randint(0, 2, (16, 48), generator=g)
        p = orc.rademacher_projection(48, 16, seed)
        np.testing.assert_array_equal(np.sign(p), (t * 2 - 1).numpy())


BUILD_CASES = sorted(os.path.basename(p) for p in glob.glob(os.path.join(GOLDEN, "build_*.npz")))


def _inputs(f, name):
    if name == "build_cfg1.npz":
        g = torch.Generator().manual_seed(0)
        K = torch.randn(4096, 128, generator=g, dtype=torch.float64).numpy()
        V = torch.randn(4096, 128, generator=g, dtype=torch.float64).numpy()
        Q = torch.randn(512, 128, generator=g, dtype=torch.float64).numpy()
        return K, V, Q
    return f["K"].astype(np.float64), f["V"].astype(np.float64), f["Q"].astype(np.float64)


@pytest.mark.parametrize("name", BUILD_CASES)
def test_build_compact_kv_matches_reference(name):
    f = _load(name)
    K, V, Q = _inputs(f, name)
    c = orc.build_compact_kv(K, V, Q, int(f["budget"]), int(f["M"]), int(f["dp"]),
                             float(f["lambda_beta"]), float(f["lambda_value"]), int(f["seed"]))
    np.testing.assert_array_equal(c.repr_indices, f["repr_indices"])
    np.testing.assert_array_equal(c.selected_indices, f["selected_indices"])
    np.testing.assert_array_equal(c.keys, f["keys"])
    # The closed-form ridge systems are ill-conditioned (cond(G^T G + lam I)
    # reaches 1e7-1e8), so two LAPACK builds of the same LU solve (numpy's vs
    # torch's) differ by about cond * eps: bound the error relative to the
    # largest entry at 1e-7 (measured worst case 2.3e-8).
    for got, want in ((c.logit_bias, f["logit_bias"]), (c.values, f["values"])):
        np.testing.assert_allclose(got, want, rtol=0, atol=1e-7 * np.abs(want).max())


def test_online_softmax_matches_reference():
    f = _load("online_softmax.npz")
    s1 = orc.online_softmax_state(f["logits1"], np.broadcast_to(f["values1"], (16,) + f["values1"].shape))
    s2 = orc.online_softmax_state(f["logits2"], np.broadcast_to(f["values2"], (16,) + f["values2"].shape),
                                  logit_bias=f["bias"])
    for got, key in zip(s1, ("m1", "l1", "o1")):
        np.testing.assert_allclose(got, f[key], rtol=1e-13, atol=1e-13)
    for got, key in zip(s2, ("m2", "l2", "o2")):
        np.testing.assert_allclose(got, f[key], rtol=1e-13, atol=1e-13)
    m = orc.merge_states(s1, s2)
    for got, key in zip(m, ("m", "l", "o")):
        np.testing.assert_allclose(got, f[key], rtol=1e-13, atol=1e-13)


def test_cfg1_merged_output_matches_reference():
    f = _load("layer_cfg1.npz")
    g = torch.Generator().manual_seed(0)
    K = torch.randn(4096, 128, generator=g, dtype=torch.float64).numpy()
    V = torch.randn(4096, 128, generator=g, dtype=torch.float64).numpy()
    Q = torch.randn(512, 128, generator=g, dtype=torch.float64).numpy()
    Kl = torch.randn(512, 128, generator=g, dtype=torch.float64).numpy()
    Vl = torch.randn(512, 128, generator=g, dtype=torch.float64).numpy()
    c = orc.build_compact_kv(K, V, Q, 64)
    o_l, lse_l = orc.attention_partial(Q, Kl, Vl, positions=np.arange(512))
    o_c, lse_c = orc.attention_partial(Q, c.keys, c.values, bias=c.logit_bias)
    out, _ = orc.merge_lse([o_l, o_c], [lse_l, lse_c])
    np.testing.assert_allclose(out, f["merged"], rtol=0, atol=1e-9)
    # the full-attention check is informational: compression error is large
    full = orc.full_causal_attention(np.concatenate([np.zeros((4096, 128)), Q]), np.concatenate([K, Kl]),
                                     np.concatenate([V, Vl]), np.arange(4096, 4608))
    np.testing.assert_allclose(full, f["full"], rtol=0, atol=1e-9)


def test_small_layer_matches_reference():
    f = _load("layer_small.npz")
    nb = f["Q"].shape[0]
    budgets = {(int(s), int(r)): int(b) for s, r, b in f["budgets"]}
    out, comp = orc.layer_forward(list(f["Q"]), list(f["K"]), list(f["V"]), budgets, int(f["window"]),
                                  int(f["M"]), int(f["dp"]))
    for r in range(nb):
        np.testing.assert_allclose(out[r], f["out"][r], rtol=0, atol=1e-9)
    k = 0
    for r in range(1, nb):
        for s in range(r):
            for g in range(f["K"].shape[1]):
                np.testing.assert_array_equal(comp[(s, r, g)].selected_indices[:16], f["sel"][k][g])
            k += 1


@pytest.mark.parametrize("causal", [True, False])
def test_shared_compaction_baselines_match_reference(causal):
    """FastKV (one compact per chunk from all queries) and APB (anchors by
    attention mass) against the reference's own baseline functions."""
    from gpu_util import baseline_inputs
    f = _load("baselines_small.npz")
    Q, K, V = (x.numpy() for x in baseline_inputs(f))
    tag = "causal" if causal else "full"
    fk = orc.fast_kv(Q, K, V, int(f["chunk"]), int(f["world"]), int(f["fk_budget"]), int(f["fk_M"]),
                     int(f["fk_dp"]), causal=causal)
    ap = orc.apb(Q, K, V, int(f["chunk"]), int(f["world"]), int(f["apb_budget"]), causal=causal)
    # ring attention is exact attention over the concatenated chunks
    T = Q.shape[0]
    ring = orc.attention_partial(Q, K, V, positions=np.arange(T) if causal else None)[0]
    for got, want in ((fk, f[f"fastkv_{tag}"]), (ap, f[f"apb_{tag}"]), (ring, f[f"ring_{tag}"])):
        assert np.abs(got - want).max() / np.abs(want).max() < 1e-6
