"""GPU parity of the compact-KV build against the oracle and the golden
vectors of the reference (FP64 CPU).

Bars (from the north-star statement):
  * float32 / float64 inputs: selected_indices and representative indices
    bit-exact; logit_bias and compact values within 1e-4 relative
    (max |err| / max |ref|) -- the FP64 kernels land near 1e-9;
  * bfloat16 inputs: checked end to end on the layer output (2e-2).
"""
from __future__ import annotations

import glob
import os

import numpy as np
import pytest
import torch

import dcc_kv_b200 as dk
from oracle import dcc_kv_oracle as orc

from conftest import GOLDEN
from gpu_util import assert_no_device_timeouts, build_inputs, dev, golden, np64, rel_err, to_gpu

pytestmark = pytest.mark.gpu

CASES = sorted(os.path.basename(p) for p in glob.glob(os.path.join(GOLDEN, "build_*.npz")))


@pytest.mark.parametrize("dtype", [torch.float64, torch.float32])
@pytest.mark.parametrize("name", CASES)
def test_build_compact_kv_golden(name, dtype):
    f = golden(name)
    K, V, Q = build_inputs(f, name)
    if dtype == torch.float32 and not all(np.array_equal(x, x.astype(np.float32)) for x in (K, V, Q)):
        # float32 inputs are a different problem: compare with the oracle on them
        K, V, Q = (x.astype(np.float32).astype(np.float64) for x in (K, V, Q))
        ref = orc.build_compact_kv(K, V, Q, int(f["budget"]), int(f["M"]), int(f["dp"]))
        want = dict(selected_indices=ref.selected_indices, logit_bias=ref.logit_bias, values=ref.values,
                    keys=ref.keys)
    else:
        want = {k: f[k] for k in ("selected_indices", "logit_bias", "values", "keys")}
    c = dk.build_compact_kv(to_gpu(K, dtype), to_gpu(V, dtype), to_gpu(Q, dtype), int(f["budget"]),
                            num_representative_queries=int(f["M"]), projection_dim=int(f["dp"]))
    torch.cuda.synchronize()
    np.testing.assert_array_equal(c.selected_indices.cpu().numpy(), want["selected_indices"])
    np.testing.assert_array_equal(np64(c.keys), np.asarray(want["keys"], np.float64).astype(
        np.float32 if dtype == torch.float32 else np.float64))
    tol = 1e-4 if dtype == torch.float32 else 1e-7
    assert rel_err(np64(c.logit_bias), want["logit_bias"]) < tol
    assert rel_err(np64(c.values), want["values"]) < tol


@pytest.mark.parametrize("name", CASES)
def test_representative_queries_golden(name):
    f = golden(name)
    _, _, Q = build_inputs(f, name)
    rep, idx = dk.select_representative_queries(to_gpu(Q, torch.float64), int(f["M"]), int(f["dp"]))
    np.testing.assert_array_equal(idx.cpu().numpy(), f["repr_indices"])
    np.testing.assert_array_equal(np64(rep), Q[f["repr_indices"]])


def test_farthest_point_sampling_matches_oracle():
    g = torch.Generator().manual_seed(3)
    for n, dim, m in ((700, 16, 40), (9000, 32, 64), (20000, 8, 17), (5, 8, 9)):
        feat = torch.randn(n, dim, generator=g, dtype=torch.float64)
        got = dk.farthest_point_sampling(feat.to(dev()), m, seed=7).cpu().numpy()
        np.testing.assert_array_equal(got, orc.farthest_point_sampling(feat.numpy(), m, seed=7))


def test_stage_functions_match_oracle():
    f = golden("build_closed_form.npz")
    K, V, Q = build_inputs(f, "build_closed_form.npz")
    M = int(f["M"])
    qh, _ = orc.select_representative_queries(Q, M, int(f["dp"]))
    B = int(f["budget"])
    d64 = torch.float64
    # select_topk_keys
    ck, idx = dk.select_topk_keys(to_gpu(K, d64), to_gpu(qh, d64), B)
    ck_ref, idx_ref = orc.select_topk_keys(K, qh, B)
    np.testing.assert_array_equal(idx.cpu().numpy(), idx_ref)
    # rms_per_token_score
    A = orc.attention_scores(K, qh)
    u = dk.rms_per_token_score(to_gpu(A, d64))
    assert rel_err(np64(u), orc.rms_per_token_score(A)) < 1e-12
    # fit_logit_bias
    mass = A.sum(-1)
    beta = dk.fit_logit_bias(to_gpu(qh, d64), to_gpu(ck_ref, d64), to_gpu(mass, d64))
    beta_ref = orc.fit_logit_bias(qh, ck_ref, mass)
    assert rel_err(np64(beta), beta_ref) < 1e-7
    # fit_compact_value
    cv = dk.fit_compact_value(to_gpu(qh, d64), to_gpu(K, d64), to_gpu(V, d64), to_gpu(ck_ref, d64),
                              to_gpu(beta_ref, d64))
    assert rel_err(np64(cv), orc.fit_compact_value(qh, K, V, ck_ref, beta_ref)) < 1e-7
    # nonneg_least_squares, both branches
    G = np.exp(qh @ ck_ref.T / np.sqrt(K.shape[1]))
    for Gm in (G, G[:, :M]):
        w = dk.nonneg_least_squares(to_gpu(Gm, d64), to_gpu(mass, d64))
        assert rel_err(np64(w), orc.nonneg_least_squares(Gm, mass)) < 1e-7
    # ridge_regression_value, both branches
    X = orc.softmax(qh @ ck_ref.T / np.sqrt(K.shape[1]))
    Y = A @ V
    for Xm in (X, X[:, :M - 4]):
        out = dk.ridge_regression_value(to_gpu(Xm, d64), to_gpu(Y, d64))
        assert rel_err(np64(out), orc.ridge_regression_value(Xm, Y)) < 1e-7


def test_gqa_batched_build_full_size_bf16():
    """cfg3 geometry (one block pair): 8 KV heads, L_s = 16384, 4 x 2048
    destination queries per KV head, budget 512, bf16 inputs.  The FP64
    oracle runs on two KV heads; the scoring path accumulates in fp32, so
    index sets may differ only at near-ties and the compact attention output
    of the destination queries must agree within 2e-2."""
    from dcc_kv_b200.workloads import gqa_block
    q, k, v = gqa_block(32, 8, 16384, 128, seed=0, q_len=2048)
    repr_q = []
    for h in range(8):
        dq = torch.cat([q[4 * h + j] for j in range(4)]).to(dev())
        rep, _ = dk.select_representative_queries(dq, 64, 32)
        repr_q.append(rep)
    comps = dk.build_compact_kv_batched(k.to(dev()), v.to(dev()), torch.stack(repr_q), 512)
    torch.cuda.synchronize()
    assert_no_device_timeouts()
    for h in (0, 5):
        dq = np.concatenate([q[4 * h + j].double().numpy() for j in range(4)])
        ref = orc.build_compact_kv(k[h].double().numpy(), v[h].double().numpy(), dq, 512)
        got = comps[h]
        overlap = len(np.intersect1d(got.selected_indices.cpu().numpy(), ref.selected_indices)) / 512
        assert overlap > 0.98, overlap
        sample = dq[::97]
        o_ref, _ = orc.attention_partial(sample, ref.keys, ref.values, bias=ref.logit_bias)
        o_got, _ = orc.attention_partial(sample, np64(got.keys), np64(got.values), bias=np64(got.logit_bias))
        assert rel_err(o_got, o_ref) < 2e-2


def _assert_same_topk_up_to_ties(got, want, scores, budget, rel_gap=1e-6):
    """``got`` and ``want`` are top-``budget`` index lists sorted by score,
    descending.  They must be equal, except that keys whose FP64 RMS scores
    lie within ``rel_gap`` (relative) of each other may trade places -- the
    documented score-tie allowance.  Returns the positions that differ."""
    got, want = np.asarray(got), np.asarray(want)
    diff = np.nonzero(got != want)[0]
    if diff.size == 0:
        return diff
    boundary = scores[want[-1]]
    for i in diff:
        a, b = scores[got[i]], scores[want[i]]
        assert abs(a - b) <= rel_gap * abs(b), f"position {i}: {got[i]} vs {want[i]} ({a!r} vs {b!r})"
    # a key that left or entered the set must tie with the B-th score
    for j in np.setxor1d(got, want):
        assert abs(scores[j] - boundary) <= rel_gap * abs(boundary), f"key {j} is not a boundary tie"
    return diff


def test_gqa_batched_build_full_size_f32_indices_bit_exact():
    """cfg3 geometry in float32 mode: 8 KV heads, L_s = 16384, 4 x 2048
    destination queries per KV head, budget 512.  Every KV head against the
    FP64 oracle: representative indices and selected_indices bit-exact (the
    float32 path scores in FP64) except at documented score ties (relative
    gap below 1e-6, listed when they occur); logit_bias and compact values
    within 1e-4 relative."""
    from dcc_kv_b200.workloads import gqa_block
    q, k, v = gqa_block(32, 8, 16384, 128, seed=0, q_len=2048, dtype=torch.float32)
    repr_q, repr_idx = [], []
    for h in range(8):
        dq = torch.cat([q[4 * h + j] for j in range(4)]).to(dev())
        rep, idx = dk.select_representative_queries(dq, 64, 32)
        repr_q.append(rep)
        repr_idx.append(idx.cpu().numpy())
    comps = dk.build_compact_kv_batched(k.to(dev()), v.to(dev()), torch.stack(repr_q), 512)
    torch.cuda.synchronize()
    ties = {}
    for h in range(8):
        dq = np.concatenate([q[4 * h + j].double().numpy() for j in range(4)])
        K, V = k[h].double().numpy(), v[h].double().numpy()
        qh, ridx = orc.select_representative_queries(dq, 64, 32)
        np.testing.assert_array_equal(repr_idx[h], ridx)
        ref = orc.build_compact_kv_from_repr(K, V, qh, 512)
        scores = orc.rms_per_token_score(orc.attention_scores(K, qh))
        diff = _assert_same_topk_up_to_ties(comps[h].selected_indices.cpu().numpy(), ref.selected_indices,
                                            scores, 512)
        got = comps[h]
        if diff.size == 0:
            assert rel_err(np64(got.logit_bias), ref.logit_bias) < 1e-4, h
            assert rel_err(np64(got.values), ref.values) < 1e-4, h
        else:
            # a tie swapped keys: the compacts are then compared by what they compute
            ties[h] = diff.tolist()
            sample = dq[::97]
            o_ref, _ = orc.attention_partial(sample, ref.keys, ref.values, bias=ref.logit_bias)
            o_got, _ = orc.attention_partial(sample, np64(got.keys), np64(got.values), bias=np64(got.logit_bias))
            assert rel_err(o_got, o_ref) < 1e-4, h
    print(f"score ties (KV head: positions): {ties or 'none'}")
