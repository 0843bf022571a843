"""GPU parity of the whole DCC-KV sync layer (build + local attention +
compact attention with logit bias + online-softmax merge).

* small layer (4 blocks x 64 tokens, 4/2 heads, d 32, ragged budgets): the
  reference's own composition (golden vectors), float32 within 1e-4;
* config 1 (K,V [4096,128], Q [512,128], budget 64, local block 512): golden
  merged output, float32 within 1e-4;
* bf16 layer at reduced size against the FP64 oracle within 2e-2;
* full 128K layer (8 x 16384, 32/8 heads, budget 1024, bf16) and the 1M
  layer with variable budgets: sampled query rows of every block against
  the oracle within 2e-2.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import dcc_kv_b200 as dk
from oracle import dcc_kv_oracle as orc

from gpu_util import assert_no_device_timeouts, dev, golden, np64, rel_err, to_gpu

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("schedule", ["batched", "pipelined"])
def test_small_layer_golden_f32(schedule):
    f = golden("layer_small.npz")
    nb, hq, L, d = f["Q"].shape
    hkv = f["K"].shape[1]
    budgets = {(int(s), int(r)): int(b) for s, r, b in f["budgets"]}
    layer = dk.DccKvSyncLayer(nb, L, hq, hkv, d, budgets, int(f["window"]), int(f["M"]), int(f["dp"]),
                              dtype=torch.float32)
    layer.schedule = schedule
    out = layer(to_gpu(f["Q"], torch.float32), to_gpu(f["K"], torch.float32), to_gpu(f["V"], torch.float32))
    torch.cuda.synchronize()
    assert rel_err(np64(out), f["out"]) < 1e-4
    k = 0
    for r in range(1, nb):
        for s in range(r):
            for g in range(hkv):
                np.testing.assert_array_equal(layer.compact(s, r, g).selected_indices[:16].cpu().numpy(),
                                              f["sel"][k][g])
            k += 1


def test_cfg1_two_block_merge_golden_f32():
    f = golden("layer_cfg1.npz")
    g = torch.Generator().manual_seed(0)
    K = torch.randn(4096, 128, generator=g, dtype=torch.float64)
    V = torch.randn(4096, 128, generator=g, dtype=torch.float64)
    Q = torch.randn(512, 128, generator=g, dtype=torch.float64)
    Kl = torch.randn(512, 128, generator=g, dtype=torch.float64)
    Vl = torch.randn(512, 128, generator=g, dtype=torch.float64)
    f32 = torch.float32
    c = dk.build_compact_kv(K.to(f32).to(dev()), V.to(f32).to(dev()), Q.to(f32).to(dev()), 64)
    q = Q.to(f32).to(dev())[None]
    o_l, lse_l = dk.attention(q, [(Kl.to(f32).to(dev())[None], Vl.to(f32).to(dev())[None], None)], causal=True)
    o_c, lse_c = dk.attention(q, [(c.keys[None], c.values[None], c.logit_bias[None])])
    out, _ = dk.merge_lse([o_l, o_c], [lse_l, lse_c])
    torch.cuda.synchronize()
    assert rel_err(np64(out[0]), f["merged"]) < 1e-4


def _oracle_layer(q, k, v, budgets, window, M, dp, rows=None):
    # float32 holds bf16 / float32 inputs exactly; the oracle widens each
    # head to FP64 as it reads it (a 1M-token block in FP64 would be GBs)
    qb = [x.float().numpy() for x in q]
    kb = [x.float().numpy() for x in k]
    vb = [x.float().numpy() for x in v]
    return orc.layer_forward(qb, kb, vb, budgets, window, M, dp, rows=rows)


@pytest.mark.parametrize("schedule", ["batched", "pipelined"])
def test_layer_bf16_small(schedule):
    from dcc_kv_b200.workloads import layer_inputs
    nb, L, hq, hkv, d = 4, 512, 8, 2, 128
    q, k, v = layer_inputs(nb, L, hq, hkv, d, device="cpu", first_seed=7)
    budgets = {(s, r): [64, 96, 128][(s + 2 * r) % 3] for r in range(nb) for s in range(r)}
    layer = dk.DccKvSyncLayer(nb, L, hq, hkv, d, budgets, window=128)
    layer.schedule = schedule
    out = layer(q.to(dev()), k.to(dev()), v.to(dev()))
    torch.cuda.synchronize()
    assert_no_device_timeouts()
    ref, _ = _oracle_layer(q, k, v, budgets, 128, 64, 32)
    for r in range(nb):
        assert rel_err(np64(out[r]), ref[r]) < 2e-2, r


def _kv_head_slice(q, k, v, g, group):
    """The layer is independent across KV heads: KV head g with its query
    heads g*group .. (g+1)*group-1, every block."""
    return q[:, g * group:(g + 1) * group].cpu(), k[:, g:g + 1].cpu(), v[:, g:g + 1].cpu()


@pytest.mark.slow
def test_layer_full_128k_bf16_all_blocks_sampled():
    """The benchmarked layer (8 x 16384, 32/8 heads, budget 1024, window
    2048): sampled query rows of every block -- block 7 with its seven
    compact sources included -- for KV heads 0 and 5 (their query heads
    0-3 and 20-23) against the FP64 oracle, which builds every edge into
    each block for that head (dcc_kv_sync_cpu.py:52-84)."""
    from dcc_kv_b200.workloads import layer_inputs
    nb, L, hq, hkv, d = 8, 16384, 32, 8, 128
    q, k, v = layer_inputs(nb, L, hq, hkv, d, device="cpu")
    layer = dk.DccKvSyncLayer(nb, L, hq, hkv, d, 1024, window=2048)
    out = layer(q.to(dev()), k.to(dev()), v.to(dev()))
    torch.cuda.synchronize()
    assert_no_device_timeouts()
    assert torch.isfinite(out).all()
    rows = {b: np.array([0, 1, 777, 2047, 2048, 8191, 12345, L - 1]) for b in range(nb)}
    budgets = {(s, r): 1024 for r in range(nb) for s in range(r)}
    group = hq // hkv
    for g in (0, 5):
        qh, kh, vh = _kv_head_slice(q, k, v, g, group)
        ref, _ = _oracle_layer(qh, kh, vh, budgets, 2048, 64, 32, rows=rows)
        for r in range(nb):
            got = np64(out[r, g * group:(g + 1) * group][:, rows[r]])
            assert rel_err(got, ref[r]) < 2e-2, (g, r)


def test_layer_host_buffers_match_device_path():
    """Host inputs stream through the per-block pipeline (copy-in, pooling and
    builds on a side stream, attention, copy-out); two calls in a row with
    different inputs must each equal the device-resident forward bit for bit."""
    from dcc_kv_b200.workloads import layer_inputs
    nb, L, hq, hkv, d = 4, 1024, 8, 2, 128
    budgets = {(s, r): [64, 96, 128][(s + 2 * r) % 3] for r in range(nb) for s in range(r)}
    layer = dk.DccKvSyncLayer(nb, L, hq, hkv, d, budgets, window=256)
    inputs = [layer_inputs(nb, L, hq, hkv, d, device="cpu", first_seed=s) for s in (11, 23)]
    want = []
    for q, k, v in inputs:
        dq, dk_, dv = q.to(dev()), k.to(dev()), v.to(dev())
        layer.schedule = "batched"
        want.append(layer(dq, dk_, dv).cpu())
        # the overlapped per-block schedule runs the same kernels per block
        layer.schedule = "pipelined"
        assert torch.equal(layer(dq, dk_, dv).cpu(), want[-1])
    outs = [torch.empty(q.shape, dtype=q.dtype).pin_memory() for q, _, _ in inputs]
    pinned = [tuple(t.pin_memory() for t in x) for x in inputs]
    for (q, k, v), o in zip(pinned, outs):
        layer(q, k, v, out=o)
    torch.cuda.synchronize()
    assert_no_device_timeouts()
    for o, w in zip(outs, want):
        assert torch.equal(o, w)
    with pytest.raises(ValueError):
        layer(pinned[0][0][:, :4], pinned[0][1], pinned[0][2])


@pytest.mark.slow
def test_layer_1m_variable_budgets_all_blocks_sampled():
    """1M-token layer (8 x 131072, 32/8 heads, window 2048, budgets drawn from
    {256, 512, 1024, 2048} with seed 1): the whole layer runs on the GPU;
    sampled rows of every block for KV head 3 (query heads 12-15) are
    recomputed by the oracle, which builds all 28 edges of that head."""
    from dcc_kv_b200.workloads import layer_inputs, variable_budgets
    nb, L, hq, hkv, d = 8, 131072, 32, 8, 128
    budgets = variable_budgets(nb)
    q, k, v = layer_inputs(nb, L, hq, hkv, d, device="cuda")
    layer = dk.DccKvSyncLayer(nb, L, hq, hkv, d, budgets, window=2048)
    out = layer(q, k, v)
    torch.cuda.synchronize()
    assert_no_device_timeouts()
    assert torch.isfinite(out).all()
    group, g = hq // hkv, 3
    rows = {b: np.array([0, 1, 2047, 2048, 77777, L - 1]) for b in range(nb)}
    qh, kh, vh = _kv_head_slice(q, k, v, g, group)
    ref, _ = _oracle_layer(qh, kh, vh, budgets, 2048, 64, 32, rows=rows)
    for r in range(nb):
        got = np64(out[r, g * group:(g + 1) * group][:, rows[r]])
        assert rel_err(got, ref[r]) < 2e-2, r


def test_device_timeout_reaches_the_caller():
    """A bounded device wait that runs out -- an mbarrier nothing arrives at,
    10 ms limit, no fault -- surfaces as DccError(DCC_ERR_TIMEOUT): from the
    layer's next call (each forward reports the error flags to pinned host
    memory without synchronising) and from check().  The context stays
    usable and the next forward is right again."""
    from dcc_kv_b200 import _lib as L
    from dcc_kv_b200.workloads import layer_inputs
    nb, Lb, hq, hkv, d = 3, 256, 4, 2, 128
    q, k, v = (t.to(dev()) for t in layer_inputs(nb, Lb, hq, hkv, d, device="cpu", first_seed=5))
    layer = dk.DccKvSyncLayer(nb, Lb, hq, hkv, d, 64, window=64)
    want = layer(q, k, v).clone()
    layer.check()
    stream = L.stream_ptr(dev())
    L.check(L.lib().dcc_debug_expire_wait(10_000_000, stream), "debug_expire_wait")
    layer(q, k, v)  # its flag report runs after the expired wait
    torch.cuda.synchronize()
    with pytest.raises(L.DccError) as err:
        layer(q, k, v)
    assert err.value.status == L.DCC_ERR_TIMEOUT
    assert torch.equal(layer(q, k, v), want)
    layer.check()
    L.check(L.lib().dcc_debug_expire_wait(10_000_000, stream), "debug_expire_wait")
    with pytest.raises(L.DccError) as err:
        layer.check()
    assert err.value.status == L.DCC_ERR_TIMEOUT
    assert torch.equal(layer(q, k, v), want)
    layer.check()
