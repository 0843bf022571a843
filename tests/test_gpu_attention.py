"""GPU parity of the destination side: segmented biased attention, the
online-softmax kernels and the P-way LSE merge, against the oracle and the
reference's golden vectors.

Bars: float32 / float64 paths within 1e-4 relative (FP64 accumulation lands
near 1e-7); bf16 inputs within 2e-2 relative on attention outputs.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import dcc_kv_b200 as dk
from dcc_kv_b200 import _lib as L
from oracle import dcc_kv_oracle as orc

from gpu_util import dev, golden, np64, rel_err, to_gpu

pytestmark = pytest.mark.gpu


def test_online_softmax_golden():
    f = golden("online_softmax.npz")
    d64 = torch.float64
    s1 = dk.online_softmax_from_attention(to_gpu(f["logits1"], d64), to_gpu(f["values1"], d64))
    s2 = dk.online_softmax_from_attention(to_gpu(f["logits2"], d64), to_gpu(f["values2"], d64),
                                          logit_bias=to_gpu(f["bias"], d64))
    for st, keys in ((s1, ("m1", "l1", "o1")), (s2, ("m2", "l2", "o2"))):
        for got, k in zip((st.m, st.l, st.o), keys):
            assert rel_err(np64(got), f[k]) < 1e-13
    m = dk.merge_softmax_states(s1, s2)
    for got, k in zip((m.m, m.l, m.o), ("m", "l", "o")):
        assert rel_err(np64(got), f[k]) < 1e-13
    # single-row form, as the reference calls it
    one = dk.online_softmax_from_attention(to_gpu(f["logits1"][0], d64), to_gpu(f["values1"], d64))
    assert one.o.shape == (f["values1"].shape[1],)
    assert abs(float(one.m) - f["m1"][0]) < 1e-13


def test_reference_kats():
    """The reference's own online-softmax KATs (tests/test_dist_equivalence.py:45-119)."""
    d = dev()
    logits = torch.tensor([1.0, 2.0, 3.0], device=d)
    values = torch.tensor([[1.0, 1.0], [2.0, 2.0], [3.0, 3.0]], device=d)
    st = dk.online_softmax_from_attention(logits, values)
    assert torch.allclose(st.o / st.l, torch.softmax(logits, -1) @ values, atol=1e-6)
    s1 = dk.online_softmax_from_attention(torch.tensor([1.0, 2.0], device=d), torch.tensor([[1.0], [2.0]], device=d))
    s2 = dk.online_softmax_from_attention(torch.tensor([3.0, 4.0], device=d), torch.tensor([[3.0], [4.0]], device=d))
    full = dk.online_softmax_from_attention(torch.tensor([1.0, 2.0, 3.0, 4.0], device=d),
                                            torch.tensor([[1.0], [2.0], [3.0], [4.0]], device=d))
    mg = dk.merge_softmax_states(s1, s2)
    assert torch.allclose(mg.o / mg.l, full.o / full.l, atol=1e-6)
    bias = torch.tensor([0.0, 1.0, -1.0], device=d)
    a = dk.online_softmax_from_attention(logits, values[:, :1], logit_bias=bias)
    b = dk.online_softmax_from_attention(logits + bias, values[:, :1])
    assert torch.allclose(a.m, b.m) and torch.allclose(a.l, b.l) and torch.allclose(a.o, b.o)
    g = torch.Generator().manual_seed(0)
    assert dk.verify_order_invariance([])
    same_d = []
    for _ in range(8):
        n = int(torch.randint(4, 32, (1,), generator=g))
        same_d.append(dk.online_softmax_from_attention(torch.randn(n, generator=g).to(d), torch.randn(n, 8, generator=g).to(d)))
    assert dk.verify_order_invariance(same_d, n_trials=20, seed=42)


@pytest.mark.parametrize("dtype,n_parts,dim", [(torch.bfloat16, 8, 128), (torch.bfloat16, 2, 128),
                                               (torch.float32, 3, 64), (torch.float32, 5, 33),
                                               (torch.float64, 4, 16)])
def test_merge_lse(dtype, n_parts, dim):
    g = torch.Generator().manual_seed(n_parts * 100 + dim)
    outs = [torch.randn(4, 257, dim, generator=g, dtype=torch.float64) for _ in range(n_parts)]
    lses = [torch.randn(4, 257, generator=g, dtype=torch.float64) * 4 for _ in range(n_parts)]
    lses[0][0, :5] = -float("inf")  # an empty partial contributes nothing
    o, lse = dk.merge_lse([x.to(dtype).to(dev()) for x in outs], [x.float().to(dev()) for x in lses])
    ro = [x.to(dtype).double().numpy() for x in outs]
    rl = [x.float().double().numpy() for x in lses]
    want_o, want_l = orc.merge_lse(ro, rl)
    tol = 2e-2 if dtype == torch.bfloat16 else 1e-4
    assert rel_err(np64(o), want_o) < tol
    assert rel_err(np64(lse), want_l) < 1e-5


def _attn_case(dtype, hq, hkv, lq, d, segs, causal, seed):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(hq, lq, d, generator=g, dtype=torch.float64)
    segments = []
    for n, with_bias in segs:
        k = torch.randn(hkv, n, d, generator=g, dtype=torch.float64)
        v = torch.randn(hkv, n, d, generator=g, dtype=torch.float64)
        b = torch.randn(hkv, n, generator=g, dtype=torch.float64) * 3 if with_bias else None
        segments.append((k, v, b))
    qd = q.to(dtype)
    o, lse = dk.attention(qd.to(dev()), [(k.to(dtype).to(dev()), v.to(dtype).to(dev()),
                                          None if b is None else b.float().to(dev())) for k, v, b in segments],
                          causal=causal)
    torch.cuda.synchronize()
    assert L.lib().dcc_device_error_status(1) == 0, "a bounded device wait expired"
    grp = hq // hkv
    for h in range(hq):
        qh = qd[h].double().numpy()
        parts = []
        for i, (k, v, b) in enumerate(segments):
            kk = k[h // grp].to(dtype).double().numpy()
            vv = v[h // grp].to(dtype).double().numpy()
            bb = None if b is None else b[h // grp].float().double().numpy()
            pos = np.arange(lq) if (causal and i == 0) else None
            parts.append(orc.attention_partial(qh, kk, vv, bias=bb, positions=pos))
        want_o, want_l = orc.merge_lse([p[0] for p in parts], [p[1] for p in parts])
        tol = 2e-2 if dtype == torch.bfloat16 else 1e-4
        assert np.isfinite(np64(o[h])).all()
        assert rel_err(np64(o[h]), want_o) < tol, h
        assert rel_err(np64(lse[h]), want_l) < (1e-2 if dtype == torch.bfloat16 else 1e-5)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_attention_local_causal(dtype):
    _attn_case(dtype, 8, 2, 300, 128, [(300, False)], True, 1)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_attention_biased_segments(dtype):
    _attn_case(dtype, 4, 4, 129, 128, [(77, True), (64, True), (200, True)], False, 2)


def test_attention_small_head_dim_f32():
    _attn_case(torch.float32, 4, 2, 50, 32, [(50, False), (17, True)], True, 3)


@pytest.mark.parametrize("hq,hkv,lq,segs,causal", [
    (8, 2, 1000, [(1000, False)], True),                       # ragged causal, 8 tiles
    (8, 2, 256, [(300, True), (128, True), (5, True)], False),  # three biased segments, ragged
    (4, 1, 130, [(130, False), (64, True)], True),              # causal + compact in one launch
    (2, 1, 64, [(1, True), (40, True)], False),                 # a one-key segment
])
def test_attention_tc05_shapes_bf16(hq, hkv, lq, segs, causal):
    _attn_case(torch.bfloat16, hq, hkv, lq, 128, segs, causal, hq * 7 + lq)


@pytest.mark.parametrize("dtype,hq,hkv,d", [
    (torch.bfloat16, 8, 2, 128),   # tcgen05 kernel
    (torch.bfloat16, 3, 3, 128),   # odd GQA group: the mma.sync kernel
    (torch.float32, 4, 2, 64),     # FP64-accumulating CUDA-core kernel
])
def test_attention_continues_from_initial_state(dtype, hq, hkv, d):
    """Two launches -- causal local keys, then biased compact keys starting
    from the first launch's (O, LSE), in place -- equal the one-pass merge;
    an empty second segment passes the state through."""
    g = torch.Generator().manual_seed(hq * 31 + d)
    lq = 300
    q = torch.randn(hq, lq, d, generator=g, dtype=torch.float64)
    k1, v1 = (torch.randn(hkv, lq, d, generator=g, dtype=torch.float64) for _ in range(2))
    k2, v2 = (torch.randn(hkv, 200, d, generator=g, dtype=torch.float64) for _ in range(2))
    b2 = torch.randn(hkv, 200, generator=g, dtype=torch.float64) * 3 + 4  # compact logits above the local ones
    cast = lambda t: t.to(dtype).to(dev())
    o1, l1 = dk.attention(cast(q), [(cast(k1), cast(v1), None)], causal=True)
    o2, l2 = dk.attention(cast(q), [(cast(k2), cast(v2), b2.float().to(dev()))], init=(o1, l1))
    o3, l3 = dk.attention(cast(q), [(cast(k2[:, :0]), cast(v2[:, :0]), None)], init=(o1, l1))
    torch.cuda.synchronize()
    assert L.lib().dcc_device_error_status(1) == 0, "a bounded device wait expired"
    tol = 2e-2 if dtype == torch.bfloat16 else 1e-4
    grp = hq // hkv
    qd = q.to(dtype).double().numpy()
    for h in range(hq):
        kk1, vv1 = (x[h // grp].to(dtype).double().numpy() for x in (k1, v1))
        kk2, vv2 = (x[h // grp].to(dtype).double().numpy() for x in (k2, v2))
        p1 = orc.attention_partial(qd[h], kk1, vv1, positions=np.arange(lq))
        p2 = orc.attention_partial(qd[h], kk2, vv2, bias=b2[h // grp].float().double().numpy())
        want_o, want_l = orc.merge_lse([p1[0], p2[0]], [p1[1], p2[1]])
        assert rel_err(np64(o2[h]), want_o) < tol, h
        assert rel_err(np64(l2[h]), want_l) < (1e-2 if dtype == torch.bfloat16 else 1e-5), h
        assert rel_err(np64(o3[h]), p1[0]) < tol, h
        assert rel_err(np64(l3[h]), p1[1]) < (1e-2 if dtype == torch.bfloat16 else 1e-5), h
    # in place: the initial state aliasing the outputs
    from dcc_kv_b200.attention import attn_problem, kv_segment, run_attention
    o_in, l_in = o1.clone(), l1.clone()
    qc, kc, vc, bc = cast(q), cast(k2), cast(v2), b2.float().to(dev())
    prob = attn_problem(qc, o_in, l_in, [kv_segment(kc, vc, bc)], o_init=o_in, lse_init=l_in)
    run_attention([prob], hq, hkv, d, 1.0 / d ** 0.5, L.dtype_code(qc), dev())
    torch.cuda.synchronize()
    assert torch.equal(o_in, o2) and torch.equal(l_in, l2)


def test_merge_lse_cfg2_full_size():
    """The merge microbenchmark at full size: 8 partial outputs
    [32, 4096, 128] bf16 with fp32 LSE ~ N(0,1)*4.  The whole output against
    the LSE-weighted sum in fp32 (torch, on the device) and 64 sampled
    (head, query) rows against the FP64 oracle fold of
    online_softmax.py:92-111; bf16 output within 2e-2 relative (it lands
    at bf16 rounding), LSE within 1e-5."""
    from dcc_kv_b200.workloads import merge_inputs
    outs, lses = merge_inputs(8, 32, 4096, 128, seed=0, device="cuda")
    o, lse = dk.merge_lse(outs, lses)
    torch.cuda.synchronize()
    ls = torch.stack(lses)                       # [8, 32, 4096]
    m = ls.max(dim=0).values
    w = torch.exp(ls - m)
    want = (w[..., None] * torch.stack([x.float() for x in outs])).sum(0) / w.sum(0)[..., None]
    want_lse = m + torch.log(w.sum(0))
    err = ((o.float() - want).abs().max() / want.abs().max()).item()
    assert err < 2e-2, err
    assert ((lse - want_lse).abs().max() / want_lse.abs().max()).item() < 1e-5
    g = torch.Generator().manual_seed(9)
    hs = torch.randint(0, 32, (64,), generator=g)
    qs = torch.randint(0, 4096, (64,), generator=g)
    ro = [x[hs, qs].double().cpu().numpy() for x in outs]
    rl = [x[hs, qs].double().cpu().numpy() for x in lses]
    want_o, want_l = orc.merge_lse(ro, rl)
    assert rel_err(np64(o[hs, qs]), want_o) < 2e-2
    assert rel_err(np64(lse[hs, qs]), want_l) < 1e-5
