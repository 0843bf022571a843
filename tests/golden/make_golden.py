"""Generate the golden vectors in this folder by running the reference itself.

Run once in a container that holds the reference checkout (read-only):

    python tests/golden/make_golden.py REFERENCE_CHECKOUT             # everything
    python tests/golden/make_golden.py REFERENCE_CHECKOUT baselines   # baselines_small.npz only

It imports ``src.dcc_kv_ref`` from that checkout, applies the FP64 dtype shim
to ``rademacher_projection`` (the reference casts the projection to float32,
representative_query.py:30, which makes a float64 matmul fail; the +-1/sqrt(d_p)
entries are the float32 values either way), runs each case in float64 and
writes compressed ``.npz`` fixtures.  Nothing at test time reads the reference.
"""
from __future__ import annotations

import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def load_reference(root: str):
    sys.path.insert(0, root)
    import src.dcc_kv_ref.representative_query as rq  # noqa: E402
    orig = rq.rademacher_projection

    def shim(queries, projection_dim=32, seed=42):
        return orig(queries, projection_dim, seed).to(queries.dtype)

    rq.rademacher_projection = shim
    import src.dcc_kv_ref as ref  # noqa: E402
    return ref, orig


def bf16_values(t: torch.Tensor) -> torch.Tensor:
    return t.to(torch.bfloat16).to(torch.float64)


def build_case(ref, name, K, V, Q, budget, M, dp, seed=42, lam_b=1e-3, lam_v=1e-3, store_inputs=True):
    c = ref.build_compact_kv(K, V, Q, budget, num_representative_queries=M, projection_dim=dp,
                             lambda_beta=lam_b, lambda_value=lam_v, seed=seed)
    qh, ridx = ref.select_representative_queries(Q, num_samples=M, projection_dim=dp, seed=seed)
    d = dict(budget=budget, M=M, dp=dp, seed=seed, lambda_beta=lam_b, lambda_value=lam_v,
             repr_indices=ridx.numpy(), selected_indices=c.selected_indices.numpy(),
             keys=c.keys.numpy(), logit_bias=c.logit_bias.numpy(), values=c.values.numpy())
    if store_inputs:
        # bf16-valued inputs are exact in float32; store them that way
        exact32 = all(torch.equal(x, x.float().double()) for x in (K, V, Q))
        cast = (lambda x: x.float().numpy()) if exact32 else (lambda x: x.numpy())
        d.update(K=cast(K), V=cast(V), Q=cast(Q))
    np.savez_compressed(os.path.join(HERE, f"build_{name}.npz"), **d)
    return c


def main(root: str) -> None:
    ref, orig_proj = load_reference(root)

    # -- random draws: projection matrices and FPS start indices ------------
    rng = {}
    for seed in (0, 1, 42, 12345):
        for dp, d in ((32, 128), (8, 32), (16, 64), (5, 7)):
            rng[f"proj_{seed}_{dp}_{d}"] = orig_proj(torch.zeros(1, d), dp, seed).numpy()
        for n in (7, 100, 512, 8192):
            g = torch.Generator().manual_seed(seed)
            rng[f"start_{seed}_{n}"] = np.array(int(torch.randint(0, n, (1,), generator=g).item()))
    np.savez_compressed(os.path.join(HERE, "rng.npz"), **rng)

    # -- config 1: K,V [4096,128], Q [512,128] N(0,1) seed 0, budget 64 ------
    # Inputs are regenerated at test time from the same torch CPU generator;
    # the local block K_loc, V_loc [512,128] is the next draw.
    g = torch.Generator().manual_seed(0)
    K = torch.randn(4096, 128, generator=g, dtype=torch.float64)
    V = torch.randn(4096, 128, generator=g, dtype=torch.float64)
    Q = torch.randn(512, 128, generator=g, dtype=torch.float64)
    Kl = torch.randn(512, 128, generator=g, dtype=torch.float64)
    Vl = torch.randn(512, 128, generator=g, dtype=torch.float64)
    c = build_case(ref, "cfg1", K, V, Q, 64, 64, 32, store_inputs=False)
    # destination side: local causal block + compact block (+beta), merged
    scale = 1.0 / 128 ** 0.5
    outs = []
    for i in range(512):
        st_l = ref.online_softmax_from_attention((Q[i] @ Kl[: i + 1].T) * scale, Vl[: i + 1])
        st_c = ref.online_softmax_from_attention((Q[i] @ c.keys.T) * scale, c.values,
                                                 logit_bias=c.logit_bias)
        st = ref.merge_softmax_states(st_l, st_c)
        outs.append((st.o / st.l).numpy())
    full = []
    Kf = torch.cat([K, Kl])
    Vf = torch.cat([V, Vl])
    for i in range(512):
        s = (Q[i] @ Kf[: 4096 + i + 1].T) * scale
        st = ref.online_softmax_from_attention(s, Vf[: 4096 + i + 1])
        full.append((st.o / st.l).numpy())
    np.savez_compressed(os.path.join(HERE, "layer_cfg1.npz"), merged=np.stack(outs), full=np.stack(full))

    # -- small build cases (inputs stored) ------------------------------------
    torch.manual_seed(42)
    cases = [
        # name, L_s, L_r, d, budget, M, d_p, bf16-valued
        ("reftest", 256, 100, 32, 64, 16, 8, False),   # tests/test_dist_equivalence.py:128-176 shapes
        ("closed_form", 512, 300, 64, 128, 32, 16, False),  # M < B: ridge start only
        ("pgd_eq", 300, 200, 32, 48, 48, 8, False),    # B == M: projected gradient
        ("pgd_lt", 200, 150, 32, 24, 40, 16, False),   # B < M: projected gradient
        ("b_ge_ls", 96, 80, 32, 96, 16, 8, False),     # budget >= L_s: early exit
        ("m_ge_n", 256, 12, 32, 40, 16, 8, False),     # M >= N: FPS returns arange
        ("odd", 333, 77, 48, 45, 20, 5, False),        # ragged sizes, odd d_p
        ("bf16_outlier", 2048, 1024, 128, 128, 64, 32, True),  # cfg3-like head, reduced
    ]
    for name, ls, lr, d, b, m, dp, bf in cases:
        gen = torch.Generator().manual_seed(len(name) * 7919 + ls)
        K = torch.randn(ls, d, generator=gen, dtype=torch.float64)
        V = torch.randn(ls, d, generator=gen, dtype=torch.float64)
        Q = torch.randn(lr, d, generator=gen, dtype=torch.float64)
        if bf:
            ch = torch.randperm(d, generator=gen)[:4]
            K[:, ch] *= 8
            V[:, ch] *= 8
            Q = Q / d ** 0.5
            K, V, Q = bf16_values(K), bf16_values(V), bf16_values(Q)
        build_case(ref, name, K, V, Q, b, m, dp)

    # -- online softmax KATs on a batch (reference functions, one row each) ---
    gen = torch.Generator().manual_seed(5)
    R, L1, L2, dv = 16, 24, 40, 8
    l1 = torch.randn(R, L1, generator=gen, dtype=torch.float64) * 3
    l2 = torch.randn(R, L2, generator=gen, dtype=torch.float64) * 3
    v1 = torch.randn(L1, dv, generator=gen, dtype=torch.float64)
    v2 = torch.randn(L2, dv, generator=gen, dtype=torch.float64)
    bias = torch.randn(L2, generator=gen, dtype=torch.float64)
    m1, ll1, o1, m2, ll2, o2, mm, lm, om = ([] for _ in range(9))
    for i in range(R):
        s1 = ref.online_softmax_from_attention(l1[i], v1)
        s2 = ref.online_softmax_from_attention(l2[i], v2, logit_bias=bias)
        s = ref.merge_softmax_states(s1, s2)
        for lst, val in ((m1, s1.m), (ll1, s1.l), (o1, s1.o), (m2, s2.m), (ll2, s2.l), (o2, s2.o),
                         (mm, s.m), (lm, s.l), (om, s.o)):
            lst.append(val.numpy())
    np.savez_compressed(os.path.join(HERE, "online_softmax.npz"),
                        logits1=l1.numpy(), logits2=l2.numpy(), values1=v1.numpy(), values2=v2.numpy(),
                        bias=bias.numpy(), m1=np.array(m1), l1=np.array(ll1), o1=np.array(o1),
                        m2=np.array(m2), l2=np.array(ll2), o2=np.array(o2),
                        m=np.array(mm), l=np.array(lm), o=np.array(om))

    # -- small layer: 4 blocks x 64 tokens, 4 query / 2 KV heads, d 32 --------
    # composed from the reference's build_compact_kv, online_softmax_from_attention
    # and merge_softmax_states; block r attends causally to itself and to
    # C_{s->r} (+beta) for s < r, compacts built from r's destination window.
    gen = torch.Generator().manual_seed(77)
    nb, L, hq, hkv, d, win, M, dp = 4, 64, 4, 2, 32, 24, 8, 8
    budgets = {(s, r): [16, 24, 32][(s + r) % 3] for r in range(nb) for s in range(r)}
    Qb = [torch.randn(hq, L, d, generator=gen, dtype=torch.float64) for _ in range(nb)]
    Kb = [torch.randn(hkv, L, d, generator=gen, dtype=torch.float64) for _ in range(nb)]
    Vb = [torch.randn(hkv, L, d, generator=gen, dtype=torch.float64) for _ in range(nb)]
    group = hq // hkv
    compacts = {}
    for r in range(1, nb):
        for gh in range(hkv):
            dq = torch.cat([Qb[r][h, :win] for h in range(gh * group, (gh + 1) * group)])
            for s in range(r):
                compacts[(s, r, gh)] = ref.build_compact_kv(Kb[s][gh], Vb[s][gh], dq, budgets[(s, r)],
                                                            num_representative_queries=M, projection_dim=dp)
    out = np.zeros((nb, hq, L, d))
    scale = 1.0 / d ** 0.5
    for r in range(nb):
        for h in range(hq):
            gh = h // group
            for i in range(L):
                q = Qb[r][h, i]
                st = ref.online_softmax_from_attention((q @ Kb[r][gh, : i + 1].T) * scale, Vb[r][gh, : i + 1])
                for s in range(r):
                    c = compacts[(s, r, gh)]
                    st = ref.merge_softmax_states(
                        st, ref.online_softmax_from_attention((q @ c.keys.T) * scale, c.values,
                                                              logit_bias=c.logit_bias))
                out[r, h, i] = (st.o / st.l).numpy()
    np.savez_compressed(
        os.path.join(HERE, "layer_small.npz"),
        Q=np.stack([x.numpy() for x in Qb]), K=np.stack([x.numpy() for x in Kb]),
        V=np.stack([x.numpy() for x in Vb]), out=out, window=win, M=M, dp=dp,
        budgets=np.array([[s, r, b] for (s, r), b in sorted(budgets.items())]),
        sel=np.stack([np.stack([compacts[(s, r, gh)].selected_indices.numpy()[:16]
                                for gh in range(hkv)]) for r in range(1, nb) for s in range(r)]))
    print("golden vectors written to", HERE)


def baselines(root: str) -> None:
    """Shared-compaction baselines (src/baselines/fast_kv_cpu.py, apb_cpu.py)
    in float64 on ragged chunks (the last chunk shorter), causal and not."""
    ref, _ = load_reference(root)
    from src.baselines import fast_kv_cpu as _fk  # the package re-exports the functions
    from src.baselines import apb_cpu as _apb
    fast_kv_cpu = _fk if callable(_fk) else _fk.fast_kv_cpu
    apb_cpu = _apb if callable(_apb) else _apb.apb_cpu
    from src.baselines.ring_attention_cpu import ring_attention_cpu
    from src.baselines.fast_kv_cpu import FastKVConfig
    from src.baselines.apb_cpu import APBConfig
    g = torch.Generator().manual_seed(21)
    T, d, chunk, world = 320, 32, 96, 4
    Q = torch.randn(T, d, generator=g, dtype=torch.float64)
    K = torch.randn(T, d, generator=g, dtype=torch.float64)
    V = torch.randn(T, d, generator=g, dtype=torch.float64)
    fcfg = FastKVConfig(budget=24, num_repr_queries=16, projection_dim=8)
    acfg = APBConfig(anchor_budget=20)
    # inputs are not stored: tests redraw them (CPU generator, seed 21, T x d float64: Q, K, V);
    # outputs are stored as float32 (the bar is 1e-4 relative)
    out = dict(seed=21, T=T, d=d, chunk=chunk, world=world, fk_budget=24, fk_M=16, fk_dp=8, apb_budget=20)
    for causal in (True, False):
        tag = "causal" if causal else "full"
        out[f"fastkv_{tag}"] = fast_kv_cpu(Q, K, V, chunk, world, fcfg, causal=causal).float().numpy()
        out[f"apb_{tag}"] = apb_cpu(Q, K, V, chunk, world, acfg, causal=causal).float().numpy()
        bounds = [(s * chunk, (s + 1) * chunk if s < world - 1 else T) for s in range(world)]
        out[f"ring_{tag}"] = ring_attention_cpu(Q, [K[a:b] for a, b in bounds], [V[a:b] for a, b in bounds],
                                                causal=causal).float().numpy()
    np.savez_compressed(os.path.join(HERE, "baselines_small.npz"), **out)
    print("baseline golden vectors written to", HERE)


if __name__ == "__main__":
    if len(sys.argv) < 2:
        sys.exit("usage: make_golden.py REFERENCE_CHECKOUT [baselines]")
    root = sys.argv[1]
    if len(sys.argv) > 2 and sys.argv[2] == "baselines":
        baselines(root)
    else:
        main(root)
        baselines(root)
