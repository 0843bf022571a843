"""CPU oracle for the DCC-KV compact-KV path.

TEST INFRASTRUCTURE ONLY.  This module is the checker: only ``tests/``,
``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` may import
it.  The product path (``dcc_kv_b200``) never calls it and has no CPU fallback.

It restates the reference algorithm (lfei7199-star/dcc-kv, ``src/dcc_kv_ref``)
in numpy float64, function by function, with the reference's own numerical
quirks preserved (see each docstring for the file:line it follows).  It is
pinned against golden vectors produced by running the reference itself
(``tests/golden/make_golden.py``) and against torch's CPU generator for the
two random draws.

Deliberate restatement differences (all exact in real arithmetic):
  * farthest-point sampling computes each distance row on demand instead of
    materialising the N x N matrix (representative_query.py:63-65);
  * top-k breaks exact score ties by the lower token index (torch.topk's
    order for exact ties is unspecified).
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np

F64 = np.float64


# ---------------------------------------------------------------------------
# Random draws (torch.Generator on CPU == raw mt19937, value % range)
# ---------------------------------------------------------------------------
def mt19937_raw(seed: int, n: int) -> np.ndarray:
    """First ``n`` raw 32-bit outputs of mt19937 seeded like
    ``torch.Generator().manual_seed(seed)`` (init_genrand with the low 32
    bits of the seed).  numpy's legacy RandomState uses the same seeding."""
    bg = np.random.RandomState(seed & 0xFFFFFFFF)._bit_generator
    return np.fromiter((bg.random_raw() for _ in range(n)), dtype=np.uint64, count=n)


def rademacher_projection(head_dim: int, projection_dim: int = 32, seed: int = 42) -> np.ndarray:
    """P[d_p, d] = (2*randint{0,1} - 1) / sqrt(d_p), rounded through float32
    exactly as representative_query.py:28-30 does, returned as float64 (the
    FP64 shim casts the float32 matrix to the query dtype)."""
    raw = mt19937_raw(seed, projection_dim * head_dim) % 2
    signs = (raw.astype(np.int64) * 2 - 1).astype(np.float32)
    proj = signs / np.float32(projection_dim ** 0.5)
    return proj.astype(np.float32).reshape(projection_dim, head_dim).astype(F64)


def fps_start_index(num_points: int, seed: int = 42) -> int:
    """``int(torch.randint(0, N, (1,), generator=Generator().manual_seed(seed)))``
    (representative_query.py:68)."""
    return int(mt19937_raw(seed, 1)[0] % np.uint64(num_points))


# ---------------------------------------------------------------------------
# Representative queries  (representative_query.py)
# ---------------------------------------------------------------------------
def _row_normalise(x: np.ndarray) -> np.ndarray:
    return x / (np.linalg.norm(x, axis=-1, keepdims=True) + 1e-8)


def farthest_point_sampling(features: np.ndarray, num_samples: int, seed: int = 42) -> np.ndarray:
    """representative_query.py:34-79.  Re-normalises the (already normalised)
    features, cosine distance 1 - <u, v>, random start, then M-1 steps of
    ``argmax(min_dist)`` (first maximum) and ``min_dist = min(min_dist, dist[next])``."""
    n = features.shape[0]
    if num_samples >= n:
        return np.arange(n, dtype=np.int64)
    normed = _row_normalise(np.asarray(features, dtype=F64))
    start = fps_start_index(n, seed)
    selected = [start]
    min_dist = 1.0 - normed @ normed[start]
    for _ in range(num_samples - 1):
        nxt = int(np.argmax(min_dist))
        selected.append(nxt)
        min_dist = np.minimum(min_dist, 1.0 - normed @ normed[nxt])
    return np.asarray(selected, dtype=np.int64)


def projected_features(queries: np.ndarray, projection_dim: int = 32, seed: int = 42) -> np.ndarray:
    """z = Q P^T, z /= (||z|| + 1e-8)  (representative_query.py:106-108)."""
    proj = rademacher_projection(queries.shape[-1], projection_dim, seed)
    z = np.asarray(queries, dtype=F64) @ proj.T
    return _row_normalise(z)


def select_representative_queries(queries: np.ndarray, num_samples: int = 64,
                                  projection_dim: int = 32, seed: int = 42):
    """representative_query.py:82-110 -> (Q[idx], idx)."""
    q = np.asarray(queries, dtype=F64)
    z = projected_features(q, projection_dim, seed)
    idx = farthest_point_sampling(z, num_samples, seed)
    return q[idx], idx


# ---------------------------------------------------------------------------
# Key selection  (key_selection.py)
# ---------------------------------------------------------------------------
def softmax(x: np.ndarray, axis: int = -1) -> np.ndarray:
    m = np.max(x, axis=axis, keepdims=True)
    e = np.exp(x - m)
    return e / np.sum(e, axis=axis, keepdims=True)


def rms_per_token_score(attention_weights: np.ndarray) -> np.ndarray:
    """key_selection.py:14-26: u_j = sqrt(sum_a A_aj^2 / M)."""
    a = np.asarray(attention_weights, dtype=F64)
    return np.sqrt((a ** 2).sum(axis=0) / a.shape[0])


def topk_desc(scores: np.ndarray, k: int) -> np.ndarray:
    """Indices of the k largest scores, sorted by (score desc, index asc)."""
    order = np.argsort(-np.asarray(scores, dtype=F64), kind="stable")
    return order[:k].astype(np.int64)


def attention_scores(keys: np.ndarray, repr_queries: np.ndarray) -> np.ndarray:
    """softmax(Q^ K^T / sqrt(d)) over the keys (key_selection.py:52-54)."""
    d = keys.shape[1]
    return softmax((repr_queries @ keys.T) * (1.0 / d ** 0.5), axis=-1)


def select_topk_keys(keys: np.ndarray, repr_queries: np.ndarray, budget: int):
    """key_selection.py:29-62 -> (K[idx], idx); early exit when budget >= L_s."""
    k = np.asarray(keys, dtype=F64)
    ls = k.shape[0]
    if budget >= ls:
        return k, np.arange(ls, dtype=np.int64)
    u = rms_per_token_score(attention_scores(k, np.asarray(repr_queries, dtype=F64)))
    idx = topk_desc(u, budget)
    return k[idx], idx


# ---------------------------------------------------------------------------
# Calibration  (calibration.py)
# ---------------------------------------------------------------------------
def nonneg_least_squares(G: np.ndarray, target: np.ndarray, lambda_reg: float = 1e-3,
                         n_iter: int = 100) -> np.ndarray:
    """calibration.py:17-60.  Ridge start clamp(solve(G^T G + lam I, G^T t), 0)
    (toward 0); returned as-is when M < B; otherwise ``n_iter`` projected
    gradient steps with lr 1e-2 whose ridge term pulls toward 1."""
    G = np.asarray(G, dtype=F64)
    t = np.asarray(target, dtype=F64)
    m, b = G.shape
    gtg = G.T @ G + lambda_reg * np.eye(b, dtype=F64)
    w = np.maximum(np.linalg.solve(gtg, G.T @ t), 0.0)
    if m < b:
        return w
    lr = 1e-2
    for _ in range(n_iter):
        grad = G.T @ (G @ w - t) + lambda_reg * (w - 1.0)
        w = np.maximum(w - lr * grad, 0.0)
    return w


def fit_logit_bias(repr_queries: np.ndarray, compact_keys: np.ndarray,
                   block_mass: np.ndarray, lambda_reg: float = 1e-3) -> np.ndarray:
    """calibration.py:63-94: G = exp(Q^ C_K^T / sqrt(d)), w = NNLS, beta = log(max(w, 1e-6))."""
    d = repr_queries.shape[1]
    G = np.exp((repr_queries @ compact_keys.T) * (1.0 / d ** 0.5))
    w = nonneg_least_squares(G, block_mass, lambda_reg=lambda_reg)
    return np.log(np.maximum(w, 1e-6))


# ---------------------------------------------------------------------------
# Value regression  (value_regression.py)
# ---------------------------------------------------------------------------
def ridge_regression_value(X: np.ndarray, Y: np.ndarray, lambda_reg: float = 1e-3) -> np.ndarray:
    """value_regression.py:15-35: (X^T X + lam I)^-1 X^T Y."""
    b = X.shape[1]
    return np.linalg.solve(X.T @ X + lambda_reg * np.eye(b, dtype=F64), X.T @ Y)


def fit_compact_value(repr_queries, original_keys, original_values, compact_keys,
                      logit_bias, lambda_reg: float = 1e-3) -> np.ndarray:
    """value_regression.py:38-78: Y = softmax(Q^K^T/sqrt d) V,
    X = softmax(Q^ C_K^T/sqrt d + beta/M) (beta divided by M here only)."""
    m, d = repr_queries.shape
    scale = 1.0 / d ** 0.5
    Y = softmax((repr_queries @ original_keys.T) * scale, axis=-1) @ original_values
    X = softmax((repr_queries @ compact_keys.T) * scale + logit_bias[None, :] / m, axis=-1)
    return ridge_regression_value(X, Y, lambda_reg=lambda_reg)


# ---------------------------------------------------------------------------
# CompactKV + build  (compact_kv.py)
# ---------------------------------------------------------------------------
@dataclass(frozen=True)
class CompactKV:
    keys: np.ndarray
    logit_bias: np.ndarray
    values: np.ndarray
    selected_indices: np.ndarray
    repr_indices: Optional[np.ndarray] = None
    block_mass: Optional[np.ndarray] = None


def build_compact_kv(source_keys, source_values, destination_queries, budget: int,
                     num_representative_queries: int = 64, projection_dim: int = 32,
                     lambda_beta: float = 1e-3, lambda_value: float = 1e-3,
                     seed: int = 42) -> CompactKV:
    """compact_kv.py:50-118 (four stages; block mass = row sums of the
    normalised attention, which is 1 up to rounding, compact_kv.py:97-101)."""
    K = np.asarray(source_keys, dtype=F64)
    V = np.asarray(source_values, dtype=F64)
    Q = np.asarray(destination_queries, dtype=F64)
    qh, ridx = select_representative_queries(Q, num_representative_queries, projection_dim, seed)
    ck, sidx = select_topk_keys(K, qh, budget)
    mass = attention_scores(K, qh).sum(axis=-1)
    beta = fit_logit_bias(qh, ck, mass, lambda_reg=lambda_beta)
    cv = fit_compact_value(qh, K, V, ck, beta, lambda_reg=lambda_value)
    return CompactKV(ck, beta, cv, sidx, ridx, mass)


def build_compact_kv_from_repr(source_keys, source_values, repr_queries, budget: int,
                               lambda_beta: float = 1e-3, lambda_value: float = 1e-3) -> CompactKV:
    """Stages 2-4 of compact_kv.py:50-118 for given representative queries."""
    K = np.asarray(source_keys, dtype=F64)
    V = np.asarray(source_values, dtype=F64)
    qh = np.asarray(repr_queries, dtype=F64)
    ck, sidx = select_topk_keys(K, qh, budget)
    mass = attention_scores(K, qh).sum(axis=-1)
    beta = fit_logit_bias(qh, ck, mass, lambda_reg=lambda_beta)
    cv = fit_compact_value(qh, K, V, ck, beta, lambda_reg=lambda_value)
    return CompactKV(ck, beta, cv, sidx, None, mass)


# ---------------------------------------------------------------------------
# Online softmax  (online_softmax.py)
# ---------------------------------------------------------------------------
def online_softmax_state(logits: np.ndarray, values: np.ndarray, logit_bias=None):
    """online_softmax.py:52-89, batched over leading dims of ``logits``
    [..., L] with ``values`` [..., L, d]: (m, l, o) with o unnormalised."""
    x = np.asarray(logits, dtype=F64)
    if logit_bias is not None:
        x = x + logit_bias
    m = x.max(axis=-1)
    e = np.exp(x - m[..., None])
    l = e.sum(axis=-1)
    o = np.einsum("...l,...ld->...d", e, np.asarray(values, dtype=F64))
    return m, l, o


def merge_states(a, b):
    """online_softmax.py:92-111 on (m, l, o) triples."""
    ma, la, oa = a
    mb, lb, ob = b
    m = np.maximum(ma, mb)
    ea = np.exp(ma - m)
    eb = np.exp(mb - m)
    return m, ea * la + eb * lb, ea[..., None] * oa + eb[..., None] * ob


def merge_lse(outputs: Sequence[np.ndarray], lses: Sequence[np.ndarray]):
    """P-way merge of normalised partial outputs O_p with log-sum-exp L_p:
    the state (m=L_p, l=1, o=O_p) folded left to right with merge_states."""
    state = (np.asarray(lses[0], F64), np.ones_like(lses[0], dtype=F64), np.asarray(outputs[0], F64))
    for o, lse in zip(outputs[1:], lses[1:]):
        state = merge_states(state, (np.asarray(lse, F64), np.ones_like(lse, dtype=F64), np.asarray(o, F64)))
    m, l, o = state
    return o / l[..., None], m + np.log(l)


# ---------------------------------------------------------------------------
# Attention pieces used by the layer (dcc_kv_sync_cpu.py, full_attention_cpu.py)
# ---------------------------------------------------------------------------
def attention_partial(q: np.ndarray, k: np.ndarray, v: np.ndarray, bias=None,
                      positions: Optional[np.ndarray] = None):
    """Normalised attention output and LSE for query rows ``q`` [R, d] over
    keys ``k`` [L, d].  ``bias`` [L] is added to the logits at full weight
    (dcc_kv_sync_cpu.py:71-73).  ``positions`` [R]: causal mask, query row i
    may see keys j <= positions[i] (full_attention_cpu.py:104-107)."""
    d = q.shape[-1]
    s = (np.asarray(q, F64) @ np.asarray(k, F64).T) * (1.0 / d ** 0.5)
    if bias is not None:
        s = s + np.asarray(bias, F64)[None, :]
    if positions is not None:
        s = np.where(np.arange(k.shape[0])[None, :] <= np.asarray(positions)[:, None], s, -np.inf)
    m = s.max(axis=-1)
    e = np.exp(s - m[:, None])
    l = e.sum(axis=-1)
    o = (e @ np.asarray(v, F64)) / l[:, None]
    return o, m + np.log(l)


def destination_window(q_block: np.ndarray, kv_head: int, group: int, window: int) -> np.ndarray:
    """Destination queries for one KV head: the first ``window`` rows of each
    of its ``group`` query heads, concatenated head by head.  ``q_block`` is
    [Hq, L, d]."""
    heads = range(kv_head * group, (kv_head + 1) * group)
    return np.concatenate([np.asarray(q_block[h, :window], F64) for h in heads], axis=0)


def layer_forward(q_blocks: List[np.ndarray], k_blocks: List[np.ndarray], v_blocks: List[np.ndarray],
                  budgets: Dict[Tuple[int, int], int], window: int,
                  num_representative_queries: int = 64, projection_dim: int = 32,
                  lambda_beta: float = 1e-3, lambda_value: float = 1e-3, seed: int = 42,
                  rows: Optional[Dict[int, np.ndarray]] = None):
    """DCC-KV sync layer over logical blocks (all arrays head-major:
    Q [Hq, L, d], K/V [Hkv, L, d]).  Block r attends causally to itself and,
    for every s < r, to C_{s->r} built from r's destination queries with the
    logit bias added at full weight; the partial states are merged in block
    order (dcc_kv_sync_cpu.py:52-84, compact built as compact_kv.py:50-118).

    ``rows``: optional {block: query-row indices} to evaluate only a sample.
    Returns ({block: O [Hq, R, d]}, {(s, r, kv_head): CompactKV})."""
    nb = len(q_blocks)
    hq, _, d = q_blocks[0].shape
    hkv = k_blocks[0].shape[0]
    group = hq // hkv
    compacts = {}
    for r in range(1, nb):
        for g in range(hkv):
            dq = destination_window(q_blocks[r], g, group, window)
            qh, ridx = select_representative_queries(dq, num_representative_queries, projection_dim, seed)
            for s in range(r):
                c = build_compact_kv_from_repr(k_blocks[s][g], v_blocks[s][g], qh, budgets[(s, r)],
                                               lambda_beta, lambda_value)
                compacts[(s, r, g)] = CompactKV(c.keys, c.logit_bias, c.values, c.selected_indices,
                                                ridx, c.block_mass)
    out = {}
    for r in range(nb):
        L = q_blocks[r].shape[1]
        sel = np.arange(L) if rows is None or r not in rows else np.asarray(rows[r])
        o_r = np.zeros((hq, len(sel), d))
        for h in range(hq):
            g = h // group
            q = np.asarray(q_blocks[r][h][sel], F64)
            # local block, causal: row i sees keys [0, sel[i]]
            o_l, lse_l = attention_partial(q, k_blocks[r][g], v_blocks[r][g], positions=sel)
            state = (lse_l, np.ones_like(lse_l), o_l)
            for src in range(r):
                c = compacts[(src, r, g)]
                o_c, lse_c = attention_partial(q, c.keys, c.values, bias=c.logit_bias)
                state = merge_states(state, (lse_c, np.ones_like(lse_c), o_c))
            m, l, o = state
            o_r[h] = o / l[:, None]
        out[r] = o_r
    return out, compacts


def full_causal_attention(q_full: np.ndarray, k_full: np.ndarray, v_full: np.ndarray,
                          rows: np.ndarray) -> np.ndarray:
    """Dense causal attention (full_attention_cpu.py:69-113) for selected
    global row indices of one head: q_full [T, d], k/v_full [T, d]."""
    d = q_full.shape[-1]
    out = np.zeros((len(rows), v_full.shape[-1]))
    for i, r in enumerate(rows):
        s = (np.asarray(k_full[: r + 1], F64) @ np.asarray(q_full[r], F64)) * (1.0 / d ** 0.5)
        p = softmax(s)
        out[i] = p @ np.asarray(v_full[: r + 1], F64)
    return out


# ---------------------------------------------------------------------------
# Shared-compaction baselines (src/baselines): one compact per source chunk,
# used by every later query, with the reference's causal prefix on the compact
# index (query r sees the first r + 1 - offset_s entries of chunk s's compact).
# ---------------------------------------------------------------------------
def _chunk_bounds(total: int, chunk_size: int, world_size: int):
    """fast_kv_cpu.py:68-71 / apb_cpu.py:99-102: chunk s = [s * chunk, (s + 1) * chunk),
    the last chunk runs to the end of the sequence."""
    out = []
    for s in range(world_size):
        lo = s * chunk_size
        hi = (s + 1) * chunk_size if s < world_size - 1 else total
        out.append((lo, hi))
    return out


def _ring_over_compacts(queries, compacts, offsets, causal: bool):
    """fast_kv_cpu.py:89-125 / apb_cpu.py:117-146: every query row merges one
    online-softmax state per visible chunk; rows with none get zeros.
    ``compacts``: list of (keys, values, bias or None)."""
    q = np.asarray(queries, F64)
    T, d = q.shape
    dv = compacts[0][1].shape[-1]
    out = np.zeros((T, dv))
    scale = 1.0 / d ** 0.5
    for r in range(T):
        state = None
        for (k, v, bias), off in zip(compacts, offsets):
            if causal and off > r:
                continue
            n = min(r + 1 - off, k.shape[0]) if causal else k.shape[0]
            if n <= 0:
                continue
            logits = (np.asarray(k[:n], F64) @ q[r]) * scale
            st = online_softmax_state(logits, np.asarray(v[:n], F64), None if bias is None else bias[:n])
            state = st if state is None else merge_states(state, st)
        if state is not None:
            out[r] = state[2] / state[1]
    return out


def fast_kv(queries, keys, values, chunk_size: int, world_size: int, budget: int = 256,
            num_repr_queries: int = 64, projection_dim: int = 32, lambda_beta: float = 1e-3,
            lambda_value: float = 1e-3, seed: int = 42, causal: bool = True):
    """fast_kv_cpu.py:35-125: each chunk is compacted once with ALL queries as
    destination queries (min(budget, chunk) entries), then ring attention
    over the compacts with their logit bias."""
    T = queries.shape[0]
    compacts, offsets = [], []
    for lo, hi in _chunk_bounds(T, chunk_size, world_size):
        c = build_compact_kv(keys[lo:hi], values[lo:hi], queries, min(budget, hi - lo), num_repr_queries,
                             projection_dim, lambda_beta, lambda_value, seed)
        compacts.append((c.keys, c.values, c.logit_bias))
        offsets.append(lo)
    return _ring_over_compacts(queries, compacts, offsets, causal)


def select_anchor_blocks(keys, values, queries, budget: int):
    """apb_cpu.py:36-61: the ``budget`` keys with the largest attention mass
    sum_a softmax(q_a K^T / sqrt(d))[j] over the given queries (sorted by mass,
    ties by lower index)."""
    d = keys.shape[-1]
    A = softmax((np.asarray(queries, F64) @ np.asarray(keys, F64).T) * (1.0 / d ** 0.5))
    idx = topk_desc(A.sum(axis=0), budget)
    return np.asarray(keys, F64)[idx], np.asarray(values, F64)[idx], idx


def apb(queries, keys, values, chunk_size: int, world_size: int, anchor_budget: int = 128,
        causal: bool = True):
    """apb_cpu.py:64-152: anchors of chunk s chosen by the attention mass of
    queries[offset_s:] (all queries if that is empty), then ring attention
    over the anchors (no bias)."""
    T = queries.shape[0]
    compacts, offsets = [], []
    for lo, hi in _chunk_bounds(T, chunk_size, world_size):
        fut = queries[lo:] if T - lo > 0 else queries
        ak, av, _ = select_anchor_blocks(keys[lo:hi], values[lo:hi], fut, min(anchor_budget, hi - lo))
        compacts.append((ak, av, None))
        offsets.append(lo)
    return _ring_over_compacts(queries, compacts, offsets, causal)
