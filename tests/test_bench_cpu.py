"""The benchmark's workload arithmetic on CPU: algorithmic FLOPs and bytes
of each configuration (the denominators of its roofline figures) and the
per-edge budget tables."""
from __future__ import annotations

import bench


def test_layer_128k_attention_flops_and_bytes():
    wl = bench._layer_128k()
    local, compact = bench.causal_attention_flops(wl)
    assert wl.tokens == 131072 and len(wl.budgets) == 28
    # local causal: 8 blocks x 32 heads x L(L+1)/2 pairs x 4 d; compact: block r sees r x 1024 keys
    assert local == 8 * 32 * (16384 * 16385 // 2) * 4 * 128
    assert compact == sum(32 * 16384 * r * 1024 * 4 * 128 for r in range(8))
    assert local + compact == 25_289_841_180_672
    read, write = bench.attention_bytes(wl, [wl.compact_rows(r) for r in range(8)])
    assert write == 8 * 32 * 16384 * 128 * 2
    assert bench.attention_traffic(wl) > read + write * 0.99


def test_layer_1m_variable_budgets():
    wl = bench._layer_1m()
    assert wl.tokens == 1 << 20
    assert set(wl.budgets.values()) <= {256, 512, 1024, 2048} and len(wl.budgets) == 28
    assert bench.attention_traffic(wl) is None  # nothing profiled at this size
    assert sum(bench.causal_attention_flops(wl)) == 1_176_486_031_654_912


def test_merge_and_build_bytes():
    assert bench.MERGE_BYTES == 8 * 32 * 4096 * (128 * 2 + 4) + 32 * 4096 * (128 * 2 + 4) == 306_708_480
    assert bench.MERGE_PROFILED_DRAM <= bench.MERGE_BYTES
    assert bench._build_bytes() == 2 * 8 * 16384 * 128 * 2 + 32 * 2048 * 128 * 2 + 8 * 512 * (2 * 128 * 2 + 12)
