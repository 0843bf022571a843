"""The C-ABI library on a CPU-only machine: it loads, exports every symbol
include/dcc_kv.h declares (and the ctypes table binds them), its host-side
random draws equal torch's CPU generator, and the compute entry points
reject bad arguments before touching a device."""
from __future__ import annotations

import ctypes as C
import os
import re

import numpy as np
import pytest
import torch

from conftest import ROOT

from dcc_kv_b200 import _lib as L

HEADER = os.path.join(ROOT, "include", "dcc_kv.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(dcc_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = L.lib()
    names = declared_functions()
    assert len(names) >= 20
    for n in names:
        assert hasattr(lib, n), f"{n} declared in dcc_kv.h but not exported"
        assert n in L.SIGNATURES, f"{n} has no ctypes signature"
    assert set(L.SIGNATURES) == set(names)


def test_status_strings():
    lib = L.lib()
    assert lib.dcc_status_string(0) == b"ok"
    assert lib.dcc_status_string(L.DCC_ERR_WORKSPACE) == b"workspace too small"
    assert lib.dcc_version() >= 2


def test_ctypes_struct_layouts_match_the_library():
    lib = L.lib()
    for cls in (L.dcc_query_set, L.dcc_build_problem, L.dcc_kv_segment, L.dcc_attn_problem):
        assert lib.dcc_struct_size(cls.__name__.encode()) == C.sizeof(cls), cls.__name__
    assert lib.dcc_struct_size(b"no_such_struct") == 0


@pytest.mark.parametrize("seed,dp,d", [(42, 32, 128), (0, 8, 32), (12345, 16, 64), (7, 5, 7)])
def test_projection_matches_torch(seed, dp, d):
    buf = (C.c_float * (dp * d))()
    assert L.lib().dcc_rademacher_projection(d, dp, seed, buf) == 0
    got = np.frombuffer(buf, dtype=np.float32).reshape(dp, d)
    g = torch.Generator().manual_seed(seed)
    want = (torch.randint(0, 2, (dp, d), generator=g) * 2 - 1).float() / (dp ** 0.5)
    np.testing.assert_array_equal(got, want.numpy())


def test_fps_start_matches_torch():
    for seed in (0, 1, 42, 99999):
        for n in (1, 7, 512, 8192, 123457):
            g = torch.Generator().manual_seed(seed)
            assert L.lib().dcc_fps_start_index(n, seed) == int(torch.randint(0, n, (1,), generator=g))


def test_argument_errors_without_device():
    lib = L.lib()
    # bad sizes are rejected on the host, before any CUDA call
    assert lib.dcc_merge_lse(None, None, 0, 4, 4, 0, None, None, None) == L.DCC_ERR_INVALID_ARGUMENT
    assert lib.dcc_attention_fwd(None, 1, 4, 3, 128, 1.0, 1, None) == L.DCC_ERR_INVALID_ARGUMENT
    p = L.dcc_build_problem()
    assert lib.dcc_build_compact_kv_batched(C.byref(p), 1, 128, 128, 1e-3, 1e-3, 1, None, 0, None) \
        == L.DCC_ERR_INVALID_ARGUMENT
    with pytest.raises(ValueError):
        L.check(L.DCC_ERR_INVALID_ARGUMENT, "x")
    with pytest.raises(AssertionError):
        L.check(L.DCC_ERR_SHAPE, "x")
    with pytest.raises(L.DccError):
        L.check(L.DCC_ERR_CUDA, "x")


def test_cpu_tensors_fail_loudly():
    import dcc_kv_b200 as dk
    x = torch.zeros(4, 8)
    with pytest.raises(ValueError, match="CUDA"):
        dk.build_compact_kv(x, x, x, 2)
    with pytest.raises(ValueError, match="CUDA"):
        dk.merge_lse([x], [x[:, 0]])
