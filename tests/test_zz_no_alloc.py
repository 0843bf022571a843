"""The allocation-free single-head build (dcc_build_compact_kv_noalloc).

Some callers cannot call cudaMalloc -- a plugin inside a host application
that owns all device memory through its own fixed pool, or a path where an
allocation could fail or stall.  For them the library keeps a fixed 16 MiB
scratch array on each GPU and this entry point uses it instead of a caller
workspace.  The test calls it through the C ABI twice in a row, on two
different problems (so the second call runs on scratch the first one left
behind), and checks each result against the workspace entry point
dcc_build_compact_kv on the same inputs: indices bit-exact, values and logit
bias within the 1e-4 relative bar used for the float32 path.  It also checks
that a problem too large for the fixed scratch is refused.

The file is named so pytest collects it last.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from dcc_kv_b200 import _lib as L

pytestmark = pytest.mark.gpu


def _inputs(ls, lr, d, seed):
    g = torch.Generator().manual_seed(seed)
    dev = torch.device("cuda", 0)
    return tuple(torch.randn(n, d, generator=g).to(dev) for n in (ls, ls, lr))


def _outputs(b, d):
    dev = torch.device("cuda", 0)
    return (torch.empty(b, d, device=dev), torch.empty(b, device=dev), torch.empty(b, d, device=dev),
            torch.empty(b, dtype=torch.int64, device=dev))


def _run(noalloc, K, V, Q, budget, m=64, dp=32):
    lib = L.lib()
    ls, d = K.shape
    lr = Q.shape[0]
    bp = min(budget, ls)
    keys, bias, values, idx = _outputs(bp, d)
    stream = torch.cuda.current_stream().cuda_stream
    common = (K.data_ptr(), V.data_ptr(), Q.data_ptr(), ls, lr, d, d, budget, m, dp, 1e-3, 1e-3, 42, L.DCC_F32,
              keys.data_ptr(), bias.data_ptr(), values.data_ptr(), idx.data_ptr(), None)
    if noalloc:
        rc = lib.dcc_build_compact_kv_noalloc(*common, stream)
    else:
        ws = torch.empty(lib.dcc_build_compact_kv_workspace(ls, lr, d, d, budget, m, dp, L.DCC_F32),
                         dtype=torch.uint8, device=K.device)
        rc = lib.dcc_build_compact_kv(*common, ws.data_ptr(), ws.numel(), stream)
    L.check(rc, "build")
    torch.cuda.synchronize()
    return keys, bias, values, idx


def _rel(a, b):
    a, b = a.double().cpu().numpy(), b.double().cpu().numpy()
    return np.abs(a - b).max() / np.abs(b).max()


def test_noalloc_matches_workspace_entry_point_twice():
    cases = [(_inputs(4096, 512, 128, 0), 64),     # config-1 shape: B == M, projected-gradient branch
             (_inputs(2048, 700, 128, 1), 256)]    # B > M: closed-form branch
    for (K, V, Q), budget in cases:
        got = _run(True, K, V, Q, budget)
        want = _run(False, K, V, Q, budget)
        np.testing.assert_array_equal(got[3].cpu().numpy(), want[3].cpu().numpy())
        np.testing.assert_array_equal(got[0].cpu().numpy(), want[0].cpu().numpy())
        assert _rel(got[1], want[1]) < 1e-4
        assert _rel(got[2], want[2]) < 1e-4


def test_noalloc_rejects_oversized_problem():
    lib = L.lib()
    ls, lr, d = 1 << 20, 1 << 16, 128
    assert lib.dcc_build_compact_kv_workspace(ls, lr, d, d, 4096, 64, 32, L.DCC_F32) > (16 << 20)
    dummy = torch.empty(1, device="cuda")
    p = dummy.data_ptr()
    rc = lib.dcc_build_compact_kv_noalloc(p, p, p, ls, lr, d, d, 4096, 64, 32, 1e-3, 1e-3, 42, L.DCC_F32,
                                          p, p, p, p, None, torch.cuda.current_stream().cuda_stream)
    assert rc == L.DCC_ERR_UNSUPPORTED
    assert b"16777216" in lib.dcc_last_error()
