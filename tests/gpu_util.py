"""Helpers shared by the GPU parity tests."""
from __future__ import annotations

import os

import numpy as np
import torch

from conftest import GOLDEN


def dev():
    return torch.device("cuda", 0)


def golden(name):
    return np.load(os.path.join(GOLDEN, name))


def to_gpu(a, dtype):
    return torch.as_tensor(np.asarray(a, dtype=np.float64)).to(dtype).to(dev())


def np64(t):
    return t.detach().double().cpu().numpy()


def rel_err(got, want) -> float:
    """max |got - want| / max |want|  (the relative tolerance used throughout)."""
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    return float(np.abs(got - want).max() / max(np.abs(want).max(), 1e-300))


def build_inputs(f, name):
    if name == "build_cfg1.npz":
        g = torch.Generator().manual_seed(0)
        K = torch.randn(4096, 128, generator=g, dtype=torch.float64).numpy()
        V = torch.randn(4096, 128, generator=g, dtype=torch.float64).numpy()
        Q = torch.randn(512, 128, generator=g, dtype=torch.float64).numpy()
        return K, V, Q
    return f["K"].astype(np.float64), f["V"].astype(np.float64), f["Q"].astype(np.float64)


def assert_no_device_timeouts():
    """No bounded device-side wait (tcgen05 attention, tcgen05 scoring) expired."""
    from dcc_kv_b200 import _lib as L
    assert L.lib().dcc_device_error_status(1) == 0, "attention: a bounded device wait expired"
    assert L.lib().dcc_build_error_status(1) == 0, "scoring: a bounded device wait expired"


def baseline_inputs(f):
    """Q, K, V of the baseline fixtures: drawn again with torch's CPU generator
    (seed from the fixture, T x d float64, in that order)."""
    g = torch.Generator().manual_seed(int(f["seed"]))
    T, d = int(f["T"]), int(f["d"])
    return tuple(torch.randn(T, d, generator=g, dtype=torch.float64) for _ in range(3))
