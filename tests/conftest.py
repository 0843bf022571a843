"""Shared pytest setup: the ``gpu`` marker and paths.

``-m "not gpu"`` runs on a CPU-only machine: the oracle against the golden
vectors, host logic, the C-ABI library's symbol table and gloo multi-process
tests.  ``-m gpu`` runs the CUDA kernels against the oracle on a B200.
"""
from __future__ import annotations

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: long-running case")


@pytest.fixture(scope="session")
def golden_dir():
    return GOLDEN
