"""Build ``libdcckv.so`` for sm_100a in-tree: ``python -m dcc_kv_b200.build``.

nvcc cross-compiles without a GPU.  Objects go to ``_build/`` at the repo
root; the library lands next to this file so it travels with the package.
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))


def build(jobs: int = 8, verbose: bool = False) -> str:
    csrc = os.path.join(HERE, "csrc")
    cmd = ["make", "-C", csrc, f"-j{jobs}"]
    r = subprocess.run(cmd, capture_output=not verbose, text=True)
    if r.returncode != 0:
        sys.stderr.write((r.stdout or "") + (r.stderr or ""))
        raise RuntimeError("building libdcckv.so failed")
    return os.path.join(HERE, "libdcckv.so")


if __name__ == "__main__":
    print(build(verbose=True))
