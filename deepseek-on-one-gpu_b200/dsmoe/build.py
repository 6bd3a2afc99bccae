"""Build ``libdsmoe.so`` for sm_100a in-tree (``csrc/Makefile``)."""
from __future__ import annotations

import os
import subprocess
import sys

CSRC = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "csrc")


def build(verbose: bool = False) -> str:
    cmd = ["make", "-C", CSRC]
    r = subprocess.run(cmd, capture_output=not verbose, text=True)
    if r.returncode != 0:
        sys.stderr.write((r.stdout or "") + (r.stderr or ""))
        raise RuntimeError("libdsmoe build failed")
    from ._lib import LIB_PATH
    return LIB_PATH


if __name__ == "__main__":
    print(build(verbose=True))
