"""Builds libobjeta_b200.so in-tree with nvcc for sm_100a (no other arch).

    python -m objeta_b200.build
"""
from __future__ import annotations

import os
import subprocess
import sys

_HERE = os.path.dirname(os.path.abspath(__file__))


def build(jobs: int = 8) -> str:
    subprocess.run(["make", "-s", f"-j{jobs}", "-C", os.path.join(_HERE, "csrc")], check=True)
    out = os.path.join(_HERE, "libobjeta_b200.so")
    if not os.path.exists(out):
        raise RuntimeError("build finished without producing libobjeta_b200.so")
    return out


if __name__ == "__main__":
    print(build())
    sys.exit(0)
