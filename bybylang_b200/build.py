"""Builds libbybycuda.so in-tree for sm_100a (`python -m bybylang_b200.build`)."""
from __future__ import annotations

import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))


def build(verbose: bool = False) -> str:
    subprocess.run(["make", "-C", os.path.join(HERE, "csrc")] + ([] if verbose else ["-s"]), check=True)
    return os.path.join(HERE, "libbybycuda.so")


if __name__ == "__main__":
    print(build(verbose=True))
