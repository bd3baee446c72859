"""Build libbs_moe.so in-tree for sm_100a (nvcc cross-compiles without a GPU)."""

from __future__ import annotations

import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")


def build(jobs: int = 8, verbose: bool = False) -> str:
    """Run the csrc Makefile; returns the path of the built library."""
    cmd = ["make", "-C", CSRC, f"-j{jobs}"]
    res = subprocess.run(cmd, capture_output=not verbose, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"building libbs_moe.so failed:\n{res.stdout}\n{res.stderr}")
    return os.path.join(HERE, "libbs_moe.so")


if __name__ == "__main__":
    print(build(verbose=True))
