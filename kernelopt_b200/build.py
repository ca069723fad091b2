"""Builds libkernelopt.so in-tree (sm_100a only) with nvcc via the Makefile in csrc/.

    python -m kernelopt_b200.build [--clean]
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

CSRC = Path(__file__).with_name("csrc")


def build(clean: bool = False, jobs: int | None = None) -> Path:
    if clean:
        subprocess.run(["make", "-C", str(CSRC), "clean"], check=True)
    jobs = jobs or max(1, min(8, os.cpu_count() or 1))
    subprocess.run(["make", "-C", str(CSRC), f"-j{jobs}"], check=True)
    out = CSRC.parent / "libkernelopt.so"
    if not out.exists():
        raise RuntimeError("build finished without producing libkernelopt.so")
    return out


if __name__ == "__main__":
    print(build(clean="--clean" in sys.argv))
