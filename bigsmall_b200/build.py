"""Build the in-tree CUDA extension ``bigsmall_b200/libbsgpu.so`` (sm_100a).

nvcc cross-compiles without a GPU.  Flags: ``-gencode
arch=compute_100a,code=sm_100a -O3 -lineinfo`` (see csrc/Makefile).
"""
from __future__ import annotations

import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libbsgpu.so")


def build(verbose: bool = False, extra_flags: str = "") -> str:
    cmd = ["make", "-C", CSRC]
    if not verbose:
        cmd.insert(1, "-s")
    if extra_flags:
        cmd.append(f"EXTRA_NVFLAGS={extra_flags}")
    subprocess.run(cmd, check=True)
    if not os.path.exists(LIB):
        raise RuntimeError(f"build did not produce {LIB}")
    return LIB


if __name__ == "__main__":
    print(build(verbose=True))
