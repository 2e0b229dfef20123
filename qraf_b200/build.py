"""Build libqraf_cuda.so in-tree with nvcc for sm_100a.

    python -m qraf_b200.build          # rebuild when a source is newer than the .so
"""
from __future__ import annotations

import glob
import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
LIB = os.path.join(PKG, "libqraf_cuda.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
# -fmad=false: no multiply/add pair is ever contracted into an FMA.  The EXACT
# kernels depend on separately rounded products and sums (the reference's x86
# order); every FMA the FAST kernels want is written explicitly.
CUDA_FLAGS = ["-std=c++17", "-O3", "-lineinfo", "-fmad=false", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
              "--expt-relaxed-constexpr"]


def sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cuh")) +
                  glob.glob(os.path.join(CSRC, "*.cpp")) + glob.glob(os.path.join(ROOT, "include", "*.h")))


def needs_build() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    return any(os.path.getmtime(s) > t for s in sources())


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and not needs_build():
        return LIB
    units = [os.path.join(CSRC, "capi.cu")]
    cmd = [NVCC, *ARCH_FLAGS, *CUDA_FLAGS, "-shared", "-o", LIB + ".tmp", *units]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True, cwd=ROOT)
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB)
