"""Builds libtinyoai_cuda.so in-tree with nvcc for sm_100a.

The library is a single translation unit (csrc/runtime.cu) with the C ABI of
include/tinyoai_cuda.h. nvcc cross-compiles without a GPU.
"""
import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
LIB = PKG / "libtinyoai_cuda.so"
SOURCES = [PKG / "csrc" / "runtime.cu"]
DEPS = sorted((PKG / "csrc").glob("*.cu*")) + [ROOT / "include" / "tinyoai_cuda.h"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
    "-Xcudafe", "--diag_suppress=177",
]


def nvcc():
    for cand in [os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"]:
        if cand and (os.path.isabs(cand) and os.path.exists(cand) or not os.path.isabs(cand)):
            return cand
    return "nvcc"


def stale():
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    return any(p.stat().st_mtime > t for p in DEPS)


def build(force=False, verbose=False):
    if not force and not stale():
        return LIB
    cmd = [nvcc(), *NVCC_FLAGS, "-o", str(LIB) + ".tmp", *map(str, SOURCES)]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(str(LIB) + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
    print(LIB)
