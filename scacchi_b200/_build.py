"""Build the CUDA library in-tree (sm_100a only)."""

from __future__ import annotations

import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libscacchi_b200.so")
SOURCES = [os.path.join(CSRC, "search.cu")]
HEADERS = [os.path.join(CSRC, h) for h in ("smath.h", "threefry.h", "synthetic_env.h")] + [
    os.path.join(ROOT, "include", "scacchi_b200.h")]

NVCC_FLAGS = [
    "-O3", "-std=c++17", "-shared", "-Xcompiler", "-fPIC",
    "-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo",
    # Bit-reproducibility with the oracle: no implicit multiply-add
    # contraction; the kernels use explicit fmaf() where they want one.
    "-fmad=false",
]


def nvcc() -> str:
    cuda = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    path = os.path.join(cuda, "bin", "nvcc")
    return path if os.path.exists(path) else "nvcc"


def stale() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    return any(os.path.getmtime(p) > t for p in SOURCES + HEADERS)


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and not stale():
        return LIB
    cmd = [nvcc(), *NVCC_FLAGS, "-I", os.path.join(ROOT, "include"), "-o", LIB, *SOURCES]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    print(build(force=True, verbose=True))
