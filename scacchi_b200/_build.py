"""Build the CUDA library in-tree (sm_100a only)."""

from __future__ import annotations

import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libscacchi_b200.so")
# (source, extra flags).  The search kernels are bit-reproducible against
# the oracle: no implicit multiply-add contraction (they call fmaf()
# explicitly where they want one).  The network kernels are checked to a
# tolerance and keep contraction.
UNITS = [(os.path.join(CSRC, "search.cu"), ["-fmad=false"]), (os.path.join(CSRC, "tower.cu"), []),
         (os.path.join(CSRC, "hex.cu"), ["-fmad=false"]), (os.path.join(CSRC, "targets.cu"), ["-fmad=false"])]
SOURCES = [u[0] for u in UNITS]
HEADERS = [os.path.join(CSRC, h) for h in ("smath.h", "threefry.h", "synthetic_env.h", "lane_cta.cuh")] + [
    os.path.join(ROOT, "include", "scacchi_b200.h")]

NVCC_FLAGS = ["-O3", "-std=c++17", "-Xcompiler", "-fPIC", "-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo"]


def nvcc() -> str:
    cuda = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    path = os.path.join(cuda, "bin", "nvcc")
    return path if os.path.exists(path) else "nvcc"


def stale() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    return any(os.path.getmtime(p) > t for p in SOURCES + HEADERS)


def build(force: bool = False, verbose: bool = False, out: str | None = None, defines: tuple = ()) -> str:
    out = out or LIB
    if out == LIB and not force and not stale():
        return LIB
    objs = []
    build_dir = os.path.join(HERE, "_build")
    os.makedirs(build_dir, exist_ok=True)
    procs = []
    for src, extra in UNITS:
        obj = os.path.join(build_dir, os.path.basename(src) + ".o")
        cmd = [nvcc(), *NVCC_FLAGS, *extra, *defines, "-I", os.path.join(ROOT, "include"), "-c", src, "-o", obj]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
        procs.append(subprocess.Popen(cmd))
        objs.append(obj)
    for p in procs:
        if p.wait() != 0:
            raise RuntimeError("nvcc failed")
    subprocess.run([nvcc(), "-shared", "-gencode", "arch=compute_100a,code=sm_100a", "-o", out, *objs], check=True)
    return out


if __name__ == "__main__":
    print(build(force=True, verbose=True))
