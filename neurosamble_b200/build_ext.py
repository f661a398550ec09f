"""Build librbq.so (the C-ABI CUDA library) in-tree for sm_100a.

Usage: ``python -m neurosamble_b200.build_ext`` (or ``build()`` from Python).  The shared
library lands in ``neurosamble_b200/_lib/librbq.so`` so it travels with the source tree.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OUT_DIR = os.path.join(HERE, "_lib")
LIB = os.path.join(OUT_DIR, "librbq.so")

SOURCES = ["rbq_host_math.cpp", "rbq_build.cu", "rbq_search.cu", "rbq_coarse_tc.cu", "rbq_capi.cu"]
HEADERS = ["rbq_internal.cuh", os.path.join("..", "..", "include", "rbq.h")]

# -fmad=false: no FMA contraction anywhere, so every expression is evaluated as written and
# the results match the CPU oracle bit for bit.  IEEE division / sqrt stay on (no fast math).
NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17", "-fmad=false",
    "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC,-ffp-contract=off,-O3",
    "-Xptxas", "-warn-spills",
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _cxx() -> str:
    for cand in ("/usr/bin/g++", shutil.which("g++")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("g++ not found")


def _stale() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    for f in SOURCES + HEADERS:
        if os.path.getmtime(os.path.join(CSRC, f)) > t:
            return True
    return False


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and not _stale():
        return LIB
    os.makedirs(OUT_DIR, exist_ok=True)
    objs = []
    nvcc = _nvcc()
    env = dict(os.environ)
    env.pop("CXX", None)
    env.pop("CC", None)
    for src in SOURCES:
        obj = os.path.join(OUT_DIR, os.path.splitext(src)[0] + ".o")
        extra = os.environ.get("RBQ_NVCC_EXTRA", "").split()
        cmd = [nvcc, *NVCC_FLAGS, *extra, "-c", os.path.join(CSRC, src), "-o", obj]
        if src.endswith(".cpp"):
            cmd = [_cxx(), "-std=c++17", "-O3", "-fPIC", "-ffp-contract=off", "-fno-fast-math",
                   "-I/usr/local/cuda/include", "-c", os.path.join(CSRC, src), "-o", obj]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True, env=env)
        objs.append(obj)
    tmp = LIB + ".tmp"
    # Static CUDA runtime: the library does not bind to whichever libcudart the host process
    # (e.g. PyTorch) loaded first; device pointers and streams are shared through the driver.
    cmd = [nvcc, "-shared", "-cudart=static", "-gencode", "arch=compute_100a,code=sm_100a", "-o", tmp, *objs]
    subprocess.run(cmd, check=True, env=env)
    os.replace(tmp, LIB)
    for o in objs:
        os.remove(o)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
