"""Build recipe for libnoor_moe.so (sm_100a), in-tree.

One nvcc invocation compiles the kernels and the C ABI into a shared library
next to this file; the CUDA runtime is linked statically, NCCL dynamically.
The debug build libnoor_moe_check.so is the same source compiled with
-DNOOR_CHECK: every data-dependent row index a kernel uses (permute
destinations, peer receive rows, row-map outputs, combine gathers, the
router's pick total) is checked against its buffer, and a bad one is
reported through the handle's error word (NOOR_MOE_ERR_INVALID) instead of
being accessed.  Set NOOR_MOE_CHECK=1 to load it.
"""
from __future__ import annotations

import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libnoor_moe.so")
LIB_CHECK = os.path.join(HERE, "libnoor_moe_check.so")
SOURCES = ["noor_moe.cu"]


def headers() -> list:
    """Every header beside the sources: an edit to any of them rebuilds."""
    return sorted(os.path.basename(p) for p in glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")))

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC,-O3,-fvisibility=hidden",
    "-shared", "-cudart", "static",
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if cand and (os.path.isabs(cand) and os.path.exists(cand) or not os.path.isabs(cand)):
            return cand
    return "nvcc"


def stale(lib: str = LIB) -> bool:
    if not os.path.exists(lib):
        return True
    t = os.path.getmtime(lib)
    deps = [os.path.join(CSRC, f) for f in SOURCES + headers()]
    deps.append(os.path.join(ROOT, "include", "noor_moe.h"))
    return any(os.path.getmtime(p) > t for p in deps if os.path.exists(p))


def build(force: bool = False, verbose: bool = False, extra=(), check: bool = False) -> str:
    """Compile the library (check=True: the bounds-checked debug build)."""
    lib = LIB_CHECK if check else LIB
    if not force and not stale(lib):
        return lib
    defs = ["-DNOOR_CHECK"] if check else []
    cmd = [nvcc(), *NVCC_FLAGS, *defs, *extra, "-I", os.path.join(ROOT, "include"), "-I", CSRC,
           "-o", lib + ".tmp", *[os.path.join(CSRC, f) for f in SOURCES], "-ldl"]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    os.replace(lib + ".tmp", lib)
    return lib


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True,
          extra=["-Xptxas", "-v"] if "--ptxas-v" in sys.argv else [], check="--check" in sys.argv)
