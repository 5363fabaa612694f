"""CPU: the C-ABI library loads and exports exactly what include/noor_moe.h
declares; host-only entry points behave; the product never reaches the oracle."""
import ctypes
import os
import re
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "noor_moe.h")
PKG_DIR = os.path.join(ROOT, "noor_-_bangla_ai_b200")


def header_functions():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"NOOR_MOE_API\s+[\w\s\*]+?\b(noor_\w+)\s*\(", src)))


def test_header_declares_entry_points(pkg):
    names = header_functions()
    assert "noor_moe_forward" in names and "noor_matmul_f32" in names
    assert sorted(pkg.api.EXPORTED_SYMBOLS) == names


def test_library_exports_every_declared_symbol(pkg):
    lib = pkg.api.lib()
    for name in header_functions():
        assert hasattr(lib, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", pkg.api.LIB_PATH], capture_output=True, text=True).stdout
    exported = set(re.findall(r"\bT (noor_\w+)", out))
    assert exported == set(header_functions())


def test_check_build_exports_the_same_symbols(pkg):
    """The bounds-checked debug build (build.py --check) is a drop-in for the
    product library: same exported entry points."""
    path = os.path.join(PKG_DIR, "libnoor_moe_check.so")
    assert os.path.exists(path), "build the debug library: python noor_-_bangla_ai_b200/build.py --check"
    ctypes.CDLL(path)
    out = subprocess.run(["nm", "-D", "--defined-only", path], capture_output=True, text=True).stdout
    assert set(re.findall(r"\bT (noor_\w+)", out)) == set(header_functions())


def test_library_does_not_link_nccl_or_cuda_driver(pkg):
    out = subprocess.run(["ldd", pkg.api.LIB_PATH], capture_output=True, text=True).stdout
    assert "libnccl" not in out and "libcuda.so" not in out


def test_last_error_and_bad_args_on_cpu(pkg):
    lib = pkg.api.lib()
    assert isinstance(lib.noor_moe_last_error(), bytes)
    out = ctypes.c_void_p()
    rc = lib.noor_moe_create(None, None, ctypes.byref(out))
    assert rc == 1 and b"null descriptor" in lib.noor_moe_last_error()
    assert lib.noor_moe_forward(None, None, None, 0, None, None, None, None) == 1


def test_ep_plan_host_arithmetic(pkg):
    lib = pkg.api.lib()
    E, G = 8, 2
    counts_local = np.array([3, 0, 5, 1, 2, 2, 0, 7], np.int64)          # this rank's picks per expert
    counts_recv = np.array([4, 1, 0, 6, 2, 2, 9, 0], np.int64)           # [src][local expert]
    sr, so, rr, ro = (np.zeros(G, np.int64) for _ in range(4))
    row, mt, wi = (np.zeros(G * (E // G) + 1, np.int32) for _ in range(3))
    P = lambda a: a.ctypes.data_as(ctypes.c_void_p)
    lib.noor_moe_ep_plan.argtypes = [ctypes.c_void_p] * 2 + [ctypes.c_int] * 3 + [ctypes.c_void_p] * 7
    rc = lib.noor_moe_ep_plan(P(counts_local), P(counts_recv), E, G, 128, P(sr), P(so), P(rr), P(ro), P(row),
                              P(mt), P(wi))
    assert rc == 0
    assert sr.tolist() == [9, 11] and so.tolist() == [0, 9]
    assert rr.tolist() == [11, 13] and ro.tolist() == [0, 11]
    assert row.tolist() == [0, 4, 5, 5, 11, 13, 15, 24, 24]
    assert mt.tolist() == [0, 1, 2, 2, 3, 4, 5, 6, 6]
    assert wi[:-1].tolist() == [0, 1, 2, 3, 0, 1, 2, 3]
    bad = counts_recv.copy()
    bad[0] = -1
    assert lib.noor_moe_ep_plan(P(counts_local), P(bad), E, G, 128, P(sr), P(so), P(rr), P(ro), P(row), P(mt),
                                P(wi)) == 1


def test_product_never_imports_the_oracle():
    for dirpath, _, files in os.walk(PKG_DIR):
        for f in files:
            if f.endswith((".py", ".cu", ".cuh", ".h")):
                src = open(os.path.join(dirpath, f)).read()
                assert "import oracle" not in src and "from oracle" not in src, f
                assert "noor_oracle" not in src, f
