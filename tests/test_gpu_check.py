"""GPU: the bounds-checked debug build (libnoor_moe_check.so, -DNOOR_CHECK)
runs small odd-shape layers -- ragged token counts, k = E, E = 128 with
k = 8, d not a multiple of 256 (one-CTA GEMMs), no dense branch, F32 and
BF16 -- with every row-index check passing and outputs matching the oracle.
It stands in for a memory checker on this GPU pool.  The cases run in a
child process that loads the debug library (tests/check_build_cases.py)."""
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_check_build_odd_shapes():
    env = dict(os.environ, NOOR_MOE_CHECK="1")
    r = subprocess.run([sys.executable, os.path.join(ROOT, "tests", "check_build_cases.py")], env=env, cwd=ROOT,
                       capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert '"ok": true' in r.stdout, r.stdout[-3000:]
