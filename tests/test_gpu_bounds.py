"""The debug bounds build (libmamba_ss_b200_bounds.so, -DMSS_BOUNDS_CHECK).

It stands in for compute-sanitizer, which cannot be run on every machine: its
kernels check every computed global index and TMA store coordinate against
the extent of its array and count a violation instead of making the access.
The GPU test runs small odd shapes (L in {1, 17, 31, 777, ...}, N in
{1, 2, 4, 8, 16}, channel counts that are not a multiple of a CTA's, right
padding, time segments, ZOH, bf16, the deterministic dB/dC mode) through that
library in a child process, and requires oracle parity and zero violations;
its self-test proves that a violation is recorded. The CPU tests check the
query entry points of both libraries without a GPU.
"""
import ctypes
import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
LIB_DIR = ROOT / "jax-mambas_b200" / "lib"
BOUNDS_LIB = LIB_DIR / "libmamba_ss_b200_bounds.so"
NORMAL_LIB = LIB_DIR / "libmamba_ss_b200.so"


def _lib(path):
    if not path.is_file():
        pytest.fail(f"{path.name} is not built (python jax-mambas_b200/build.py"
                    f"{' --bounds' if 'bounds' in path.name else ''})")
    lib = ctypes.CDLL(str(path))
    lib.mamba_ss_bounds_checked.restype = ctypes.c_int32
    lib.mamba_ss_take_bounds_violations.restype = ctypes.c_uint64
    lib.mamba_ss_take_bounds_violations.argtypes = [ctypes.POINTER(ctypes.c_int64)]
    return lib


def test_normal_library_has_no_checks():
    lib = _lib(NORMAL_LIB)
    assert lib.mamba_ss_bounds_checked() == 0
    first = (ctypes.c_int64 * 3)(7, 7, 7)
    assert lib.mamba_ss_take_bounds_violations(first) == 0  # no CUDA call in this build
    assert list(first) == [0, 0, 0]


def test_bounds_library_reports_itself():
    assert _lib(BOUNDS_LIB).mamba_ss_bounds_checked() == 1


@pytest.mark.gpu
def test_kernels_make_no_out_of_bounds_access():
    env = dict(os.environ, MAMBA_SS_B200_LIB=str(BOUNDS_LIB))
    r = subprocess.run([sys.executable, str(ROOT / "tests" / "_bounds_check.py")], env=env,
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]
    res = json.loads(r.stdout.strip().splitlines()[-1])
    assert res["checked"] == 1
    assert res["selftest"] == {"violations": 1, "first": [99, 1007, 1000]}
    bad = [c for c in res["cases"] if c["violations"] or c["mismatch"]]
    assert not bad, bad
    assert res["device_error"] == 0
