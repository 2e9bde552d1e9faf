"""Child process of tests/test_gpu_bounds.py: runs the scan kernels of the
debug bounds library (loaded through MAMBA_SS_B200_LIB) over small odd shapes,
checks every output against the CPU oracle, and prints one JSON line with the
per-case results and the index violations the kernels recorded.

The bounds library's kernels check each computed global index (and each TMA
store coordinate) against its array's extent and skip the access instead of
faulting, so a wrong index shows up here as a nonzero violation count."""
import ctypes
import json
import os
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
for p in (ROOT / "jax-mambas_b200", ROOT, ROOT / "tests"):
    sys.path.insert(0, str(p))

import numpy as np  # noqa: E402
import torch  # noqa: E402

from _helpers import (BWD_TOL, FWD_TOL, assert_bf16_close, assert_close, bf16_round,  # noqa: E402
                      oracle_fused, run_fused)
from mamba import _native  # noqa: E402
from mamba import selective_scan_cuda as ssc  # noqa: E402
from oracle import selective_scan_oracle as orc  # noqa: E402

GRAD_KEYS = ("du", "ddelta", "dA", "dB", "dC", "dD", "dz", "ddelta_bias", "dinitial_state")

# (name, batch, dim, length, dstate, io dtype, zoh, valid lengths, segments, deterministic)
CASES = [
    ("f32_n16_tma_h0", 2, 40, 1000, 16, "f32", False, None, 1, False),
    ("f32_n16_seg3", 1, 24, 1000, 16, "f32", False, None, 3, False),
    ("f32_n8_plain_seg3", 1, 20, 777, 8, "f32", False, None, 3, False),
    ("f32_n4_zoh_L31", 2, 13, 31, 4, "f32", True, None, 1, False),
    ("f32_n2_L17", 2, 33, 17, 2, "f32", False, None, 1, False),
    ("f32_n1_L1", 3, 7, 1, 1, "f32", False, None, 1, False),
    ("bf16_n16_padded", 3, 24, 1100, 16, "bf16", False, (300, 1100), 1, False),
    ("bf16_n16_padded_seg2", 2, 24, 1100, 16, "bf16", False, (300, 1100), 2, False),
    ("f32_n16_padded_det", 3, 40, 520, 16, "f32", False, (1, 520), 1, True),
]


def _run_case(lib, case):
    name, b, d, L, n, io, zoh, valid, seg, det = case
    os.environ["MAMBA_SS_SEGMENTS"] = str(seg)
    ssc.set_deterministic(det)
    x = orc.make_inputs(b, d, L, n, seed=17 + CASES.index(case), initial_state=True,
                        valid_lengths=valid)
    x["dlast"] = np.random.default_rng(3).standard_normal((b, d, n)).astype(np.float32)
    bf16 = io == "bf16"
    res = run_fused(x, io_dtype=torch.bfloat16 if bf16 else torch.float32, zoh=zoh,
                    with_dlast=True)
    ref = oracle_fused(x, zoh=zoh, with_dlast=True, io_round=bf16_round if bf16 else None)
    first = (ctypes.c_int64 * 3)()
    count = lib.mamba_ss_take_bounds_violations(first)
    err = None
    try:
        for k in ("out", "last_state") + GRAD_KEYS:
            if ref.get(k) is None or k not in res:
                continue
            if bf16 and k in ("out", "du", "ddelta", "dB", "dC", "dz"):
                assert_bf16_close(res[k], ref[k], k)
            else:
                assert_close(res[k], ref[k], FWD_TOL if k in ("out", "last_state") else BWD_TOL, k)
    except AssertionError as e:
        err = str(e)[:400]
    ssc.set_deterministic(False)
    return {"case": name, "violations": int(count), "first": list(first), "mismatch": err}


def main():
    lib = _native.load()
    out = {"lib": os.environ.get("MAMBA_SS_B200_LIB"), "checked": lib.mamba_ss_bounds_checked()}
    # the checker itself: one recorded violation of site 99, no memory touched
    assert lib.mamba_ss_bounds_selftest() == 0, lib.mamba_ss_last_error()
    torch.cuda.synchronize()
    first = (ctypes.c_int64 * 3)()
    out["selftest"] = {"violations": int(lib.mamba_ss_take_bounds_violations(first)),
                       "first": list(first)}
    out["cases"] = [_run_case(lib, c) for c in CASES]
    out["device_error"] = int(lib.mamba_ss_take_device_error())
    print(json.dumps(out))


if __name__ == "__main__":
    main()
