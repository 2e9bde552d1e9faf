"""Writes tests/golden/fused_small.npz from the CPU oracle (float64).

The fixture pins the oracle's fused forward/backward on one seeded case
(batch 2, dim 16, length 300, dstate 16, every fused feature, nonzero
initial state) so GPU tests and later oracle edits can be checked against
stored numbers without re-deriving them. Run from the repository root:
    python tests/golden/make_golden.py
"""
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tests"))

from oracle import selective_scan_oracle as orc  # noqa: E402
from test_oracle import orc_checksum  # noqa: E402

SPEC = dict(batch=2, dim=16, length=300, dstate=16, seed=1234)


def main():
    x = orc.make_inputs(SPEC["batch"], SPEC["dim"], SPEC["length"], SPEC["dstate"],
                        seed=SPEC["seed"], initial_state=True)
    ref = orc.fused_backward(x["u"], x["delta"], x["A"], x["B"], x["C"], x["D"], x["z"],
                             x["delta_bias"], True, x["initial_state"], True, None,
                             dout=x["dout"])
    out = {f"spec_{k}": np.int64(v) for k, v in SPEC.items()}
    out["input_checksum"] = orc_checksum(x)
    for k in ("out", "last_state", "du", "ddelta", "dA", "dB", "dC", "dD", "dz",
              "ddelta_bias", "dinitial_state"):
        out[k] = ref[k]
    np.savez_compressed(Path(__file__).with_name("fused_small.npz"), **out)


if __name__ == "__main__":
    main()
