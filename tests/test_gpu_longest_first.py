"""Right-padded batches run longest sequence first (the CTAs of grid row y
take the batch of rank y by valid length). Parity with the CPU oracle when
the ranking spans more than one warp's worth of batches (40), with tied and
zero lengths, and past the ranking's limit of 128 batches (grid order)."""
import numpy as np
import pytest
import torch

from _helpers import BWD_TOL, FWD_TOL, assert_close, oracle_fused, run_fused
from oracle import selective_scan_oracle as orc

pytestmark = pytest.mark.gpu

KEYS = ("du", "ddelta", "dA", "dB", "dC", "dD", "dz", "ddelta_bias")


@pytest.mark.parametrize("batch", [40, 130])
def test_many_batches_with_ties(batch, monkeypatch):
    monkeypatch.setenv("MAMBA_SS_SEGMENTS", "1")
    x = orc.make_inputs(batch, 8, 96, 16, seed=batch, valid_lengths=(1, 96))
    lens = np.asarray(x["seq_lens"]).copy()
    lens[::5] = 64   # ties
    lens[3] = 0      # an empty sequence
    lens[7] = 96
    x["seq_lens"] = lens.astype(lens.dtype)
    res = run_fused(x)
    ref = oracle_fused(x)
    assert_close(res["out"], ref["out"], FWD_TOL, "out")
    assert_close(res["last_state"], ref["last_state"], FWD_TOL, "last_state")
    for k in KEYS:
        assert_close(res[k], ref[k], BWD_TOL, k)
    for b, n in enumerate(lens):
        assert np.all(res["out"][b, :, n:] == 0.0)
