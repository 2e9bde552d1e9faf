"""Deterministic dB / dC: with mamba_ss_set_deterministic(1) every warp
writes its channel-block sums of dB and dC to a partial buffer and a second
kernel adds them in a fixed order, so two runs give bitwise-equal dB and dC
(all other outputs are bitwise reproducible in either mode). Each case also
matches the float64 oracle at the parity tolerances (fp32 backward 1e-4,
bf16 per element 2e-2 with its floor), through the N = 16 shuffle flush (one-
and two-warp CTAs), the N < 16 shared-memory flush, right padding, time
segments and the plain-load staging."""
import numpy as np
import pytest
import torch

from _helpers import (BWD_TOL, FWD_TOL, assert_bf16_close, assert_close, bf16_round,
                      oracle_fused, run_fused)
from oracle import selective_scan_oracle as orc

pytestmark = pytest.mark.gpu

ALL = ("out", "last_state", "du", "ddelta", "dA", "dB", "dC", "dD", "dz", "ddelta_bias")


@pytest.fixture
def det():
    from mamba import selective_scan_cuda as ssc

    ssc.set_deterministic(True)
    assert ssc.is_deterministic()
    yield
    ssc.set_deterministic(False)


def _twice(x, **kw):
    r1, r2 = run_fused(x, **kw), run_fused(x, **kw)
    for k in ALL:
        if k in r1:
            np.testing.assert_array_equal(r1[k], r2[k], err_msg=k)
    return r1


@pytest.mark.parametrize("dstate,L", [(16, 1000), (16, 1001), (8, 640), (4, 300)])
def test_fp32_bitwise_and_oracle(det, dstate, L):
    x = orc.make_inputs(2, 40, L, dstate, seed=L + dstate, initial_state=True)
    res = _twice(x)
    ref = oracle_fused(x)
    assert_close(res["out"], ref["out"], FWD_TOL, "out")
    for k in ("du", "ddelta", "dA", "dB", "dC", "dD", "dz", "ddelta_bias", "dinitial_state"):
        assert_close(res[k], ref[k], BWD_TOL, k)


@pytest.mark.parametrize("warps", [1, 2])
def test_bf16_padded_bitwise_and_oracle(det, warps, monkeypatch):
    monkeypatch.setenv("MAMBA_SS_BWD_WARPS", str(warps))
    x = orc.make_inputs(4, 48, 1024, 16, seed=7, valid_lengths=(1, 1024))
    x["seq_lens"] = np.array([1024, 1, 333, 700], dtype=np.int32)
    res = _twice(x, io_dtype=torch.bfloat16)
    ref = oracle_fused(x, io_round=bf16_round)
    for k in ("out", "du", "ddelta", "dA", "dB", "dC", "dD", "dz", "ddelta_bias"):
        assert_bf16_close(res[k], ref[k], k)
    for b, n in enumerate(x["seq_lens"]):
        for k in ("dB", "dC"):
            assert np.all(res[k][b, :, n:] == 0.0), (k, b)


def test_segments_bitwise_and_oracle(det, monkeypatch):
    monkeypatch.setenv("MAMBA_SS_SEGMENTS", "3")
    x = orc.make_inputs(1, 24, 1000, 16, seed=21, initial_state=True)
    res = _twice(x)
    ref = oracle_fused(x)
    for k in ("du", "ddelta", "dA", "dB", "dC", "dD", "dz", "ddelta_bias"):
        assert_close(res[k], ref[k], BWD_TOL, k)


def test_mode_changes_the_workspace_size():
    from mamba import selective_scan_cuda as ssc

    base = ssc.bwd_workspace_bytes(2, 1000, 40, 16)
    ssc.set_deterministic(True)
    try:
        more = ssc.bwd_workspace_bytes(2, 1000, 40, 16)
    finally:
        ssc.set_deterministic(False)
    assert more >= base + 2 * 5 * 2 * 16 * 1000 * 4  # batch * cols * (dB, dC) * N * L * fp32
