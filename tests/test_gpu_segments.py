"""Time-segmented scans (a single long sequence cut into segments that run in
parallel): parity with the CPU oracle at forced segment counts.

The launcher cuts L into segments when a problem has too few (batch,
channel-block) CTAs to fill the GPU; the environment variable
MAMBA_SS_SEGMENTS forces the count. Each case runs the same inputs unsegmented
(1) and with 3 and 7 segments, through the forward, the end-state and adjoint
passes, the combines and the backward, and checks every output against the
oracle with the tolerances of the other parity tests.
"""
import numpy as np
import pytest
import torch

from _helpers import assert_bf16_close, BF16_TOL, BWD_TOL, FWD_TOL, assert_close, bf16_round, oracle_fused, \
    rel_err, run_fused
from oracle import selective_scan_oracle as orc

pytestmark = pytest.mark.gpu

GRAD_KEYS = ("du", "ddelta", "dA", "dB", "dC", "dD", "dz", "ddelta_bias", "dinitial_state")


def _with_dlast(x, seed=5):
    b, d, _ = x["u"].shape
    n = x["A"].shape[1]
    x["dlast"] = np.random.default_rng(seed).standard_normal((b, d, n)).astype(np.float32)
    return x


@pytest.fixture(params=[1, 3, 7], ids=lambda n: f"seg{n}")
def segments(request, monkeypatch):
    monkeypatch.setenv("MAMBA_SS_SEGMENTS", str(request.param))
    return request.param


def _check_fp32(res, ref):
    assert_close(res["out"], ref["out"], FWD_TOL, "out")
    assert_close(res["last_state"], ref["last_state"], FWD_TOL, "last_state")
    for k in GRAD_KEYS:
        if ref.get(k) is not None and k in res:
            assert_close(res[k], ref[k], BWD_TOL, k)


def test_fp32_long_row(segments):
    x = _with_dlast(orc.make_inputs(1, 24, 1000, 16, seed=21, initial_state=True))
    _check_fp32(run_fused(x, with_dlast=True), oracle_fused(x, with_dlast=True))


def test_unaligned_length_n8(segments):
    # L * 4 bytes not a multiple of 16: plain-load staging; N = 8: 16 channels per CTA
    x = _with_dlast(orc.make_inputs(1, 20, 777, 8, seed=22, initial_state=True))
    _check_fp32(run_fused(x, with_dlast=True), oracle_fused(x, with_dlast=True))


def test_zoh(segments):
    x = _with_dlast(orc.make_inputs(1, 8, 700, 8, seed=23, initial_state=True))
    _check_fp32(run_fused(x, zoh=True, with_dlast=True),
                oracle_fused(x, zoh=True, with_dlast=True))


def test_bf16(segments):
    x = orc.make_inputs(1, 16, 1024, 16, seed=24)
    res = run_fused(x, io_dtype=torch.bfloat16)
    ref = oracle_fused(x, io_round=bf16_round)
    for k in ("out", "last_state", "du", "ddelta", "dA", "dB", "dC", "dD", "dz", "ddelta_bias"):
        assert_bf16_close(res[k], ref[k], k)


def test_padding(segments):
    """Right padding that ends inside, at, and before segment boundaries."""
    x = orc.make_inputs(3, 8, 900, 16, seed=25, valid_lengths=(1, 900))
    x["seq_lens"] = np.array([900, 333, 64], dtype=np.int32)
    res = run_fused(x)
    _check_fp32(res, oracle_fused(x))
    for b, n in enumerate(x["seq_lens"]):
        for k in ("out", "du", "ddelta", "dz", "dB", "dC"):
            assert np.all(res[k][b, :, n:] == 0.0), (k, b)


def test_no_device_error(segments):
    from mamba import _native

    x = orc.make_inputs(1, 8, 2048, 16, seed=26)
    run_fused(x)
    assert _native.load().mamba_ss_take_device_error() == 0
