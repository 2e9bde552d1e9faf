"""The N = 16 backward in both CTA shapes against the CPU oracle.

The launcher runs the N = 16 backward with two-warp CTAs (16 channels, one
shared B/C staging, one CTA barrier per tile); MAMBA_SS_BWD_WARPS=1 forces the
one-warp CTAs. Each case runs under both, through the TMA path (aligned
rows) and the plain-load path (L * esize not a multiple of 16), with a
channel count that leaves the last CTA partly empty, fp32 and bf16 I/O,
longest-first right padding, and time segments. Tolerances as the other
parity tests."""
import numpy as np
import pytest
import torch

from _helpers import (BWD_TOL, FWD_TOL, assert_bf16_close, assert_close, bf16_round,
                      oracle_fused, run_fused)
from oracle import selective_scan_oracle as orc

pytestmark = pytest.mark.gpu

GRAD_KEYS = ("du", "ddelta", "dA", "dB", "dC", "dD", "dz", "ddelta_bias", "dinitial_state")


@pytest.fixture(params=[1, 2], ids=lambda n: f"warps{n}")
def warps(request, monkeypatch):
    monkeypatch.setenv("MAMBA_SS_BWD_WARPS", str(request.param))
    return request.param


def _check(res, ref):
    assert_close(res["out"], ref["out"], FWD_TOL, "out")
    for k in GRAD_KEYS:
        if ref.get(k) is not None and k in res:
            assert_close(res[k], ref[k], BWD_TOL, k)


@pytest.mark.parametrize("L", [512, 777], ids=["tma", "plain"])
@pytest.mark.parametrize("dim", [16, 40])
def test_fp32(warps, L, dim):
    x = orc.make_inputs(2, dim, L, 16, seed=L + dim, initial_state=True)
    x["dlast"] = np.random.default_rng(3).standard_normal((2, dim, 16)).astype(np.float32)
    _check(run_fused(x, with_dlast=True), oracle_fused(x, with_dlast=True))


@pytest.mark.parametrize("L", [1024, 1020], ids=["tma", "plain"])
def test_bf16_padded(warps, L):
    x = orc.make_inputs(4, 40, L, 16, seed=L, valid_lengths=(1, L))
    x["seq_lens"] = np.array([L, 1, 333, 700], dtype=np.int32)
    res = run_fused(x, io_dtype=torch.bfloat16)
    ref = oracle_fused(x, io_round=bf16_round)
    for k in ("out", "du", "ddelta", "dA", "dB", "dC", "dD", "dz", "ddelta_bias"):
        assert_bf16_close(res[k], ref[k], k)
    for b, n in enumerate(x["seq_lens"]):
        for k in ("out", "du", "ddelta", "dz", "dB", "dC"):
            assert np.all(res[k][b, :, n:] == 0.0), (k, b)


@pytest.mark.parametrize("segments", [1, 3])
def test_fp32_padded_segments(warps, segments, monkeypatch):
    monkeypatch.setenv("MAMBA_SS_SEGMENTS", str(segments))
    x = orc.make_inputs(3, 24, 900, 16, seed=25, valid_lengths=(1, 900))
    x["seq_lens"] = np.array([900, 333, 64], dtype=np.int32)
    res = run_fused(x)
    _check(res, oracle_fused(x))
    for b, n in enumerate(x["seq_lens"]):
        for k in ("out", "du", "ddelta", "dz", "dB", "dC"):
            assert np.all(res[k][b, :, n:] == 0.0), (k, b)


def test_zoh(warps):
    x = orc.make_inputs(2, 24, 640, 16, seed=5, initial_state=True)
    _check(run_fused(x, zoh=True), oracle_fused(x, zoh=True))


def test_no_device_error(warps):
    from mamba import _native

    x = orc.make_inputs(2, 32, 2048, 16, seed=26)
    run_fused(x)
    torch.cuda.synchronize()
    assert _native.load().mamba_ss_take_device_error() == 0
