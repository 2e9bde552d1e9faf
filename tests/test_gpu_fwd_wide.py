"""The four-warp forward (N = 16, 32 channels per CTA sharing one B/C
staging), which the launcher picks for grids of several waves: parity with
the CPU oracle on small problems, the variant forced by MAMBA_SS_FWD_WIDE=1
(and, for comparison, the one-warp forward forced by 0). Covers channel
counts that leave part of the last CTA idle, lengths that end inside a tile
or are not 16-byte multiples (plain staging), bf16, right padding, initial
states and forward-only calls."""
import numpy as np
import pytest
import torch

from _helpers import assert_bf16_close, BF16_TOL, BWD_TOL, FWD_TOL, assert_close, bf16_round, oracle_fused, \
    rel_err, run_fused
from oracle import selective_scan_oracle as orc

pytestmark = pytest.mark.gpu

GRAD_KEYS = ("du", "ddelta", "dA", "dB", "dC", "dD", "dz", "ddelta_bias", "dinitial_state")


@pytest.fixture(params=[1, 0], ids=["wide", "narrow"])
def wide(request, monkeypatch):
    monkeypatch.setenv("MAMBA_SS_FWD_WIDE", str(request.param))
    monkeypatch.setenv("MAMBA_SS_SEGMENTS", "1")
    return request.param


def _check(res, ref):
    assert_close(res["out"], ref["out"], FWD_TOL, "out")
    assert_close(res["last_state"], ref["last_state"], FWD_TOL, "last_state")
    for k in GRAD_KEYS:
        if ref.get(k) is not None and k in res:
            assert_close(res[k], ref[k], BWD_TOL, k)


@pytest.mark.parametrize("dim,length", [(64, 256), (40, 300), (100, 513), (33, 1)])
def test_fp32(wide, dim, length):
    x = orc.make_inputs(2, dim, length, 16, seed=dim + length, initial_state=True)
    _check(run_fused(x), oracle_fused(x))


def test_unaligned_length(wide):
    # L * 4 bytes not a multiple of 16: plain-load staging
    x = orc.make_inputs(2, 48, 301, 16, seed=7)
    _check(run_fused(x), oracle_fused(x))


def test_zoh_no_z(wide):
    x = orc.make_inputs(2, 32, 200, 16, seed=8, with_z=False)
    _check(run_fused(x, zoh=True), oracle_fused(x, zoh=True))


def test_bf16_padded(wide):
    x = orc.make_inputs(4, 96, 512, 16, seed=9, valid_lengths=(1, 512))
    res = run_fused(x, io_dtype=torch.bfloat16)
    ref = oracle_fused(x, io_round=bf16_round)
    for k in ("out", "last_state", "du", "ddelta", "dA", "dB", "dC", "dD", "dz", "ddelta_bias"):
        assert_bf16_close(res[k], ref[k], k)
    for b, n in enumerate(x["seq_lens"]):
        assert np.all(res["out"][b, :, n:] == 0.0)


def test_forward_only(wide):
    x = orc.make_inputs(2, 64, 384, 16, seed=10)
    ref = oracle_fused(x)
    with torch.no_grad():
        res = run_fused(x, grads=False)
    assert_close(res["out"], ref["out"], FWD_TOL, "out")
    assert_close(res["last_state"], ref["last_state"], FWD_TOL, "last_state")
