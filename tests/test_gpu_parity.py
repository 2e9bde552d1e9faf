"""GPU parity of the sm_100a kernels against the CPU oracle (float64).

Tolerances: fp32 forward 1e-5 (rtol and atol), fp32 backward 1e-4, bf16 I/O
with fp32 state 2e-2 relative to the largest magnitude; padding positions
exactly zero. Cases restate the reference's tests
(tests/test_selective_scan_cuda.py:55-113: lengths {1,17,128,513} forward,
{1,31,513,2051} VJP, both discretizations) and widen them to every N, ragged
D, chunk boundaries, bf16, the fused features and padding.
"""
import numpy as np
import pytest
import torch

from _helpers import (assert_bf16_close, BF16_TOL, BWD_TOL, FWD_TOL, assert_close, bf16_round,
                      oracle_fused, rel_err, run_fused, to_dev)
from oracle import selective_scan_oracle as orc

pytestmark = pytest.mark.gpu

GRAD_KEYS = ("du", "ddelta", "dA", "dB", "dC", "dD", "dz", "ddelta_bias", "dinitial_state")


def _check(res, ref, fwd_tol=FWD_TOL, bwd_tol=BWD_TOL, keys=GRAD_KEYS):
    assert_close(res["out"], ref["out"], fwd_tol, "out")
    assert_close(res["last_state"], ref["last_state"], fwd_tol, "last_state")
    for k in keys:
        if ref.get(k) is not None and k in res:
            assert_close(res[k], ref[k], bwd_tol, k)


def test_config0_fused_fp32():
    """B=2, D=128, L=256, N=16 with softplus(delta+bias), D, z."""
    x = orc.make_inputs(2, 128, 256, 16, seed=0)
    _check(run_fused(x), oracle_fused(x))


@pytest.mark.parametrize("length", [1, 17, 128, 255, 256, 257, 511, 512, 513, 1025, 2051])
@pytest.mark.parametrize("dstate", [1, 2, 4, 8, 16])
def test_lengths_and_states(length, dstate):
    # dim=6 leaves two idle warps in the last CTA
    x = orc.make_inputs(2, 6, length, dstate, seed=length * 31 + dstate, initial_state=True)
    x["dlast"] = np.random.default_rng(5).standard_normal((2, 6, dstate)).astype(np.float32)
    _check(run_fused(x, with_dlast=True), oracle_fused(x, with_dlast=True))


@pytest.mark.parametrize("length", [1, 31, 300, 513])
def test_zoh(length):
    x = orc.make_inputs(1, 5, length, 8, seed=length, initial_state=True)
    _check(run_fused(x, zoh=True), oracle_fused(x, zoh=True))


@pytest.mark.parametrize("features", ["plain", "bias_only", "softplus_only", "D_only", "z_only"])
def test_feature_subsets(features):
    x = orc.make_inputs(2, 8, 333, 16, seed=11,
                        with_D=features == "D_only", with_z=features == "z_only",
                        with_bias=features == "bias_only",
                        delta_softplus=features == "softplus_only")
    if features in ("plain", "bias_only", "D_only", "z_only"):
        # raw delta must stay positive-ish when no softplus is applied
        x["delta"] = np.log1p(np.exp(x["delta"])).astype(np.float32)
    if features == "bias_only":
        x["delta_bias"] = (np.abs(x["delta_bias"]) / 8.0).astype(np.float32)  # keep delta > 0
    _check(run_fused(x), oracle_fused(x))


@pytest.mark.parametrize("aligned", [True, False])
def test_bf16_io(aligned):
    L = 512 if aligned else 509
    x = orc.make_inputs(2, 16, L, 16, seed=3)
    res = run_fused(x, io_dtype=torch.bfloat16)
    ref = oracle_fused(x, io_round=bf16_round)
    assert_bf16_close(res["out"], ref["out"])
    assert_bf16_close(res["last_state"], ref["last_state"])
    for k in ("du", "ddelta", "dA", "dB", "dC", "dD", "dz", "ddelta_bias"):
        assert_bf16_close(res[k], ref[k], k)


def test_padding_exact_zeros_and_state(monkeypatch):
    """configs[2]-style right padding through seq_lens: outputs and input
    gradients at pad positions are exact zeros; the last state equals the
    state at each sequence's valid length (bitwise, so both runs use one time
    segment: segment boundaries change the order of the float operations)."""
    monkeypatch.setenv("MAMBA_SS_SEGMENTS", "1")
    x = orc.make_inputs(4, 8, 700, 16, seed=9, valid_lengths=(1, 700))
    x["seq_lens"] = np.array([700, 1, 256, 517], dtype=np.int32)
    res = run_fused(x)
    ref = oracle_fused(x)
    _check(res, ref)
    for b, n in enumerate(x["seq_lens"]):
        for k in ("out", "du", "ddelta", "dz"):
            assert np.all(res[k][b, :, n:] == 0.0), (k, b)
        for k in ("dB", "dC"):
            assert np.all(res[k][b, :, n:] == 0.0), (k, b)
    # last state == the state of an unpadded run of the valid prefix
    for b, n in enumerate(x["seq_lens"]):
        xs = {k: (v[b:b + 1, ..., :n] if k in ("u", "delta", "z", "B", "C", "dout") else v)
              for k, v in x.items()}
        xs["seq_lens"] = None
        xs["initial_state"] = None
        r1 = run_fused(xs, grads=False)
        np.testing.assert_array_equal(r1["last_state"][0], res["last_state"][b])


def test_left_padding_reference_semantics():
    """The reference masks delta and u (mamba/mamba1.py:167-168); with left
    padding and a zero initial state the outputs at pad positions are 0."""
    x = orc.make_inputs(2, 8, 300, 16, seed=4, with_z=False, with_D=False,
                        with_bias=False, delta_softplus=False)
    x["delta"] = np.log1p(np.exp(x["delta"])).astype(np.float32)
    x["delta"][:, :, :40] = 0.0
    x["u"][:, :, :40] = 0.0
    res = run_fused(x)
    assert np.all(res["out"][:, :, :40] == 0.0)
    _check(res, oracle_fused(x))


def test_determinism():
    x = orc.make_inputs(2, 64, 1000, 16, seed=21, initial_state=True)
    r1 = run_fused(x)
    r2 = run_fused(x)
    for k in ("out", "last_state", "du", "ddelta", "dz", "dA", "dD", "ddelta_bias",
              "dinitial_state"):
        np.testing.assert_array_equal(r1[k], r2[k], err_msg=k)
    for k in ("dB", "dC"):  # channel sums use float atomics across CTAs
        assert_close(r1[k], r2[k], 1e-5, k)
    from mamba import _native

    assert _native.load().mamba_ss_take_device_error() == 0


def test_poisoned_outputs_are_overwritten():
    """Every output element is written: NaN-filled buffers come back finite."""
    from mamba import selective_scan_cuda as ssc

    x = orc.make_inputs(2, 10, 777, 16, seed=8, initial_state=True)
    dev = "cuda"
    t = {k: to_dev(v, dev) if isinstance(v, np.ndarray) else v for k, v in x.items()}
    b, d, L = x["u"].shape
    out = torch.full_like(t["u"], float("nan"))
    last = torch.full((b, d, 16), float("nan"), device=dev)
    cs = torch.full((ssc.chunk_states_elems(b, L, d, 16),), float("nan"), device=dev)
    pre = torch.full_like(t["u"], float("nan"))
    ssc.fused_forward_into(t["u"], t["delta"], t["A"], t["B"], t["C"], t["D"], t["z"],
                           t["delta_bias"], True, t["initial_state"], None, out, last, cs,
                           out_pre=pre)
    grads = [torch.full_like(t[k], float("nan")) for k in
             ("u", "delta", "A", "B", "C", "D", "z", "delta_bias", "initial_state")]
    ws = ssc._alloc_workspace(b, L, d, 16, 0, dev)
    ws.fill_(255)
    du, dd, dA, dB, dC, dD, dz, dbias, dh0 = grads
    ssc.fused_backward_into(t["u"], t["delta"], t["A"], t["B"], t["C"], t["D"], t["z"],
                            t["delta_bias"], True, t["initial_state"], None, cs, t["dout"],
                            None, du, dd, dA, dB, dC, dD, dz, dbias, dh0, ws, out_pre=pre)
    torch.cuda.synchronize()
    for v in [out, last, cs, pre] + grads:
        assert torch.isfinite(v).all()


# --------------------------------------------------------------------------
# Reference contract: selective_scan(A, deltas, Bs, Cs, u, initial_x, ...)
# --------------------------------------------------------------------------
def _ref_inputs(batch=2, length=17, dim=8, n=16, seed=7):
    """The fixture recipe of tests/test_selective_scan_cuda.py:11-19 (NumPy
    seeds instead of the JAX PRNG)."""
    rng = np.random.default_rng(seed)
    A = -np.exp(rng.standard_normal((dim, n)))
    deltas = np.logaddexp(rng.standard_normal((batch, length, dim)), 0.0)
    Bs = rng.standard_normal((batch, length, n))
    Cs = rng.standard_normal((batch, length, n))
    u = rng.standard_normal((batch, length, dim))
    x0 = rng.standard_normal((batch, dim, n))
    return [a.astype(np.float32) for a in (A, deltas, Bs, Cs, u, x0)]


@pytest.mark.parametrize("length", [1, 17, 128, 513])
@pytest.mark.parametrize("use_euler", [True, False])
def test_reference_contract_forward(length, use_euler):
    from mamba.selective_scan_cuda import selective_scan

    args = _ref_inputs(length=length)
    ey, ef = orc.selective_scan_reference(*args, use_euler_barB_approx=use_euler)
    y, f = selective_scan(*[to_dev(a) for a in args], use_euler_barB_approx=use_euler,
                          use_cuda=True)
    assert_close(y.cpu().numpy(), ey, FWD_TOL, "y")
    assert_close(f.cpu().numpy(), ef, FWD_TOL, "final_x")


@pytest.mark.parametrize("length", [1, 31, 513, 2051])
@pytest.mark.parametrize("use_euler", [True, False])
def test_reference_contract_vjp(length, use_euler):
    """Loss mean(y^2) + mean(final_x^2), grads of all six inputs
    (tests/test_selective_scan_cuda.py:75-113)."""
    from mamba.selective_scan_cuda import selective_scan

    args = _ref_inputs(batch=1, length=length, dim=4, n=8)
    # float64 autograd of the oracle restatement
    targs = [torch.from_numpy(a).double().requires_grad_(True) for a in args]
    y, f = _torch_reference(*targs, use_euler)
    (torch.mean(y ** 2) + torch.mean(f ** 2)).backward()
    expected = [t.grad.numpy() for t in targs]
    dargs = [to_dev(a).requires_grad_(True) for a in args]
    y, f = selective_scan(*dargs, use_euler_barB_approx=use_euler, use_cuda=True)
    (torch.mean(y ** 2) + torch.mean(f ** 2)).backward()
    for name, a, e in zip(("A", "deltas", "Bs", "Cs", "u", "initial_x"), dargs, expected):
        assert_close(a.grad.cpu().numpy(), e, BWD_TOL, name)


def _torch_reference(A, deltas, Bs, Cs, u, x0, use_euler):
    """Sequential float64 torch restatement used only as the autograd oracle."""
    delta_a = torch.einsum("bld,dn->bldn", deltas, A)
    a_bars = torch.exp(delta_a)
    if use_euler:
        b_bars = torch.einsum("bld,bln->bldn", deltas, Bs)
    else:
        b_bars = torch.expm1(delta_a) * torch.einsum("dn,bln->bldn", torch.reciprocal(A), Bs)
    state = x0
    ys = []
    for t in range(u.shape[1]):
        state = a_bars[:, t] * state + b_bars[:, t] * u[:, t, :, None]
        ys.append(torch.einsum("bn,bdn->bd", Cs[:, t], state))
    return torch.stack(ys, 1), state


def test_invalid_arguments_raise_without_launch():
    from mamba import selective_scan_cuda as ssc

    u = torch.zeros(1, 4, 8, device="cuda")
    with pytest.raises(ValueError, match="N must be one of"):
        ssc.fused_forward_into(u, u, torch.zeros(4, 3, device="cuda"),
                               torch.zeros(1, 3, 8, device="cuda"),
                               torch.zeros(1, 3, 8, device="cuda"), None, None, None,
                               False, None, None, u, None, torch.zeros(64, device="cuda"))


def test_forward_only_skips_the_saved_state():
    """Under torch.no_grad the forward writes no carries and no pre-gate
    output (chunk_states = NULL); the outputs equal the oracle's and those of
    a grad-enabled run on the same inputs."""
    from mamba.selective_scan_cuda import selective_scan_fn

    x = orc.make_inputs(2, 16, 700, 16, seed=31, initial_state=True)
    ref = oracle_fused(x)
    with torch.no_grad():
        res = run_fused(x, grads=False)
    _check(res, ref, keys=())
    t = {k: to_dev(x[k]) for k in ("u", "delta", "A", "B", "C", "D", "z", "delta_bias",
                                   "initial_state")}
    t["u"].requires_grad_(True)
    out, last = selective_scan_fn(t["u"], t["delta"], t["A"], t["B"], t["C"], t["D"], t["z"],
                                  t["delta_bias"], True, True, initial_state=t["initial_state"])
    assert_close(res["out"], out.detach().cpu().numpy(), FWD_TOL, "out")
    assert_close(res["last_state"], last.detach().cpu().numpy(), FWD_TOL, "last_state")
