"""CPU checks that pin the oracle before the GPU tests trust it.

* the reference's known-answer test: associative scan == sequential
  recurrence (tests/test_selective_scan_cuda.py:22-52), both discretizations;
* the fused forward in kernel layout == the reference formulation after the
  caller-side math of S6.__call__ (mamba/mamba1.py:162-198);
* the analytic backward == torch.autograd in float64;
* the committed golden fixtures still match.
"""
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import selective_scan_oracle as orc

GOLDEN = Path(__file__).resolve().parent / "golden"


def _kat_inputs(batch=2, length=17, dim=8, n=16, seed=7):
    rng = np.random.default_rng(seed)
    A = -np.exp(rng.standard_normal((dim, n)))
    deltas = np.logaddexp(rng.standard_normal((batch, length, dim)), 0.0)
    Bs = rng.standard_normal((batch, length, n))
    Cs = rng.standard_normal((batch, length, n))
    u = rng.standard_normal((batch, length, dim))
    x0 = rng.standard_normal((batch, dim, n))
    return A, deltas, Bs, Cs, u, x0


@pytest.mark.parametrize("use_euler", [True, False])
def test_reference_matches_sequential_recurrence(use_euler):
    args = _kat_inputs()
    y, f = orc.selective_scan_reference(*args, use_euler_barB_approx=use_euler)
    ys, fs = orc.sequential_recurrence(*args, use_euler_barB_approx=use_euler)
    np.testing.assert_allclose(y, ys, rtol=2e-5, atol=2e-5)
    np.testing.assert_allclose(f, fs, rtol=2e-5, atol=2e-5)
    # float32 evaluation stays within the reference test's tolerance too
    y32, f32 = orc.selective_scan_reference(*args, use_euler_barB_approx=use_euler,
                                            dtype=np.float32)
    np.testing.assert_allclose(y32, ys, rtol=2e-5, atol=2e-5)


@pytest.mark.parametrize("use_euler", [True, False])
def test_fused_forward_matches_reference_formulation(use_euler):
    x = orc.make_inputs(2, 8, 40, 16, seed=3, initial_state=True)
    out, last = orc.fused_forward(x["u"], x["delta"], x["A"], x["B"], x["C"], x["D"], x["z"],
                                  x["delta_bias"], True, x["initial_state"], use_euler)
    # caller-side math of S6.__call__/Mamba.__call__ around selective_scan
    dl = np.logaddexp(x["delta"].astype(np.float64) + x["delta_bias"][None, :, None], 0.0)
    y, f = orc.selective_scan_reference(
        x["A"], dl.transpose(0, 2, 1), x["B"].transpose(0, 2, 1), x["C"].transpose(0, 2, 1),
        x["u"].transpose(0, 2, 1), x["initial_state"], use_euler_barB_approx=use_euler)
    y = y.transpose(0, 2, 1) + x["D"].astype(np.float64)[None, :, None] * x["u"]
    z = x["z"].astype(np.float64)
    y = y * z / (1.0 + np.exp(-z))
    np.testing.assert_allclose(out, y, rtol=1e-10, atol=1e-10)
    np.testing.assert_allclose(last, f, rtol=1e-10, atol=1e-10)


def _torch_fused(u, delta, A, B, C, D, z, bias, h0, use_euler, mask):
    pre = delta + bias[None, :, None]
    dl = torch.nn.functional.softplus(pre) * mask
    um = u * mask
    h = h0
    ys = []
    for t in range(u.shape[2]):
        dA = dl[:, :, t, None] * A[None]
        a = torch.exp(dA)
        bb = dl[:, :, t, None] * B[:, None, :, t] if use_euler else \
            torch.expm1(dA) / A[None] * B[:, None, :, t]
        h = a * h + bb * um[:, :, t, None]
        ys.append(torch.einsum("bn,bdn->bd", C[:, :, t], h))
    y = torch.stack(ys, 2) + D[None, :, None] * um
    out = y * torch.nn.functional.silu(z) * mask
    return out, h


@pytest.mark.parametrize("use_euler", [True, False])
@pytest.mark.parametrize("padded", [False, True])
def test_analytic_backward_matches_autograd(use_euler, padded):
    x = orc.make_inputs(2, 5, 23, 4, seed=13, initial_state=True,
                        valid_lengths=(5, 23) if padded else None)
    dlast = np.random.default_rng(1).standard_normal((2, 5, 4))
    ref = orc.fused_backward(x["u"], x["delta"], x["A"], x["B"], x["C"], x["D"], x["z"],
                             x["delta_bias"], True, x["initial_state"], use_euler,
                             x["seq_lens"], dout=x["dout"], dlast_state=dlast)
    names = ["u", "delta", "A", "B", "C", "D", "z", "delta_bias", "initial_state"]
    t = {k: torch.from_numpy(np.asarray(x[k], dtype=np.float64)).requires_grad_(True)
         for k in names}
    L = x["u"].shape[2]
    if x["seq_lens"] is not None:
        mask = torch.from_numpy((np.arange(L)[None, :] < x["seq_lens"][:, None])
                                .astype(np.float64))[:, None, :]
    else:
        mask = torch.ones(1, 1, L, dtype=torch.float64)
    out, h = _torch_fused(*(t[k] for k in names), use_euler, mask)
    loss = (out * torch.from_numpy(x["dout"].astype(np.float64))).sum() + \
        (h * torch.from_numpy(dlast)).sum()
    loss.backward()
    keys = {"u": "du", "delta": "ddelta", "A": "dA", "B": "dB", "C": "dC", "D": "dD",
            "z": "dz", "delta_bias": "ddelta_bias", "initial_state": "dinitial_state"}
    np.testing.assert_allclose(ref["out"] * mask.numpy(), out.detach().numpy(), rtol=1e-10,
                               atol=1e-12)
    for k in names:
        np.testing.assert_allclose(ref[keys[k]], t[k].grad.numpy(), rtol=1e-9, atol=1e-11,
                                   err_msg=k)


def test_golden_fixtures():
    path = GOLDEN / "fused_small.npz"
    g = np.load(path)
    spec = {k[5:]: g[k] for k in g.files if k.startswith("spec_")}
    x = orc.make_inputs(int(spec["batch"]), int(spec["dim"]), int(spec["length"]),
                        int(spec["dstate"]), seed=int(spec["seed"]), initial_state=True,
                        valid_lengths=None)
    np.testing.assert_equal(orc_checksum(x), g["input_checksum"])
    ref = orc.fused_backward(x["u"], x["delta"], x["A"], x["B"], x["C"], x["D"], x["z"],
                             x["delta_bias"], True, x["initial_state"], True, None,
                             dout=x["dout"])
    for k in ("out", "last_state", "du", "ddelta", "dA", "dB", "dC", "dD", "dz",
              "ddelta_bias", "dinitial_state"):
        np.testing.assert_allclose(ref[k], g[k], rtol=1e-6, atol=1e-6, err_msg=k)


def orc_checksum(x):
    """float64 sums of every input tensor, to detect a changed input stream."""
    return np.array([float(np.asarray(x[k], dtype=np.float64).sum())
                     for k in ("u", "delta", "A", "B", "C", "D", "z", "delta_bias",
                               "initial_state", "dout")])


@pytest.mark.parametrize("kwidth", [1, 2, 3, 4])
@pytest.mark.parametrize("padded", [False, True])
def test_conv1d_oracle_matches_torch_autograd(kwidth, padded):
    """The conv oracle (flax CAUSAL depthwise conv of mamba/mamba1.py:250-255
    over cache ++ masked input, silu, mask) against torch's grouped conv1d
    with left padding, differentiated by autograd in float64."""
    rng = np.random.default_rng(kwidth * 10 + padded)
    Bn, Dn, L = 3, 5, 23
    x = rng.standard_normal((Bn, Dn, L))
    w = rng.standard_normal((kwidth, Dn))
    b = rng.standard_normal(Dn)
    state = rng.standard_normal((Bn, Dn, kwidth - 1))
    seq = np.array([23, 7, 1], dtype=np.int32) if padded else None
    du = rng.standard_normal((Bn, Dn, L))
    u, final = orc.causal_conv1d_forward(x, w, b, seq, state)
    dx, dw, db, dstate = orc.causal_conv1d_backward(x, w, b, seq, state, du)

    tx = torch.tensor(x, requires_grad=True)
    tw = torch.tensor(w, requires_grad=True)
    tb = torch.tensor(b, requires_grad=True)
    ts = torch.tensor(state, requires_grad=True)
    mask = torch.ones(Bn, 1, L, dtype=torch.float64)
    if padded:
        mask = (torch.arange(L)[None, None, :] < torch.tensor(seq)[:, None, None]).double()
    xc = torch.cat([ts, tx * mask], dim=2)
    # torch conv1d is a cross-correlation with weight (D, 1, K): same taps
    pre = torch.nn.functional.conv1d(xc, tw.t().unsqueeze(1), tb, groups=Dn)
    tu = torch.nn.functional.silu(pre) * mask
    (tu * torch.tensor(du)).sum().backward()
    np.testing.assert_allclose(u, tu.detach().numpy(), rtol=1e-12, atol=1e-12)
    np.testing.assert_allclose(final, xc[:, :, L:].detach().numpy(), rtol=0, atol=0)
    np.testing.assert_allclose(dx, tx.grad.numpy(), rtol=1e-12, atol=1e-12)
    np.testing.assert_allclose(dw, tw.grad.numpy(), rtol=1e-12, atol=1e-12)
    np.testing.assert_allclose(db, tb.grad.numpy(), rtol=1e-12, atol=1e-12)
    np.testing.assert_allclose(dstate, ts.grad.numpy(), rtol=1e-12, atol=1e-12)


def _complex_inputs(seed, batch=2, dim=3, L=11, N=4, padded=False):
    rng = np.random.default_rng(seed)
    cplx = lambda *s: rng.standard_normal(s) + 1j * rng.standard_normal(s)
    # the reference's complex init: A = -exp(Re log(1/2 - i n)) + i Im(...)
    A = -0.5 * np.exp(rng.standard_normal((dim, N)) * 0.3) + 1j * rng.standard_normal((dim, N))
    x = {"u": rng.standard_normal((batch, dim, L)), "delta": rng.standard_normal((batch, dim, L)),
         "A": A, "B": cplx(batch, N, L), "C": cplx(batch, N, L),
         "D": rng.standard_normal(dim), "z": rng.standard_normal((batch, dim, L)),
         "delta_bias": rng.uniform(-4, -2, dim), "initial_state": cplx(batch, dim, N),
         "dout": rng.standard_normal((batch, dim, L)), "dlast": cplx(batch, dim, N),
         "seq_lens": np.array([L, L // 2], dtype=np.int32)[:batch] if padded else None}
    return x


@pytest.mark.parametrize("use_euler", [True, False])
def test_complex_reference_matches_sequential(use_euler):
    """The complex S6 path (mamba/mamba1.py:170-176: discretize, associative
    scan, einsum with C, real part) == the sequential complex loop."""
    x = _complex_inputs(3)
    # reference contract layouts: deltas/u (B, L, D), Bs/Cs (B, L, N)
    args = (x["A"], x["delta"].transpose(0, 2, 1) ** 2, x["B"].transpose(0, 2, 1),
            x["C"].transpose(0, 2, 1), x["u"].transpose(0, 2, 1), None)
    y, f = orc.selective_scan_reference(*args, use_euler_barB_approx=use_euler,
                                        dtype=np.complex128)
    out, last = orc.complex_fused_forward(
        x["u"], x["delta"] ** 2, x["A"], x["B"], x["C"], use_euler_barB_approx=use_euler)
    np.testing.assert_allclose(out, np.real(y).transpose(0, 2, 1), rtol=1e-10, atol=1e-10)
    np.testing.assert_allclose(last, f, rtol=1e-10, atol=1e-10)


@pytest.mark.parametrize("use_euler", [True, False])
@pytest.mark.parametrize("padded", [False, True])
def test_complex_backward_matches_autograd(use_euler, padded):
    """The analytic complex adjoint == torch.autograd in complex128 (torch's
    gradient of a real loss w.r.t. a complex leaf is dL/dRe + i dL/dIm)."""
    x = _complex_inputs(5, padded=padded)
    ref = orc.complex_fused_backward(**{k: v for k, v in x.items()}, delta_softplus=True,
                                     use_euler_barB_approx=use_euler)
    T = {k: torch.tensor(v, requires_grad=True) for k, v in x.items()
         if k in ("u", "delta", "A", "B", "C", "D", "z", "delta_bias", "initial_state")}
    u, dl, A, B, C = T["u"], T["delta"], T["A"], T["B"], T["C"]
    L = u.shape[2]
    mask = torch.ones(u.shape[0], 1, L, dtype=torch.float64)
    if x["seq_lens"] is not None:
        mask = (torch.arange(L)[None, None, :] < torch.tensor(x["seq_lens"])[:, None, None]).double()
    delta = torch.nn.functional.softplus(dl + T["delta_bias"][None, :, None]) * mask
    um = u * mask
    h = T["initial_state"]
    ys = []
    for t in range(L):
        dA = delta[:, :, t, None] * A[None]
        a = torch.exp(dA)
        bb = delta[:, :, t, None] if use_euler else torch.expm1(dA) / A[None]
        h = a * h + bb * B[:, None, :, t] * um[:, :, t, None]
        ys.append(torch.einsum("bn,bdn->bd", C[:, :, t], h).real)
    y = torch.stack(ys, dim=2) + T["D"][None, :, None] * um
    out = y * torch.nn.functional.silu(T["z"]) * mask
    loss = (out * torch.tensor(x["dout"])).sum() + (h * torch.tensor(x["dlast"]).conj()).real.sum()
    loss.backward()
    names = {"u": "du", "delta": "ddelta", "A": "dA", "B": "dB", "C": "dC", "D": "dD",
             "z": "dz", "delta_bias": "ddelta_bias", "initial_state": "dinitial_state"}
    for k, n in names.items():
        np.testing.assert_allclose(ref[n], T[k].grad.numpy(), rtol=1e-9, atol=1e-9, err_msg=n)
