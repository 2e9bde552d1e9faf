"""GPU parity of the complex selective scan (complex_ssm, mamba/mamba1.py:
170-176) against the float64 complex oracle: forward, last state and every
gradient (complex ones as dL/dRe + i dL/dIm), Euler and ZOH, padding, initial
state and a last-state cotangent. Tolerances: forward 1e-5 (rtol and atol,
as the real path); backward 1e-4 relative to each gradient's largest
magnitude (slowly decaying complex modes sum many large terms of opposite
sign, so single small elements carry fp32 rounding of the large ones)."""
import numpy as np
import pytest
import torch

from _helpers import BWD_TOL, FWD_TOL, assert_close, rel_err
from oracle import selective_scan_oracle as orc

pytestmark = pytest.mark.gpu


def _inputs(batch, dim, L, N, seed, padded=False):
    rng = np.random.default_rng(seed)
    cplx = lambda *s: (rng.standard_normal(s) + 1j * rng.standard_normal(s)).astype(np.complex64)
    # the reference's init: A = -1/2 + i n, kept in a stable range here
    A = (-0.5 * np.exp(rng.standard_normal((dim, N)) * 0.3)
         + 1j * (np.arange(N)[None, :] + 0.3 * rng.standard_normal((dim, N)))).astype(np.complex64)
    f32 = lambda *s: rng.standard_normal(s).astype(np.float32)
    x = {"u": f32(batch, dim, L), "delta": f32(batch, dim, L), "A": A,
         "B": cplx(batch, N, L), "C": cplx(batch, N, L), "D": f32(dim), "z": f32(batch, dim, L),
         "delta_bias": rng.uniform(-4, -2, dim).astype(np.float32),
         "initial_state": cplx(batch, dim, N), "dout": f32(batch, dim, L),
         "dlast": cplx(batch, dim, N), "seq_lens": None}
    if padded:
        x["seq_lens"] = rng.integers(1, L + 1, batch).astype(np.int32)
    return x


def _run(x, zoh):
    from mamba.selective_scan_complex import selective_scan_complex_fn

    dev = "cuda"
    T = {k: torch.from_numpy(np.ascontiguousarray(v)).to(dev) for k, v in x.items()
         if v is not None and k not in ("dout", "dlast", "seq_lens")}
    for v in T.values():
        v.requires_grad_(True)
    seq = torch.from_numpy(x["seq_lens"]).to(dev) if x["seq_lens"] is not None else None
    out, last = selective_scan_complex_fn(
        T["u"], T["delta"], T["A"], T["B"], T["C"], T["D"], T["z"], T["delta_bias"], True, True,
        initial_state=T["initial_state"], use_euler_barB_approx=not zoh, seq_lens=seq)
    dout = torch.from_numpy(x["dout"]).to(dev)
    dlast = torch.from_numpy(x["dlast"]).to(dev)
    loss = (out * dout).sum() + (last * dlast.conj()).real.sum()
    loss.backward()
    torch.cuda.synchronize()
    names = {"u": "du", "delta": "ddelta", "A": "dA", "B": "dB", "C": "dC", "D": "dD", "z": "dz",
             "delta_bias": "ddelta_bias", "initial_state": "dinitial_state"}
    res = {"out": out.detach().cpu().numpy(), "last_state": last.detach().cpu().numpy()}
    for k, n in names.items():
        res[n] = T[k].grad.cpu().numpy()
    return res


def _ref(x, zoh):
    kw = dict(D=x["D"], z=x["z"], delta_bias=x["delta_bias"], delta_softplus=True,
              initial_state=x["initial_state"], use_euler_barB_approx=not zoh,
              seq_lens=x["seq_lens"])
    out, last = orc.complex_fused_forward(x["u"], x["delta"], x["A"], x["B"], x["C"], **kw)
    g = orc.complex_fused_backward(x["u"], x["delta"], x["A"], x["B"], x["C"], **kw,
                                   dout=x["dout"], dlast=x["dlast"])
    return {"out": out, "last_state": last, **g}


def _check(res, ref):
    assert_close(res["out"], ref["out"], FWD_TOL, "out")
    assert_close(res["last_state"], ref["last_state"], FWD_TOL, "last_state")
    for k in ("du", "ddelta", "dA", "dB", "dC", "dD", "dz", "ddelta_bias", "dinitial_state"):
        assert rel_err(res[k], ref[k]) < BWD_TOL, (k, rel_err(res[k], ref[k]))


@pytest.mark.parametrize("L", [1, 17, 128, 513])
@pytest.mark.parametrize("N", [1, 4, 16])
def test_complex_euler(L, N):
    x = _inputs(2, 6, L, N, seed=L * 7 + N)
    _check(_run(x, False), _ref(x, False))


@pytest.mark.parametrize("L", [17, 300])
def test_complex_zoh(L):
    x = _inputs(2, 5, L, 8, seed=L)
    _check(_run(x, True), _ref(x, True))


def test_complex_padding():
    x = _inputs(3, 9, 200, 16, seed=99, padded=True)
    res = _run(x, False)
    _check(res, _ref(x, False))
    for b, n in enumerate(x["seq_lens"]):
        for k in ("out", "du", "ddelta", "dz"):
            assert np.all(res[k][b, :, n:] == 0.0), (k, b)
