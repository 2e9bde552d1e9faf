"""The CPU oracle against outputs of the reference's own code.

tests/golden/ref_*.npz hold y, the final state and the vector-Jacobian
products of ``selective_scan_reference`` (mamba/selective_scan_cuda.py:56-90)
and of S6's complex branch (mamba/mamba1.py:143-176), executed unmodified
under a torch-backed jax.numpy stand-in in float64 by
tests/golden/make_ref_golden.py. Agreement here pins the oracle (and with it
every GPU parity test that compares against the oracle) to the reference
itself rather than to a restatement of it. Tolerance: 1e-6 relative and
absolute (the fixtures are float64 results rounded to float32).
"""
import numpy as np
import pytest

from _helpers import load_ref_golden, ref_tags
from oracle import selective_scan_oracle as orc

TOL = 1e-6
T = lambda a: np.ascontiguousarray(np.swapaxes(a, 1, 2))  # (B, L, X) <-> (B, X, L)


def _close(a, e, name, tol=TOL):
    np.testing.assert_allclose(a, e, rtol=tol, atol=tol * max(1.0, np.abs(e).max()),
                               err_msg=name)


@pytest.mark.parametrize("tag", ref_tags())
def test_oracle_matches_reference_contract(tag):
    c = load_ref_golden("contract")[tag]
    euler = tag.startswith("euler")
    y, fin = orc.selective_scan_reference(c["A"], c["deltas"], c["Bs"], c["Cs"], c["u"],
                                          c["x0"], use_euler_barB_approx=euler)
    _close(y, c["y"], "y")
    _close(fin, c["final"], "final")
    g = orc.fused_backward(T(c["u"]), T(c["deltas"]), c["A"], T(c["Bs"]), T(c["Cs"]),
                           initial_state=c["x0"], use_euler_barB_approx=euler,
                           dout=T(c["dy"]), dlast_state=c["dfinal"])
    for key, name, tr in (("dA", "dA", False), ("ddelta", "ddeltas", True),
                          ("dB", "dBs", True), ("dC", "dCs", True), ("du", "du", True),
                          ("dinitial_state", "dx0", False)):
        _close(T(g[key]) if tr else g[key], c[name], name)


def test_oracle_matches_reference_config0_fused():
    c = load_ref_golden("config0")
    i = {k[3:]: v for k, v in c.items() if k.startswith("in/")}
    kw = dict(D=i["D"], z=i["z"], delta_bias=i["delta_bias"], delta_softplus=True)
    out, last = orc.fused_forward(i["u"], i["delta"], i["A"], i["B"], i["C"], **kw)
    _close(out, c["out"], "out")
    _close(last, c["last_state"], "last_state")
    g = orc.fused_backward(i["u"], i["delta"], i["A"], i["B"], i["C"], **kw, dout=i["dout"])
    for k in ("du", "ddelta", "dA", "dB", "dC", "dD", "dz", "ddelta_bias"):
        _close(g[k], c[k], k)


def test_oracle_matches_reference_mask_padding():
    """The reference's padding (delta and u masked before the scan) keeps the
    last valid state through padded steps, so y there is C_t . h_valid."""
    c = load_ref_golden("padded")
    y, fin = orc.selective_scan_reference(c["A"], c["deltas"], c["Bs"], c["Cs"], c["u"])
    _close(y, c["y"], "y")
    _close(fin, c["final"], "final")
    lens = c["seq_lens"]
    assert np.any(c["y"][1, 1:] != 0.0)  # padded steps are not zero in the reference


@pytest.mark.parametrize("tag", ["euler", "zoh"])
def test_complex_oracle_matches_reference(tag):
    c = load_ref_golden("complex")[tag]
    i = {k[3:]: v for k, v in c.items() if k.startswith("in/")}
    kw = dict(D=i["D"], z=i["z"], delta_bias=i["delta_bias"], delta_softplus=True,
              use_euler_barB_approx=tag == "euler")
    out, last = orc.complex_fused_forward(i["u"], i["delta"], i["A"], i["B"], i["C"], **kw)
    _close(out, c["out"], "out")
    _close(last, c["last_state"], "last_state")
    g = orc.complex_fused_backward(i["u"], i["delta"], i["A"], i["B"], i["C"], **kw,
                                   dout=i["dout"])
    for k in ("du", "ddelta", "dA", "dB", "dC", "dD", "dz", "ddelta_bias"):
        _close(g[k], c[k], k)
