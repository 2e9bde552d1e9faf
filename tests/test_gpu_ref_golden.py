"""The sm_100a kernels against outputs of the reference's own code.

The fixtures (tests/golden/ref_*.npz, written by
tests/golden/make_ref_golden.py) hold what the reference's
``selective_scan_reference`` (mamba/selective_scan_cuda.py:56-90) and S6's
complex branch (mamba/mamba1.py:143-176) return, and their vector-Jacobian
products, executed in float64. Each case goes through this package's public
ops: ``selective_scan`` (the reference's signature and (B, L, D) layout),
``selective_scan_fn`` (fused softplus/bias, D, silu(z)) and
``selective_scan_complex_fn``. Tolerances as stated for the path: fp32
forward 1e-5 (rtol and atol), fp32 backward 1e-4; complex gradients 1e-4
relative to each gradient's largest magnitude (as the complex parity tests).
"""
import numpy as np
import pytest
import torch

from _helpers import BWD_TOL, FWD_TOL, assert_close, load_ref_golden, ref_tags, rel_err, to_dev

pytestmark = pytest.mark.gpu


def _bwd_close(a, e, name):
    assert_close(a, e, BWD_TOL, name)  # 1e-4 relative and absolute, per element


@pytest.mark.parametrize("tag", ref_tags())
def test_reference_contract_matches_reference_code(tag):
    from mamba.selective_scan_cuda import selective_scan

    c = load_ref_golden("contract")[tag]
    args = [to_dev(c[k]).requires_grad_(True) for k in ("A", "deltas", "Bs", "Cs", "u", "x0")]
    y, fin = selective_scan(*args, use_euler_barB_approx=tag.startswith("euler"),
                            use_cuda=True)
    assert_close(y.detach().cpu().numpy(), c["y"], FWD_TOL, "y")
    assert_close(fin.detach().cpu().numpy(), c["final"], FWD_TOL, "final")
    ((y * to_dev(c["dy"])).sum() + (fin * to_dev(c["dfinal"])).sum()).backward()
    for a, name in zip(args, ("dA", "ddeltas", "dBs", "dCs", "du", "dx0")):
        _bwd_close(a.grad.cpu().numpy(), c[name], name)


def test_config0_fused_matches_reference_code():
    from mamba.selective_scan_cuda import selective_scan_fn

    c = load_ref_golden("config0")
    t = {k[3:]: to_dev(v) for k, v in c.items() if k.startswith("in/")}
    keys = ("u", "delta", "A", "B", "C", "D", "z", "delta_bias")
    for k in keys:
        t[k].requires_grad_(True)
    out, last = selective_scan_fn(t["u"], t["delta"], t["A"], t["B"], t["C"], t["D"], t["z"],
                                  t["delta_bias"], True, True)
    assert_close(out.detach().cpu().numpy(), c["out"], FWD_TOL, "out")
    assert_close(last.detach().cpu().numpy(), c["last_state"], FWD_TOL, "last_state")
    (out * t["dout"]).sum().backward()
    for k in keys:
        _bwd_close(t[k].grad.cpu().numpy(), c["d" + k], "d" + k)


def test_mask_padding_gives_reference_values():
    """Padding applied the reference's way, outside the kernel (delta and u
    multiplied by the mask, mamba/mamba1.py:167-168): the kernel then returns
    the reference's C_t . h_valid at padded steps, not zeros (the zeros are
    only what the seq_lens extension writes)."""
    from mamba.selective_scan_cuda import selective_scan

    c = load_ref_golden("padded")
    args = [to_dev(c[k]).requires_grad_(True) for k in ("A", "deltas", "Bs", "Cs", "u")]
    y, fin = selective_scan(*args, use_euler_barB_approx=True, use_cuda=True)
    yh = y.detach().cpu().numpy()
    assert_close(yh, c["y"], FWD_TOL, "y")
    assert_close(fin.detach().cpu().numpy(), c["final"], FWD_TOL, "final")
    assert np.any(yh[1, 1:] != 0.0)
    (y * to_dev(c["dy"])).sum().backward()
    for a, name in zip(args, ("dA", "ddeltas", "dBs", "dCs", "du")):
        _bwd_close(a.grad.cpu().numpy(), c[name], name)


@pytest.mark.parametrize("tag", ["euler", "zoh"])
def test_complex_matches_reference_code(tag):
    from mamba.selective_scan_complex import selective_scan_complex_fn

    c = load_ref_golden("complex")[tag]
    t = {k[3:]: to_dev(v) for k, v in c.items() if k.startswith("in/")}
    keys = ("u", "delta", "A", "B", "C", "D", "z", "delta_bias")
    for k in keys:
        t[k].requires_grad_(True)
    out, last = selective_scan_complex_fn(t["u"], t["delta"], t["A"], t["B"], t["C"], t["D"],
                                          t["z"], t["delta_bias"], True, True,
                                          use_euler_barB_approx=tag == "euler")
    assert_close(out.detach().cpu().numpy(), c["out"], FWD_TOL, "out")
    assert_close(last.detach().cpu().numpy(), c["last_state"], FWD_TOL, "last_state")
    (out * t["dout"]).sum().backward()
    for k in keys:
        g = t[k].grad.cpu().numpy()
        assert rel_err(g, c["d" + k]) < BWD_TOL, ("d" + k, rel_err(g, c["d" + k]))
