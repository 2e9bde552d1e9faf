"""GPU parity of the causal conv1d + SiLU kernels (mamba_ss_conv1d_fwd/bwd)
against the CPU oracle (float64).

Tolerances as for the scan: fp32 forward 1e-5, fp32 backward 1e-4, bf16 I/O
2e-2 relative to the largest magnitude; masked steps exactly zero. Cases:
every kernel width 1..4, lengths around the 128-step warp chunk and the
4-step vector groups, ragged channel counts, padding, the conv state in and
out, and the bf16 path.
"""
import numpy as np
import pytest
import torch

from _helpers import assert_bf16_close, BF16_TOL, BWD_TOL, FWD_TOL, assert_close, bf16_round, rel_err, to_dev
from oracle import selective_scan_oracle as orc

pytestmark = pytest.mark.gpu


def _inputs(Bn, Dn, L, K, seed, padded=False, state=True):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((Bn, Dn, L)).astype(np.float32)
    w = (rng.standard_normal((K, Dn)) * 0.5).astype(np.float32)
    b = rng.standard_normal(Dn).astype(np.float32)
    st = rng.standard_normal((Bn, Dn, K - 1)).astype(np.float32) if state else None
    seq = rng.integers(0, L + 1, Bn).astype(np.int32) if padded else None
    du = rng.standard_normal((Bn, Dn, L)).astype(np.float32)
    return x, w, b, seq, st, du


def _run(x, w, b, seq, st, du, io=torch.float32):
    from mamba.causal_conv1d import causal_conv1d_fn

    tx = to_dev(x, dtype=io).requires_grad_(True)
    tw = to_dev(w).requires_grad_(True)
    tb = to_dev(b).requires_grad_(True) if b is not None else None
    ts = to_dev(st, dtype=io).requires_grad_(True) if st is not None else None
    tseq = to_dev(seq) if seq is not None else None
    u, final = causal_conv1d_fn(tx, tw, tb, tseq, ts, return_final_state=True)
    (u.float() * to_dev(du)).sum().backward()
    torch.cuda.synchronize()
    out = {"u": u.detach().float().cpu().numpy(), "final": final.float().cpu().numpy(),
           "dx": tx.grad.float().cpu().numpy(), "dw": tw.grad.cpu().numpy()}
    if tb is not None:
        out["db"] = tb.grad.cpu().numpy()
    if ts is not None:
        out["dstate"] = ts.grad.float().cpu().numpy()
    return out


def _ref(x, w, b, seq, st, du):
    u, final = orc.causal_conv1d_forward(x, w, b, seq, st)
    dx, dw, db, dstate = orc.causal_conv1d_backward(x, w, b, seq, st, du)
    return {"u": u, "final": final, "dx": dx, "dw": dw, "db": db, "dstate": dstate}


@pytest.mark.parametrize("K", [1, 2, 3, 4])
@pytest.mark.parametrize("L", [1, 3, 5, 127, 128, 129, 300, 1000])
def test_fp32(K, L):
    args = _inputs(2, 7, L, K, seed=K * 1000 + L)
    res, ref = _run(*args), _ref(*args)
    assert_close(res["u"], ref["u"], FWD_TOL, "u")
    assert_close(res["final"], ref["final"], FWD_TOL, "final")
    for k in ("dx", "dw", "db", "dstate"):
        if k in res:
            assert_close(res[k], ref[k], BWD_TOL, k)


@pytest.mark.parametrize("K", [2, 4])
def test_padding_exact_zeros(K):
    args = _inputs(4, 9, 400, K, seed=77 + K, padded=True)
    x, w, b, seq, st, du = args
    seq[:] = [400, 0, 129, 3]
    res, ref = _run(*args), _ref(*args)
    for k in ("u", "final"):
        assert_close(res[k], ref[k], FWD_TOL, k)
    for k in ("dx", "dw", "db", "dstate"):
        assert_close(res[k], ref[k], BWD_TOL, k)
    for bi, n in enumerate(seq):
        assert np.all(res["u"][bi, :, n:] == 0.0)
        assert np.all(res["dx"][bi, :, n:] == 0.0)


def test_no_bias_no_state():
    x, w, b, seq, st, du = _inputs(3, 5, 256, 4, seed=5, state=False)
    res, ref = _run(x, w, None, seq, None, du), _ref(x, w, None, seq, None, du)
    assert_close(res["u"], ref["u"], FWD_TOL, "u")
    for k in ("dx", "dw"):
        assert_close(res[k], ref[k], BWD_TOL, k)


@pytest.mark.parametrize("L", [512, 509])
def test_bf16(L):
    x, w, b, seq, st, du = _inputs(2, 16, L, 4, seed=L)
    xr, str_ = bf16_round(x), bf16_round(st)
    res = _run(x, w, b, seq, st, du, io=torch.bfloat16)
    ref = _ref(xr, w, b, seq, str_, bf16_round(du))
    for k in ("u", "final", "dx", "dw", "db", "dstate"):
        assert_bf16_close(res[k], ref[k], k)


def test_rejects_bad_arguments():
    from mamba import _native
    from mamba.causal_conv1d import conv1d_forward_into

    x = torch.zeros(1, 4, 8, device="cuda")
    w = torch.zeros(5, 4, device="cuda")  # kwidth 5 is not supported
    with pytest.raises(ValueError):
        conv1d_forward_into(x, w, None, None, None, torch.empty_like(x))
    assert b"kwidth" in _native.load().mamba_ss_last_error()


@pytest.mark.parametrize("K", [2, 4])
@pytest.mark.parametrize("io", [torch.float32, torch.bfloat16])
def test_decode_steps_match_the_sequence(K, io):
    """Token-by-token conv steps reproduce the full-sequence conv (the
    reference's Mamba.step vs Mamba.__call__, mamba/mamba1.py:301-355), and
    leave the same conv state."""
    from mamba.causal_conv1d import causal_conv1d_fn, causal_conv1d_update

    x, w, b, _, st, _ = _inputs(3, 10, 9, K, seed=40 + K)
    tx, tw, tb = to_dev(x, dtype=io), to_dev(w), to_dev(b)
    tst = to_dev(st, dtype=io)
    u_seq, final = causal_conv1d_fn(tx, tw, tb, None, tst.clone(), return_final_state=True)
    state = tst.clone()
    steps = [causal_conv1d_update(tx[:, :, t], state, tw, tb) for t in range(x.shape[2])]
    u_step = torch.stack(steps, dim=2)
    tol = FWD_TOL if io == torch.float32 else BF16_TOL
    assert_close(u_step.float().cpu().numpy(), u_seq.float().cpu().numpy(), tol, "u")
    assert torch.equal(state, final)
