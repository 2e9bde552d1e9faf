"""GPU parity of the recurrent decode step (S6.step, mamba/mamba1.py:200-214)
against the CPU oracle, and its consistency with the full scan: L decode
steps reproduce the fused forward's outputs and last state."""
import numpy as np
import pytest
import torch

from _helpers import assert_bf16_close, BF16_TOL, FWD_TOL, assert_close, bf16_round, rel_err, to_dev
from oracle import selective_scan_oracle as orc

pytestmark = pytest.mark.gpu


def _step_inputs(batch, dim, n, seed):
    rng = np.random.default_rng(seed)
    f = np.float32
    return dict(state=rng.standard_normal((batch, dim, n)).astype(f),
                u=rng.standard_normal((batch, dim)).astype(f),
                delta=rng.standard_normal((batch, dim)).astype(f),
                A=-np.exp(rng.standard_normal((dim, n))).astype(f),
                B=rng.standard_normal((batch, n)).astype(f),
                C=rng.standard_normal((batch, n)).astype(f),
                D=rng.standard_normal(dim).astype(f),
                z=rng.standard_normal((batch, dim)).astype(f),
                bias=rng.uniform(-4, -2, dim).astype(f))


@pytest.mark.parametrize("dstate", [1, 2, 4, 8, 16])
@pytest.mark.parametrize("use_euler", [True, False])
def test_step_matches_oracle(dstate, use_euler):
    from mamba.selective_scan_cuda import selective_state_update

    x = _step_inputs(3, 37, dstate, seed=dstate)
    st = to_dev(x["state"])
    out = selective_state_update(st, to_dev(x["u"]), to_dev(x["delta"]), to_dev(x["A"]),
                                 to_dev(x["B"]), to_dev(x["C"]), to_dev(x["D"]), to_dev(x["z"]),
                                 to_dev(x["bias"]), True, use_euler_barB_approx=use_euler)
    ey, eh = orc.fused_step(x["state"], x["u"], x["delta"], x["A"], x["B"], x["C"], x["D"],
                            x["z"], x["bias"], True, use_euler)
    assert_close(out.cpu().numpy(), ey, FWD_TOL, "out")
    assert_close(st.cpu().numpy(), eh, FWD_TOL, "state")


def test_step_bf16():
    from mamba.selective_scan_cuda import selective_state_update

    x = _step_inputs(4, 64, 16, seed=1)
    st = to_dev(x["state"])
    bf = torch.bfloat16
    out = selective_state_update(st, to_dev(x["u"], dtype=bf), to_dev(x["delta"], dtype=bf),
                                 to_dev(x["A"]), to_dev(x["B"], dtype=bf),
                                 to_dev(x["C"], dtype=bf), to_dev(x["D"]),
                                 to_dev(x["z"], dtype=bf), to_dev(x["bias"]), True)
    r = lambda k: bf16_round(x[k])
    ey, eh = orc.fused_step(x["state"], r("u"), r("delta"), x["A"], r("B"), r("C"), x["D"],
                            r("z"), x["bias"], True)
    assert_bf16_close(out.float().cpu().numpy(), ey)
    assert_bf16_close(st.cpu().numpy(), eh)


def test_steps_reproduce_the_scan():
    """Decoding token by token equals one scan over the sequence."""
    from mamba.selective_scan_cuda import selective_scan_fn, selective_state_update

    xi = orc.make_inputs(2, 24, 40, 16, seed=12, initial_state=True)
    t = {k: to_dev(v) if isinstance(v, np.ndarray) else v for k, v in xi.items()}
    out, last = selective_scan_fn(t["u"], t["delta"], t["A"], t["B"], t["C"], t["D"], t["z"],
                                  t["delta_bias"], True, True, initial_state=t["initial_state"])
    st = t["initial_state"].clone()
    ys = []
    for s in range(xi["u"].shape[2]):
        ys.append(selective_state_update(
            st, t["u"][:, :, s], t["delta"][:, :, s], t["A"], t["B"][:, :, s], t["C"][:, :, s],
            t["D"], t["z"][:, :, s], t["delta_bias"], True))
    y = torch.stack(ys, 2)
    assert_close(y.cpu().numpy(), out.cpu().numpy(), FWD_TOL, "out")
    assert_close(st.cpu().numpy(), last.cpu().numpy(), FWD_TOL, "state")


def test_step_validation():
    from mamba.selective_scan_cuda import selective_state_update

    st = torch.zeros(2, 4, 16, device="cuda")
    v = torch.zeros(2, 4, device="cuda")
    bc = torch.zeros(2, 16, device="cuda")
    with pytest.raises(ValueError, match="B must have shape"):
        selective_state_update(st, v, v, torch.zeros(4, 16, device="cuda"), bc[:, :8], bc)
