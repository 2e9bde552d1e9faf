"""Host-side API of mamba.selective_scan_cuda without a GPU: the reference
formulation, the routing of selective_scan, validation errors, and that the
CUDA path refuses to run on CPU tensors instead of falling back."""
import numpy as np
import pytest
import torch

from oracle import selective_scan_oracle as orc
from mamba import selective_scan_cuda as ssc


def _inputs(batch=2, length=17, dim=8, n=16, seed=7):
    rng = np.random.default_rng(seed)
    A = -np.exp(rng.standard_normal((dim, n)))
    deltas = np.logaddexp(rng.standard_normal((batch, length, dim)), 0.0)
    Bs = rng.standard_normal((batch, length, n))
    Cs = rng.standard_normal((batch, length, n))
    u = rng.standard_normal((batch, length, dim))
    x0 = rng.standard_normal((batch, dim, n))
    return [a.astype(np.float32) for a in (A, deltas, Bs, Cs, u, x0)]


@pytest.mark.parametrize("use_euler", [True, False])
@pytest.mark.parametrize("remat", [False, True])
def test_reference_path_matches_oracle(use_euler, remat):
    args = _inputs()
    y, f = ssc.selective_scan(*map(torch.from_numpy, args), use_euler_barB_approx=use_euler,
                              remat=remat)
    ey, ef = orc.selective_scan_reference(*args, use_euler_barB_approx=use_euler)
    np.testing.assert_allclose(y.numpy(), ey, rtol=2e-5, atol=2e-5)
    np.testing.assert_allclose(f.numpy(), ef, rtol=2e-5, atol=2e-5)


def test_default_initial_state_is_zero():
    args = _inputs()
    y0, _ = ssc.selective_scan(*map(torch.from_numpy, args[:5]))
    ey, _ = orc.selective_scan_reference(*args[:5], np.zeros_like(args[5]))
    np.testing.assert_allclose(y0.numpy(), ey, rtol=2e-5, atol=2e-5)


def test_validation_errors():
    A, d, B, C, u, x0 = map(torch.from_numpy, _inputs())
    with pytest.raises(TypeError):
        ssc._validate_inputs(A.double(), d, B, C, u, x0)
    with pytest.raises(ValueError, match="N must be one of"):
        ssc._validate_inputs(A[:, :3], d, B[..., :3], C[..., :3], u, x0[..., :3])
    with pytest.raises(ValueError, match="Bs must have shape"):
        ssc._validate_inputs(A, d, B[:, :5], C, u, x0)
    with pytest.raises(ValueError, match="CUDA tensors"):
        ssc._validate_inputs(A, d, B, C, u, x0)


def test_cuda_path_never_falls_back_on_cpu_tensors():
    args = list(map(torch.from_numpy, _inputs()))
    with pytest.raises(ValueError, match="CUDA"):
        ssc.selective_scan(*args, use_cuda=True)
    x = orc.make_inputs(1, 4, 8, 16)
    t = {k: torch.from_numpy(v) if isinstance(v, np.ndarray) else v for k, v in x.items()}
    with pytest.raises(ValueError, match="CUDA"):
        ssc.selective_scan_fn(t["u"], t["delta"], t["A"], t["B"], t["C"], t["D"], t["z"],
                              t["delta_bias"], True)


def test_fused_validation():
    x = orc.make_inputs(1, 4, 8, 16)
    t = {k: torch.from_numpy(v) if isinstance(v, np.ndarray) else v for k, v in x.items()}
    with pytest.raises(ValueError, match="B must have shape"):
        ssc._check_fused(t["u"], t["delta"], t["A"], t["B"][:, :8], t["C"], None, None,
                         None, None, None)
    with pytest.raises(TypeError):
        ssc._check_fused(t["u"].double(), t["delta"], t["A"], t["B"], t["C"], None, None,
                         None, None, None)
    with pytest.raises(TypeError, match="delta must have dtype"):
        ssc._check_fused(t["u"], t["delta"].bfloat16(), t["A"], t["B"], t["C"], None, None,
                         None, None, None)


def test_register_missing_library_lists_paths(tmp_path):
    with pytest.raises(FileNotFoundError, match="searched"):
        ssc.register_cuda_kernel(tmp_path / "nope.so")
