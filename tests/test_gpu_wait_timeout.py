"""The bounded staging waits' failure path, forced without a GPU fault.

mamba_ss_debug_set_wait_polls(0) makes every scan kernel's wait for a tile's
TMA copies give up at once, as a copy that never completes would after 2^22
polls. The kernel must then report bit 0 through
mamba_ss_take_device_error(), let its copies in flight land, and return; the
context stays usable, so the next call with the default limit is correct and
reports no error. The copies are real local loads; nothing waits on a flag
that another kernel or rank sets."""
import numpy as np
import pytest
import torch

from _helpers import BWD_TOL, FWD_TOL, assert_close, oracle_fused, to_dev
from oracle import selective_scan_oracle as orc

pytestmark = pytest.mark.gpu


def _bufs(x, ssc):
    t = {k: to_dev(v) if isinstance(v, np.ndarray) else v for k, v in x.items()}
    b, d, L = x["u"].shape
    t["out"], t["pre"] = torch.empty_like(t["u"]), torch.empty_like(t["u"])
    t["last"] = torch.empty(b, d, 16, device="cuda")
    t["cs"] = torch.empty(ssc.chunk_states_elems(b, L, d, 16), device="cuda")
    return t


def _fwd(t, ssc):
    ssc.fused_forward_into(t["u"], t["delta"], t["A"], t["B"], t["C"], t["D"], t["z"],
                           t["delta_bias"], True, t["initial_state"], None, t["out"], t["last"],
                           t["cs"], out_pre=t["pre"])


def _bwd(t, ssc):
    b, d, L = t["u"].shape
    g = {k: torch.empty_like(t[src]) for k, src in
         (("du", "u"), ("ddelta", "delta"), ("dA", "A"), ("dB", "B"), ("dC", "C"), ("dD", "D"),
          ("dz", "z"), ("ddelta_bias", "delta_bias"), ("dinitial_state", "initial_state"))}
    ws = ssc._alloc_workspace(b, L, d, 16, 0, "cuda")
    ssc.fused_backward_into(t["u"], t["delta"], t["A"], t["B"], t["C"], t["D"], t["z"],
                            t["delta_bias"], True, t["initial_state"], None, t["cs"], t["dout"],
                            None, g["du"], g["ddelta"], g["dA"], g["dB"], g["dC"], g["dD"],
                            g["dz"], g["ddelta_bias"], g["dinitial_state"], ws, out_pre=t["pre"])
    return g


@pytest.fixture
def lib():
    from mamba import _native

    lib = _native.load()
    torch.cuda.synchronize()
    assert lib.mamba_ss_take_device_error() == 0
    yield lib
    lib.mamba_ss_debug_set_wait_polls(-1)


@pytest.mark.parametrize("segments", [1, 3], ids=lambda n: f"seg{n}")
def test_forced_wait_timeout_is_reported_and_the_next_call_is_clean(lib, segments, monkeypatch):
    from mamba import selective_scan_cuda as ssc

    monkeypatch.setenv("MAMBA_SS_SEGMENTS", str(segments))
    x = orc.make_inputs(2, 16, 512, 16, seed=13, initial_state=True)
    ref = oracle_fused(x)
    t = _bufs(x, ssc)

    # forward gives up
    lib.mamba_ss_debug_set_wait_polls(0)
    _fwd(t, ssc)
    torch.cuda.synchronize()
    assert lib.mamba_ss_take_device_error() & 1
    lib.mamba_ss_debug_set_wait_polls(-1)
    _fwd(t, ssc)
    torch.cuda.synchronize()
    assert lib.mamba_ss_take_device_error() == 0
    assert_close(t["out"].cpu().numpy(), ref["out"], FWD_TOL, "out")

    # backward gives up (after a complete forward)
    lib.mamba_ss_debug_set_wait_polls(0)
    _bwd(t, ssc)
    torch.cuda.synchronize()
    assert lib.mamba_ss_take_device_error() & 1
    lib.mamba_ss_debug_set_wait_polls(-1)
    g = _bwd(t, ssc)
    torch.cuda.synchronize()
    assert lib.mamba_ss_take_device_error() == 0
    for k in g:
        assert_close(g[k].cpu().numpy(), ref[k], BWD_TOL, k)
