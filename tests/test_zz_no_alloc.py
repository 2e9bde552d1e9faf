"""The allocation-free backward, checked against the regular one.

mamba_ss_fused_bwd_noalloc exists for callers that cannot allocate device
memory themselves (a host runtime that owns all device memory and hands over
tensor pointers only, or code running where cudaMalloc is not permitted); it
takes its scratch from a fixed array inside the library. This file is named
so that pytest collects it last: a run that stops at the first failure has
run every other test before this one.
"""
import ctypes

import numpy as np
import pytest
import torch

from _helpers import BF16_TOL, BWD_TOL, assert_close, rel_err, to_dev
from oracle import selective_scan_oracle as orc

pytestmark = pytest.mark.gpu


def _case(batch, dim, length, seed, io_dtype):
    x = orc.make_inputs(batch, dim, length, 16, seed=seed, initial_state=True)
    io = lambda k: to_dev(x[k], "cuda", io_dtype)
    t = {k: (io(k) if k in ("u", "delta", "B", "C", "z", "dout") else to_dev(v))
         if isinstance(v, np.ndarray) else v for k, v in x.items()}
    from mamba import selective_scan_cuda as ssc

    b, d, L = x["u"].shape
    out = torch.empty_like(t["u"])
    pre = torch.empty_like(t["u"])
    last = torch.empty(b, d, 16, device="cuda")
    cs = torch.empty(ssc.chunk_states_elems(b, L, d, 16), device="cuda")
    ssc.fused_forward_into(t["u"], t["delta"], t["A"], t["B"], t["C"], t["D"], t["z"],
                           t["delta_bias"], True, t["initial_state"], None, out, last, cs,
                           out_pre=pre)
    t["cs"], t["pre"] = cs, pre
    return t


def _grads(t):
    return {k: torch.full_like(t[src], float("nan")) for k, src in
            (("du", "u"), ("ddelta", "delta"), ("dA", "A"), ("dB", "B"), ("dC", "C"),
             ("dD", "D"), ("dz", "z"), ("dbias", "delta_bias"), ("dh0", "initial_state"))}


def _ptr(v):
    return None if v is None else ctypes.c_void_p(v.data_ptr())


def _call_noalloc(lib, t, g):
    from mamba import selective_scan_cuda as ssc

    b, d, L = t["u"].shape
    stream = torch.cuda.current_stream().cuda_stream
    # dinitial_state goes in as a plain int: a wrong argtypes count would cut it
    # to a 32-bit C int and the comparison below would fail
    st = lib.mamba_ss_fused_bwd_noalloc(
        stream, ssc._io_dtype(t["u"]), 0, b, L, d, 16, _ptr(t["u"]), _ptr(t["delta"]),
        _ptr(t["A"]), _ptr(t["B"]), _ptr(t["C"]), _ptr(t["D"]), _ptr(t["z"]),
        _ptr(t["delta_bias"]), 1, _ptr(t["initial_state"]), None, _ptr(t["cs"]),
        _ptr(t["pre"]), _ptr(t["dout"]), None, _ptr(g["du"]), _ptr(g["ddelta"]),
        _ptr(g["dA"]), _ptr(g["dB"]), _ptr(g["dC"]), _ptr(g["dD"]), _ptr(g["dz"]),
        _ptr(g["dbias"]), g["dh0"].data_ptr())
    assert st == 0, lib.mamba_ss_last_error()


@pytest.mark.parametrize("segments", [1, 2], ids=lambda n: f"seg{n}")
@pytest.mark.parametrize("io_dtype", [torch.float32, torch.bfloat16], ids=["f32", "bf16"])
def test_noalloc_backward_matches_regular_backward_twice(io_dtype, segments, monkeypatch):
    """Two calls in a row against mamba_ss_fused_bwd with its own workspace.

    A call of another shape and dtype runs first, so the checked calls start
    from scratch contents that a different problem left behind; bf16 uses the
    fp32 dB/dC accumulators of the scratch and two time segments use its
    segment carries."""
    from mamba import _native
    from mamba import selective_scan_cuda as ssc

    monkeypatch.setenv("MAMBA_SS_SEGMENTS", str(segments))
    lib = _native.load()
    other = torch.bfloat16 if io_dtype == torch.float32 else torch.float32
    s = _case(2, 24, 1100, 5, other)
    _call_noalloc(lib, s, _grads(s))
    t = _case(3, 40, 700, 77, io_dtype)
    b, d, L = t["u"].shape
    ref = _grads(t)
    ws = ssc._alloc_workspace(b, L, d, 16, ssc._io_dtype(t["u"]), "cuda")
    ssc.fused_backward_into(t["u"], t["delta"], t["A"], t["B"], t["C"], t["D"], t["z"],
                            t["delta_bias"], True, t["initial_state"], None, t["cs"],
                            t["dout"], None, ref["du"], ref["ddelta"], ref["dA"], ref["dB"],
                            ref["dC"], ref["dD"], ref["dz"], ref["dbias"], ref["dh0"], ws,
                            out_pre=t["pre"])
    for _ in range(2):  # the shared scratch keeps the previous call's contents
        g = _grads(t)
        _call_noalloc(lib, t, g)
        torch.cuda.synchronize()
        for k in ref:
            a, e = g[k].float().cpu().numpy(), ref[k].float().cpu().numpy()
            if io_dtype == torch.float32 or k in ("dA", "dD", "dbias", "dh0"):
                assert_close(a, e, BWD_TOL, k)
            else:  # bf16 outputs: one rounding step of the narrowed result
                assert rel_err(a, e) < BF16_TOL, k


def test_noalloc_rejects_oversized_problem():
    from mamba import _native

    lib = _native.load()
    cap = lib.mamba_ss_noalloc_scratch_bytes()
    assert cap == 16 << 20
    # batch*dim*dstate*4 bytes of dA partials alone exceed the fixed array
    p = ctypes.c_void_p(256)
    st = lib.mamba_ss_fused_bwd_noalloc(None, 0, 0, 64, 8, 8192, 16, p, p, p, p, p, None, None,
                                        None, 0, None, None, p, None, p, None, p, p, p, p, p,
                                        None, None, None, None)
    assert st == 1
    assert b"scratch" in lib.mamba_ss_last_error()
