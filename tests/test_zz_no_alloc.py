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

from _helpers import BWD_TOL, assert_close, to_dev
from oracle import selective_scan_oracle as orc

pytestmark = pytest.mark.gpu


def _case():
    x = orc.make_inputs(3, 40, 700, 16, seed=77, initial_state=True)
    t = {k: to_dev(v) if isinstance(v, np.ndarray) else v for k, v in x.items()}
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
    b, d, L = t["u"].shape
    stream = torch.cuda.current_stream().cuda_stream
    st = lib.mamba_ss_fused_bwd_noalloc(
        stream, 0, 0, b, L, d, 16, _ptr(t["u"]), _ptr(t["delta"]), _ptr(t["A"]), _ptr(t["B"]),
        _ptr(t["C"]), _ptr(t["D"]), _ptr(t["z"]), _ptr(t["delta_bias"]), 1,
        _ptr(t["initial_state"]), None, _ptr(t["cs"]), _ptr(t["pre"]), _ptr(t["dout"]), None,
        _ptr(g["du"]), _ptr(g["ddelta"]), _ptr(g["dA"]), _ptr(g["dB"]), _ptr(g["dC"]),
        _ptr(g["dD"]), _ptr(g["dz"]), _ptr(g["dbias"]), _ptr(g["dh0"]))
    assert st == 0, lib.mamba_ss_last_error()


def test_noalloc_backward_matches_regular_backward_twice():
    from mamba import _native
    from mamba import selective_scan_cuda as ssc

    lib = _native.load()
    t = _case()
    b, d, L = t["u"].shape
    ref = _grads(t)
    ws = ssc._alloc_workspace(b, L, d, 16, 0, "cuda")
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
            assert_close(g[k].cpu().numpy(), ref[k].cpu().numpy(), BWD_TOL, k)


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
