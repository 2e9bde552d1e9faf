"""The fused scan at the benchmark's full sizes, checked through properties
that hold at any size (the float64 oracle runs the whole problem only at
small sizes):

- sampled channels against the oracle: every per-channel output (out,
  last_state, du, ddelta, dz) and parameter gradient (dA, dD, ddelta_bias,
  summed over the batch) depends only on its own channel's inputs and B, C,
  so the oracle runs those channels alone, over the full length and batch;
- dB and dC are sums over channels: the full call's equal the sum of two
  calls on the two halves of the channels (linearity);
- padded positions of out, du, ddelta and dz are exact zeros.

B=8, D=1536, L=2048, N=16, fp32. configs[2]: B=16, D=5120,
L=4096, bf16 I/O, valid lengths ~U[512, 4096]. Seeded synthetic inputs with
the configs' distributions, generated on the GPU."""
import numpy as np
import pytest
import torch

from _helpers import assert_bf16_close, BF16_TOL, BWD_TOL, FWD_TOL, assert_close, rel_err
from oracle import selective_scan_oracle as orc

pytestmark = pytest.mark.gpu


def _inputs(b, d, L, n, io, seed, padded):
    g = torch.Generator(device="cuda").manual_seed(seed)
    rn = lambda *s: torch.randn(*s, generator=g, device="cuda")
    x = {"u": rn(b, d, L).to(io), "delta": rn(b, d, L).to(io), "z": rn(b, d, L).to(io),
         "B": rn(b, n, L).to(io), "C": rn(b, n, L).to(io), "dout": rn(b, d, L).to(io),
         "D": rn(d),
         "delta_bias": torch.rand(d, generator=g, device="cuda") * 2.0 - 4.0,
         "A": -torch.arange(1, n + 1, device="cuda", dtype=torch.float32).repeat(d, 1)}
    x["seq_lens"] = (torch.randint(512, L + 1, (b,), generator=g, device="cuda",
                                   dtype=torch.int32) if padded else None)
    return x


def _run(x, ch=slice(None)):
    from mamba.selective_scan_cuda import selective_scan_fn

    t = {k: x[k][:, ch].contiguous() for k in ("u", "delta", "z")}
    t.update({k: x[k][ch].contiguous() for k in ("A", "D", "delta_bias")})
    t.update({k: x[k] for k in ("B", "C")})
    t = {k: v.detach().clone().requires_grad_(True) for k, v in t.items()}
    out, last = selective_scan_fn(t["u"], t["delta"], t["A"], t["B"], t["C"], t["D"], t["z"],
                                  t["delta_bias"], True, True, seq_lens=x["seq_lens"])
    out.backward(x["dout"][:, ch].contiguous())
    res = {"out": out.detach(), "last_state": last.detach()}
    names = {"u": "du", "delta": "ddelta", "A": "dA", "B": "dB", "C": "dC", "D": "dD",
             "z": "dz", "delta_bias": "ddelta_bias"}
    res.update({names[k]: v.grad for k, v in t.items()})
    return res


def _oracle(x, ch):
    f = lambda v: v.float().cpu().numpy()
    seq = x["seq_lens"].cpu().numpy() if x["seq_lens"] is not None else None
    return orc.fused_backward(f(x["u"][:, ch]), f(x["delta"][:, ch]), f(x["A"][ch]),
                              f(x["B"]), f(x["C"]), f(x["D"][ch]), f(x["z"][:, ch]),
                              f(x["delta_bias"][ch]), True, None, True, seq,
                              dout=f(x["dout"][:, ch]))


def _check(x, res, ch, tol_fwd, tol_bwd, bf16):
    ref = _oracle(x, ch)
    sel = {"out": res["out"][:, ch], "last_state": res["last_state"][:, ch],
           "du": res["du"][:, ch], "ddelta": res["ddelta"][:, ch], "dz": res["dz"][:, ch],
           "dA": res["dA"][ch], "dD": res["dD"][ch], "ddelta_bias": res["ddelta_bias"][ch]}
    for k, v in sel.items():
        a = v.float().cpu().numpy()
        if bf16:
            assert_bf16_close(a, ref[k], k)
        else:
            assert_close(a, ref[k], tol_fwd if k in ("out", "last_state") else tol_bwd, k)


def _check_channel_linearity(x, res, tol):
    d = x["u"].shape[1]
    h = d // 2
    lo, hi = _run(x, slice(0, h)), _run(x, slice(h, d))
    for k in ("dB", "dC"):
        rel = ((lo[k].float() + hi[k].float() - res[k].float()).abs().max()
               / res[k].float().abs().max()).item()
        assert rel < tol, (k, rel)


def test_config1_full_size():
    b, d, L, n = 8, 1536, 2048, 16
    x = _inputs(b, d, L, n, torch.float32, 1, padded=False)
    res = _run(x)
    ch = [0, 7, 8, 513, 1535]
    _check(x, res, ch, FWD_TOL, BWD_TOL, bf16=False)
    _check_channel_linearity(x, res, BWD_TOL)


def test_config2_full_size():
    b, d, L, n = 16, 5120, 4096, 16
    x = _inputs(b, d, L, n, torch.bfloat16, 2, padded=True)
    res = _run(x)
    # every padded position of every channel is an exact zero
    pos = torch.arange(L, device="cuda")[None, None, :]
    pad = pos >= x["seq_lens"].long()[:, None, None]
    for k in ("out", "du", "ddelta", "dz"):
        assert not (res[k].float().abs() * pad).any(), k
    ch = [0, 31, 32, 2600, 5119]
    _check(x, res, ch, None, None, bf16=True)
    # bf16 dB/dC are rounded once per call: the halves' sum differs from the
    # full call's by that rounding
    _check_channel_linearity(x, res, BF16_TOL)
