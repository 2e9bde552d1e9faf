"""Shared test helpers: oracle inputs -> CUDA tensors, and kernel calls."""
from __future__ import annotations

import numpy as np
import torch

from oracle import selective_scan_oracle as orc

FWD_TOL = 1e-5   # fp32 forward, relative and absolute
BWD_TOL = 1e-4   # fp32 backward
BF16_TOL = 2e-2  # bf16 inputs, fp32 state: relative, per element
BF16_ATOL = 1e-3  # floor for elements near zero, as a fraction of the tensor's peak


def to_dev(x, dev="cuda", dtype=None):
    if x is None:
        return None
    t = torch.from_numpy(np.ascontiguousarray(x)).to(dev)
    if dtype is not None and t.is_floating_point():
        t = t.to(dtype)
    return t


def run_fused(x, *, dev="cuda", io_dtype=torch.float32, zoh=False, grads=True,
              with_dlast=False):
    """Run selective_scan_fn forward (+ backward) on the GPU for oracle inputs x."""
    from mamba.selective_scan_cuda import selective_scan_fn

    io = lambda k: to_dev(x[k], dev, io_dtype)
    f32 = lambda k: to_dev(x[k], dev)
    t = {"u": io("u"), "delta": io("delta"), "B": io("B"), "C": io("C"),
         "z": io("z") if x["z"] is not None else None,
         "A": f32("A"), "D": f32("D") if x["D"] is not None else None,
         "delta_bias": f32("delta_bias") if x["delta_bias"] is not None else None,
         "initial_state": f32("initial_state") if x["initial_state"] is not None else None}
    seq = to_dev(x["seq_lens"], dev) if x["seq_lens"] is not None else None
    if grads:
        for v in t.values():
            if v is not None:
                v.requires_grad_(True)
    out, last = selective_scan_fn(t["u"], t["delta"], t["A"], t["B"], t["C"], t["D"], t["z"],
                                  t["delta_bias"], x["delta_softplus"], True,
                                  initial_state=t["initial_state"],
                                  use_euler_barB_approx=not zoh, seq_lens=seq)
    res = {"out": out.detach().float().cpu().numpy(),
           "last_state": last.detach().cpu().numpy()}
    if grads:
        dout = to_dev(x["dout"], dev, io_dtype)
        loss = (out.float() * dout.float()).sum()
        if with_dlast:
            loss = loss + (last * to_dev(x["dlast"], dev)).sum()
        loss.backward()
        names = {"u": "du", "delta": "ddelta", "A": "dA", "B": "dB", "C": "dC", "D": "dD",
                 "z": "dz", "delta_bias": "ddelta_bias", "initial_state": "dinitial_state"}
        for k, v in t.items():
            if v is not None:
                res[names[k]] = v.grad.float().cpu().numpy()
    torch.cuda.synchronize()
    return res


def oracle_fused(x, *, zoh=False, with_dlast=False, dtype=np.float64, io_round=None):
    """Oracle forward+backward in float64 for the same inputs.

    io_round: a callable applied to the I/O tensors first (e.g. bf16 rounding),
    so that the oracle sees exactly what the kernel reads.
    """
    r = (lambda v: v) if io_round is None else io_round
    g = lambda k: None if x[k] is None else r(x[k])
    return orc.fused_backward(g("u"), g("delta"), x["A"], g("B"), g("C"), x["D"], g("z"),
                              x["delta_bias"], x["delta_softplus"], x["initial_state"],
                              not zoh, x["seq_lens"], dout=g("dout"),
                              dlast_state=x.get("dlast") if with_dlast else None,
                              dtype=dtype)


def bf16_round(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(torch.bfloat16).float().numpy()


def assert_close(actual, expected, tol, name=""):
    np.testing.assert_allclose(actual, expected, rtol=tol, atol=tol, err_msg=name)


def assert_bf16_close(actual, expected, name=""):
    """Per element: |a - e| <= 2e-2 |e| + 1e-3 max|e|.

    The absolute floor covers elements that cancel to near zero: their error
    is fp32 accumulation noise of the large terms, which scales with the
    tensor's magnitude, not the element's."""
    a = np.asarray(actual, dtype=np.float64)
    e = np.asarray(expected, dtype=np.float64)
    bound = BF16_TOL * np.abs(e) + BF16_ATOL * max(np.abs(e).max(), 1e-30)
    bad = np.abs(a - e) > bound
    if bad.any():
        i = np.unravel_index(np.argmax(np.abs(a - e) - bound), a.shape)
        raise AssertionError(f"{name}: {int(bad.sum())} of {a.size} elements outside the bf16 "
                             f"bound; worst at {i}: {a[i]} vs {e[i]}")


def rel_err(actual, expected):
    """max |a-e| / max |e| (a scale-aware error for low-precision checks)."""
    den = max(np.abs(expected).max(), 1e-30)
    return float(np.abs(actual - expected).max() / den)


GOLDEN = __import__("pathlib").Path(__file__).resolve().parent / "golden"


def load_ref_golden(name):
    """Fixtures written by tests/golden/make_ref_golden.py from the reference's
    own code (keys "group/name"); returned as {group: {name: array}} or, for
    files without groups, {name: array}."""
    z = np.load(GOLDEN / f"ref_{name}.npz")
    out = {}
    for k in z.files:
        if "/" in k and not k.startswith("in/"):
            g, rest = k.split("/", 1)
            out.setdefault(g, {})[rest] = z[k]
        else:
            out[k] = z[k]
    return out


def ref_tags(lengths=None):
    """Case tags of ref_contract.npz: '{euler|zoh}_L{length}'."""
    z = np.load(GOLDEN / "ref_contract.npz")
    tags = sorted({k.split("/")[0] for k in z.files}, key=lambda t: (t.split("_")[0],
                                                                      int(t.split("L")[1])))
    return [t for t in tags if lengths is None or int(t.split("L")[1]) in lengths]
