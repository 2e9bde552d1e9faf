"""Writes tests/golden/ref_*.npz by executing the reference's own scan code.

The reference's pure formulation of the selective scan is JAX code:
``selective_scan_reference`` (mamba/selective_scan_cuda.py:56-90) for the real
path, and ``S6.discretize`` / ``S6.binary_operator`` (mamba/mamba1.py:143-158)
that S6.__call__'s complex branch feeds to ``lax.associative_scan``
(mamba/mamba1.py:170-176). JAX is not installed here, so this script lifts
those functions' source text out of the reference files with ``ast``,
unmodified, and executes it against a small torch-backed stand-in for the
parts of ``jax.numpy`` / ``jax.lax`` it touches:

* ``jnp.zeros``, ``jnp.result_type``, ``jnp.einsum``, ``jnp.exp``,
  ``jnp.expm1``, ``jnp.reciprocal``, ``jnp.newaxis`` -> the torch functions of
  the same meaning;
* ``x.at[idx].add(v)`` (JAX's out-of-place indexed update) -> a clone with
  ``idx`` incremented, on a ``torch.Tensor`` subclass carrying ``.at``;
* ``lax.associative_scan(fn, elems, axis)`` -> an inclusive scan by recursive
  doubling (Hillis and Steele, "Data parallel algorithms", CACM 1986): after
  round k element i holds fn applied over elements i-2^k+1..i. It calls the
  reference's own combine function, left operand earlier in time, as JAX does.

Everything runs in float64 (complex128), and the gradients are torch.autograd
through the reference's code, so the fixtures hold the reference's outputs
and vector-Jacobian products, not a restatement of them. Where the fused
Mamba layer math around the scan is needed (softplus(delta + bias) before
the scan, the D skip and the silu(z) gate after it: mamba/mamba1.py:162-198,
308, 332), it is written out below in torch around the reference's code.

Cases (inputs stored as float32 / complex64; outputs rounded to float32):
* ``ref_contract.npz``: the reference test recipe
  (tests/test_selective_scan_cuda.py:11-19) at lengths 1, 17, 31, 128, 513,
  2051, batch 2, dim 8, N 16, both discretizations; outputs y, final state
  and the cotangent products for all six inputs.
* ``ref_config0.npz``: configs[0] (B=2, D=128, L=256, N=16) with the fused
  softplus/bias, D and silu(z) around the reference scan; gradients of all
  eight inputs.
* ``ref_padded.npz``: right padding the reference's way: delta and u
  multiplied by the mask (mamba/mamba1.py:167-168, 325-326), so padded steps
  keep the last valid state and give y = C_t . h_valid.
* ``ref_complex.npz``: the complex branch (S6.discretize and
  S6.binary_operator from the reference, y = Re(C . h) + D u, gated by
  silu(z)), both discretizations.

Needs the reference checkout (REFERENCE_ROOT, default /root/reference); the
GPU box and the tests read only the written .npz files. Run from the
repository root:  python tests/golden/make_ref_golden.py
"""
from __future__ import annotations

import ast
import os
import textwrap
import types
from pathlib import Path

import numpy as np
import torch

OUT = Path(__file__).resolve().parent
REF = Path(os.environ.get("REFERENCE_ROOT", "/root/reference"))
F64, C128 = torch.float64, torch.complex128


# --------------------------------------------------------------------------
# torch-backed stand-in for the jax.numpy / jax.lax names the code uses
# --------------------------------------------------------------------------
class JArray(torch.Tensor):
    """torch.Tensor with JAX's ``.at[idx].add(v)`` out-of-place update."""

    @property
    def at(self):
        return _At(self)


class _At:
    def __init__(self, x):
        self.x = x

    def __getitem__(self, idx):
        return _AtIndex(self.x, idx)


class _AtIndex:
    def __init__(self, x, idx):
        self.x, self.idx = x, idx

    def add(self, v):
        y = self.x.clone()
        y[self.idx] = y[self.idx] + v
        return y


def _j(t):
    return t.as_subclass(JArray) if not isinstance(t, JArray) else t


def _result_type(*xs):
    dt = xs[0].dtype
    for x in xs[1:]:
        dt = torch.promote_types(dt, x.dtype)
    return dt


def _associative_scan(fn, elems, axis=0):
    xs = [_j(e) for e in elems]
    n = xs[0].shape[axis]
    off = 1
    while off < n:
        left = tuple(x.narrow(axis, 0, n - off) for x in xs)
        right = tuple(x.narrow(axis, off, n - off) for x in xs)
        comb = fn(left, right)
        xs = [torch.cat([x.narrow(axis, 0, off), c], dim=axis) for x, c in zip(xs, comb)]
        off *= 2
    return tuple(xs)


jnp = types.SimpleNamespace(
    zeros=lambda shape, dtype=F64: _j(torch.zeros(shape, dtype=dtype)),
    result_type=_result_type,
    einsum=lambda eq, *ops: _j(torch.einsum(eq, *ops)),
    exp=lambda x: _j(torch.exp(x)),
    expm1=lambda x: _j(torch.expm1(x)),
    reciprocal=lambda x: _j(torch.reciprocal(x)),
    newaxis=None,
    float32=torch.float32,
)
lax = types.SimpleNamespace(associative_scan=_associative_scan)
jax = types.SimpleNamespace(numpy=jnp, lax=lax)


def _lift(path, qualname):
    """Source text of a top-level function or a Class.method, unmodified."""
    src = path.read_text()
    tree = ast.parse(src)
    parts = qualname.split(".")
    body = tree.body
    node = None
    for part in parts:
        node = next(n for n in body if isinstance(n, (ast.FunctionDef, ast.ClassDef))
                    and n.name == part)
        body = node.body
    seg = ast.get_source_segment(src, node)
    # drop decorators (none on these functions) and dedent methods
    return textwrap.dedent(seg), node.lineno, node.end_lineno


def load_reference():
    ns = {"jnp": jnp, "jax": jax, "lax": lax}
    scan_file = REF / "mamba" / "selective_scan_cuda.py"
    model_file = REF / "mamba" / "mamba1.py"
    src, a, b = _lift(scan_file, "selective_scan_reference")
    exec(compile(src, f"{scan_file}:{a}-{b}", "exec"), ns)
    src, a, b = _lift(model_file, "S6.discretize")
    exec(compile(src, f"{model_file}:{a}-{b}", "exec"), ns)
    src, a, b = _lift(model_file, "S6.binary_operator")
    exec(compile(src, f"{model_file}:{a}-{b}", "exec"), ns)
    return ns


# --------------------------------------------------------------------------
# cases
# --------------------------------------------------------------------------
def _leaf(a, dtype=F64):
    return _j(torch.from_numpy(np.asarray(a)).to(dtype)).requires_grad_(True)


def _f32(t):
    return t.detach().to(torch.float32 if not t.is_complex() else torch.complex64).numpy()


def _silu(x):
    return x * torch.sigmoid(x)


def _softplus(x):
    return torch.nn.functional.softplus(x)


def contract_cases(ref):
    """The reference test recipe through the reference's own function."""
    out = {}
    for use_euler in (True, False):
        for length in (1, 17, 31, 128, 513, 2051):
            rng = np.random.default_rng(1000 + length * 2 + int(use_euler))
            batch, dim, n = 2, 8, 16
            A = -np.exp(rng.standard_normal((dim, n)))
            deltas = np.logaddexp(rng.standard_normal((batch, length, dim)), 0.0)
            Bs = rng.standard_normal((batch, length, n))
            Cs = rng.standard_normal((batch, length, n))
            u = rng.standard_normal((batch, length, dim))
            x0 = rng.standard_normal((batch, dim, n))
            dy = rng.standard_normal((batch, length, dim))
            dfin = rng.standard_normal((batch, dim, n))
            ins = [a.astype(np.float32) for a in (A, deltas, Bs, Cs, u, x0)]
            leaves = [_leaf(a) for a in ins]
            y, fin = ref["selective_scan_reference"](*leaves, use_euler_barB_approx=use_euler)
            loss = (y * torch.from_numpy(dy.astype(np.float32)).double()).sum() + \
                (fin * torch.from_numpy(dfin.astype(np.float32)).double()).sum()
            grads = torch.autograd.grad(loss, leaves)
            tag = f"{'euler' if use_euler else 'zoh'}_L{length}"
            for name, a in zip(("A", "deltas", "Bs", "Cs", "u", "x0"), ins):
                out[f"{tag}/{name}"] = a
            out[f"{tag}/dy"] = dy.astype(np.float32)
            out[f"{tag}/dfinal"] = dfin.astype(np.float32)
            out[f"{tag}/y"] = _f32(y)
            out[f"{tag}/final"] = _f32(fin)
            for name, g in zip(("dA", "ddeltas", "dBs", "dCs", "du", "dx0"), grads):
                out[f"{tag}/{name}"] = _f32(g)
    return out


def fused_layer(ref, u, delta, A, B, C, D, z, bias, initial=None, use_euler=True):
    """(B, D, L) fused layer math around the reference scan: softplus(delta +
    bias) (mamba1.py:164, tau_Delta of the biased projection), the scan on
    (B, L, D) operands, + D u (mamba1.py:195-196) and * silu(z) (mamba1.py:308,
    332). Returns out (B, D, L) and the final state."""
    d_eff = _softplus(delta + bias[None, :, None])
    y, fin = ref["selective_scan_reference"](
        A, _j(d_eff.transpose(1, 2)), _j(B.transpose(1, 2)), _j(C.transpose(1, 2)),
        _j(u.transpose(1, 2)), initial, use_euler_barB_approx=use_euler)
    y = y.transpose(1, 2) + D[None, :, None] * u
    return y * _silu(z), fin


def config0_case(ref):
    """B=2, D=128, L=256, N=16 with its value distributions."""
    rng = np.random.default_rng(2024)
    b, d, L, n = 2, 128, 256, 16
    ins = {
        "u": rng.standard_normal((b, d, L)), "delta": rng.standard_normal((b, d, L)),
        "A": -np.exp(np.log(np.tile(np.arange(1, n + 1, dtype=np.float64), (d, 1)))),
        "B": rng.standard_normal((b, n, L)), "C": rng.standard_normal((b, n, L)),
        "D": rng.standard_normal(d), "z": rng.standard_normal((b, d, L)),
        "delta_bias": rng.uniform(-4.0, -2.0, d),
    }
    ins = {k: v.astype(np.float32) for k, v in ins.items()}
    dout = rng.standard_normal((b, d, L)).astype(np.float32)
    leaves = {k: _leaf(v) for k, v in ins.items()}
    out, fin = fused_layer(ref, leaves["u"], leaves["delta"], leaves["A"], leaves["B"],
                           leaves["C"], leaves["D"], leaves["z"], leaves["delta_bias"])
    keys = list(leaves)
    grads = torch.autograd.grad((out * torch.from_numpy(dout).double()).sum(),
                                [leaves[k] for k in keys])
    res = {f"in/{k}": v for k, v in ins.items()}
    res["in/dout"] = dout
    res["out"], res["last_state"] = _f32(out), _f32(fin)
    for k, g in zip(keys, grads):
        res[f"d{k}"] = _f32(g)
    return res


def padded_case(ref):
    """Right padding as the reference layer does it: delta and u multiplied
    by the mask before the scan (mamba1.py:167-168 and 325-326)."""
    rng = np.random.default_rng(77)
    b, L, d, n = 3, 300, 8, 16
    lens = np.array([300, 1, 137], dtype=np.int32)
    mask = (np.arange(L)[None, :] < lens[:, None]).astype(np.float64)[:, :, None]
    A = -np.exp(rng.standard_normal((d, n)))
    deltas = np.logaddexp(rng.standard_normal((b, L, d)), 0.0) * mask
    Bs = rng.standard_normal((b, L, n))
    Cs = rng.standard_normal((b, L, n))
    u = rng.standard_normal((b, L, d)) * mask
    dy = rng.standard_normal((b, L, d))
    ins = [a.astype(np.float32) for a in (A, deltas, Bs, Cs, u)]
    leaves = [_leaf(a) for a in ins]
    y, fin = ref["selective_scan_reference"](*leaves, use_euler_barB_approx=True)
    grads = torch.autograd.grad((y * torch.from_numpy(dy.astype(np.float32)).double()).sum(),
                                leaves)
    res = {"seq_lens": lens, "dy": dy.astype(np.float32)}
    for name, a in zip(("A", "deltas", "Bs", "Cs", "u"), ins):
        res[name] = a
    res["y"], res["final"] = _f32(y), _f32(fin)
    for name, g in zip(("dA", "ddeltas", "dBs", "dCs", "du"), grads):
        res[name] = _f32(g)
    return res


def complex_cases(ref):
    """S6.__call__'s complex branch (mamba1.py:170-176, 195-198) run from the
    reference's discretize and binary_operator, gated by silu(z)."""
    out = {}
    for use_euler in (True, False):
        rng = np.random.default_rng(55 + int(use_euler))
        b, d, L, n = 2, 8, 129, 16
        cplx = lambda *s: (rng.standard_normal(s) + 1j * rng.standard_normal(s))
        ins = {
            "u": rng.standard_normal((b, d, L)), "delta": rng.standard_normal((b, d, L)),
            "A": -0.5 * np.exp(rng.standard_normal((d, n)) * 0.3)
            + 1j * (np.arange(n)[None, :] + 0.3 * rng.standard_normal((d, n))),
            "B": cplx(b, n, L), "C": cplx(b, n, L), "D": rng.standard_normal(d),
            "z": rng.standard_normal((b, d, L)), "delta_bias": rng.uniform(-4.0, -2.0, d),
        }
        ins = {k: v.astype(np.complex64 if np.iscomplexobj(v) else np.float32)
               for k, v in ins.items()}
        dout = rng.standard_normal((b, d, L)).astype(np.float32)
        leaves = {k: _leaf(v, C128 if np.iscomplexobj(v) else F64) for k, v in ins.items()}
        me = types.SimpleNamespace(euler_barB_approx=use_euler)
        d_eff = _softplus(leaves["delta"] + leaves["delta_bias"][None, :, None])
        x = leaves["u"].transpose(1, 2)  # (b, L, d), real
        A_bars, B_bars = ref["discretize"](me, leaves["A"], _j(leaves["B"].transpose(1, 2)),
                                           _j(d_eff.transpose(1, 2).to(C128)))
        Bx = B_bars * x[..., None]
        _, xs = lax.associative_scan(ref["binary_operator"], (A_bars, Bx), axis=1)
        ys = jnp.einsum("bln,bldn->bld", leaves["C"].transpose(1, 2), xs)
        ys = ys + leaves["D"] * x
        y = ys.real.transpose(1, 2) * _silu(leaves["z"])
        keys = list(leaves)
        grads = torch.autograd.grad((y * torch.from_numpy(dout).double()).sum(),
                                    [leaves[k] for k in keys])
        tag = "euler" if use_euler else "zoh"
        for k, v in ins.items():
            out[f"{tag}/in/{k}"] = v
        out[f"{tag}/in/dout"] = dout
        out[f"{tag}/out"], out[f"{tag}/last_state"] = _f32(y), _f32(xs[:, -1])
        for k, g in zip(keys, grads):
            out[f"{tag}/d{k}"] = _f32(g)
    return out


def main():
    ref = load_reference()
    np.savez_compressed(OUT / "ref_contract.npz", **contract_cases(ref))
    np.savez_compressed(OUT / "ref_config0.npz", **config0_case(ref))
    np.savez_compressed(OUT / "ref_padded.npz", **padded_case(ref))
    np.savez_compressed(OUT / "ref_complex.npz", **complex_cases(ref))
    for f in sorted(OUT.glob("ref_*.npz")):
        print(f.name, f.stat().st_size)


if __name__ == "__main__":
    main()
