"""Selective-scan op API for the B200 kernels (host side, PyTorch tensors).

Mirrors the public interface of JAX-Mambas ``mamba/selective_scan_cuda.py``:

* ``register_cuda_kernel(library_path=None)``      (reference :26-53)
* ``selective_scan_reference(A, deltas, Bs, Cs, u, initial_x=None, *,
  use_euler_barB_approx=True)``                    (reference :56-90)
* ``selective_scan(A, deltas, Bs, Cs, u, initial_x=None, *,
  use_euler_barB_approx=True, use_cuda=False, remat=False) -> (y, final_x)``
                                                   (reference :262-308)

and adds the fused north-star entry point

* ``selective_scan_fn(u, delta, A, B, C, D=None, z=None, delta_bias=None,
  delta_softplus=False, return_last_state=False, *, initial_state=None,
  use_euler_barB_approx=True, seq_lens=None)``

The reference differentiates through ``jax.custom_vjp``
(reference :217-259); here the same forward/backward pairing is a
``torch.autograd.Function`` whose forward and backward call the sm_100a
kernels through the C ABI. ``use_cuda=True`` and ``selective_scan_fn`` never
fall back to another implementation: without the built library they raise.
``use_cuda=False`` evaluates the reference formulation, exactly as the
reference's own default does.
"""
from __future__ import annotations

import torch

from . import _native

_REGISTERED = False
_LIBRARY = None
_VALID_N = (1, 2, 4, 8, 16)


def register_cuda_kernel(library_path=None):
    """Load the compiled selective-scan library (reference :26-53).

    Raises ``FileNotFoundError`` listing the searched paths when the library
    has not been built.
    """
    global _LIBRARY, _REGISTERED
    if _REGISTERED and library_path is None:
        return _LIBRARY
    _LIBRARY = _native.load(library_path)
    _REGISTERED = True
    return _LIBRARY


def _lib():
    return register_cuda_kernel()


def _ptr(t):
    return None if t is None else t.data_ptr()


def _stream(device):
    return torch.cuda.current_stream(device).cuda_stream


# --------------------------------------------------------------------------
# Reference formulation (reference :56-90), in torch.
# --------------------------------------------------------------------------
def _associative_scan(a, h, dim=1):
    n = a.shape[dim]
    s = 1
    while s < n:
        a_lo, a_hi = a.narrow(dim, 0, n - s), a.narrow(dim, s, n - s)
        h_lo, h_hi = h.narrow(dim, 0, n - s), h.narrow(dim, s, n - s)
        new_h_hi = a_hi * h_lo + h_hi
        new_a_hi = a_hi * a_lo
        a = torch.cat([a.narrow(dim, 0, s), new_a_hi], dim)
        h = torch.cat([h.narrow(dim, 0, s), new_h_hi], dim)
        s *= 2
    return a, h


def selective_scan_reference(A, deltas, Bs, Cs, u, initial_x=None, *,
                             use_euler_barB_approx=True):
    """Reference selective scan with the same contract as the CUDA kernel."""
    if initial_x is None:
        initial_x = torch.zeros((u.shape[0], u.shape[2], A.shape[1]),
                                dtype=torch.result_type(A, u), device=u.device)
    delta_a = torch.einsum("bld,dn->bldn", deltas, A)
    a_bars = torch.exp(delta_a)
    if use_euler_barB_approx:
        b_bars = torch.einsum("bld,bln->bldn", deltas, Bs)
    else:
        b_bars = torch.expm1(delta_a) * torch.einsum("dn,bln->bldn", torch.reciprocal(A), Bs)
    bu = b_bars * u[..., None]
    bu = torch.cat([(bu[:, :1] + a_bars[:, :1] * initial_x[:, None]), bu[:, 1:]], 1)
    _, states = _associative_scan(a_bars, bu, 1)
    y = torch.einsum("bln,bldn->bld", Cs, states)
    return y, states[:, -1]


# --------------------------------------------------------------------------
# Validation (reference :93-121)
# --------------------------------------------------------------------------
def _validate_inputs(A, deltas, Bs, Cs, u, initial_x):
    if any(v.dtype != torch.float32 for v in (A, deltas, Bs, Cs, u, initial_x)):
        raise TypeError("The CUDA selective scan currently supports float32 only")
    if A.ndim != 2 or u.ndim != 3:
        raise ValueError("A must have shape (D, N) and u must have shape (B, L, D)")
    batch, length, dim = u.shape
    n = A.shape[1]
    if length == 0:
        raise ValueError("The sequence length must be positive")
    if n not in _VALID_N:
        raise ValueError("N must be one of 1, 2, 4, 8, or 16")
    expected = {
        "A": (dim, n),
        "deltas": (batch, length, dim),
        "Bs": (batch, length, n),
        "Cs": (batch, length, n),
        "initial_x": (batch, dim, n),
    }
    actual = {
        "A": tuple(A.shape),
        "deltas": tuple(deltas.shape),
        "Bs": tuple(Bs.shape),
        "Cs": tuple(Cs.shape),
        "initial_x": tuple(initial_x.shape),
    }
    for name, shape in expected.items():
        if actual[name] != shape:
            raise ValueError(f"{name} must have shape {shape}, got {actual[name]}")
    for v in (A, deltas, Bs, Cs, u, initial_x):
        if not v.is_cuda:
            raise ValueError("The CUDA selective scan needs CUDA tensors")


# --------------------------------------------------------------------------
# Raw launches (device tensors in kernel layout, outputs preallocated)
# --------------------------------------------------------------------------
def set_deterministic(on=True):
    """Make dB and dC of every later backward bitwise reproducible (per-warp
    partial sums added in a fixed order by a second kernel, instead of fp32
    atomics in arrival order), or restore the default. Process-wide; costs
    the partials' extra memory traffic. Workspaces sized before the switch
    are too small for a deterministic backward."""
    _lib().mamba_ss_set_deterministic(1 if on else 0)


def is_deterministic():
    return bool(_lib().mamba_ss_deterministic())


def chunk_states_elems(batch, length, dim, dstate):
    return int(_lib().mamba_ss_chunk_states_elems(batch, length, dim, dstate))


def bwd_workspace_bytes(batch, length, dim, dstate, io_dtype=_native.MSS_F32):
    return int(_lib().mamba_ss_bwd_workspace_bytes(batch, length, dim, dstate, io_dtype))


def _io_dtype(t):
    if t.dtype == torch.float32:
        return _native.MSS_F32
    if t.dtype == torch.bfloat16:
        return _native.MSS_BF16
    raise TypeError("selective scan I/O must be float32 or bfloat16, got " + str(t.dtype))


def fused_forward_into(u, delta, A, B, C, D, z, delta_bias, delta_softplus,
                       initial_state, seq_lens, out, last_state, chunk_states,
                       zoh=False, out_pre=None):
    """Launch the fused forward on the current stream into given buffers."""
    lib = _lib()
    batch, dim, length = u.shape
    dstate = A.shape[1]
    st = lib.mamba_ss_fused_fwd(
        _stream(u.device), _io_dtype(u), int(zoh), batch, length, dim, dstate,
        _ptr(u), _ptr(delta), _ptr(A), _ptr(B), _ptr(C), _ptr(D), _ptr(z),
        _ptr(delta_bias), int(bool(delta_softplus)), _ptr(initial_state),
        _ptr(seq_lens), _ptr(out), _ptr(out_pre), _ptr(last_state), _ptr(chunk_states))
    _native.check(lib, st)


def fused_backward_into(u, delta, A, B, C, D, z, delta_bias, delta_softplus,
                        initial_state, seq_lens, chunk_states, dout, dlast_state,
                        du, ddelta, dA, dB, dC, dD, dz, ddelta_bias,
                        dinitial_state, workspace, zoh=False, out_pre=None):
    """Launch the fused backward on the current stream into given buffers."""
    lib = _lib()
    batch, dim, length = u.shape
    dstate = A.shape[1]
    st = lib.mamba_ss_fused_bwd(
        _stream(u.device), _io_dtype(u), int(zoh), batch, length, dim, dstate,
        _ptr(u), _ptr(delta), _ptr(A), _ptr(B), _ptr(C), _ptr(D), _ptr(z),
        _ptr(delta_bias), int(bool(delta_softplus)), _ptr(initial_state),
        _ptr(seq_lens), _ptr(chunk_states), _ptr(out_pre), _ptr(dout), _ptr(dlast_state),
        _ptr(du), _ptr(ddelta), _ptr(dA), _ptr(dB), _ptr(dC), _ptr(dD),
        _ptr(dz), _ptr(ddelta_bias), _ptr(dinitial_state), _ptr(workspace),
        0 if workspace is None else workspace.numel())
    _native.check(lib, st)


def _alloc_workspace(batch, length, dim, dstate, io_dtype, device):
    nbytes = bwd_workspace_bytes(batch, length, dim, dstate, io_dtype)
    ws = torch.empty(nbytes + 256, dtype=torch.uint8, device=device)
    off = (-ws.data_ptr()) % 256
    return ws[off:off + nbytes]


# --------------------------------------------------------------------------
# Fused op (north-star signature)
# --------------------------------------------------------------------------
def _check_fused(u, delta, A, B, C, D, z, delta_bias, initial_state, seq_lens):
    if u.ndim != 3:
        raise ValueError("u must have shape (B, D, L)")
    batch, dim, length = u.shape
    if length == 0:
        raise ValueError("The sequence length must be positive")
    if A.ndim != 2 or A.shape[0] != dim:
        raise ValueError(f"A must have shape ({dim}, N), got {tuple(A.shape)}")
    n = A.shape[1]
    if n not in _VALID_N:
        raise ValueError("N must be one of 1, 2, 4, 8, or 16")
    io = u.dtype
    if io not in (torch.float32, torch.bfloat16):
        raise TypeError("u must be float32 or bfloat16")
    shapes = {"delta": (delta, (batch, dim, length)), "B": (B, (batch, n, length)),
              "C": (C, (batch, n, length)), "z": (z, (batch, dim, length))}
    for name, (t, shape) in shapes.items():
        if t is None:
            continue
        if tuple(t.shape) != shape:
            raise ValueError(f"{name} must have shape {shape}, got {tuple(t.shape)}")
        if t.dtype != io:
            raise TypeError(f"{name} must have dtype {io}, got {t.dtype}")
    params = {"A": (A, (dim, n)), "D": (D, (dim,)), "delta_bias": (delta_bias, (dim,)),
              "initial_state": (initial_state, (batch, dim, n))}
    for name, (t, shape) in params.items():
        if t is None:
            continue
        if tuple(t.shape) != shape:
            raise ValueError(f"{name} must have shape {shape}, got {tuple(t.shape)}")
        if t.dtype != torch.float32:
            raise TypeError(f"{name} must be float32, got {t.dtype}")
    if seq_lens is not None:
        if tuple(seq_lens.shape) != (batch,) or seq_lens.dtype != torch.int32:
            raise ValueError("seq_lens must be an int32 tensor of shape (B,)")
    for t in (u, delta, A, B, C, D, z, delta_bias, initial_state, seq_lens):
        if t is not None and not t.is_cuda:
            raise ValueError("selective_scan_fn needs CUDA tensors")


class _FusedScan(torch.autograd.Function):
    @staticmethod
    def forward(ctx, u, delta, A, B, C, D, z, delta_bias, initial_state,
                delta_softplus, zoh, seq_lens):
        c = lambda t: None if t is None else t.contiguous()
        u, delta, A, B, C, D, z, delta_bias, initial_state, seq_lens = map(
            c, (u, delta, A, B, C, D, z, delta_bias, initial_state, seq_lens))
        batch, dim, length = u.shape
        n = A.shape[1]
        out = torch.empty_like(u)
        # saved carries and the pre-gate output only when a backward can follow
        # (needs_input_grad is all False under no_grad; grad mode itself is
        # always off inside forward)
        grads = any(ctx.needs_input_grad[:9])
        pre = torch.empty_like(u) if (z is not None and grads) else None
        last = torch.empty((batch, dim, n), dtype=torch.float32, device=u.device)
        cs = (torch.empty(chunk_states_elems(batch, length, dim, n),
                          dtype=torch.float32, device=u.device) if grads else None)
        fused_forward_into(u, delta, A, B, C, D, z, delta_bias, delta_softplus,
                           initial_state, seq_lens, out, last, cs, zoh, pre)
        ctx.save_for_backward(u, delta, A, B, C, D, z, delta_bias, initial_state,
                              seq_lens, cs, pre)
        ctx.delta_softplus = delta_softplus
        ctx.zoh = zoh
        return out, last

    @staticmethod
    def backward(ctx, dout, dlast):
        u, delta, A, B, C, D, z, delta_bias, h0, seq_lens, cs, pre = ctx.saved_tensors
        batch, dim, length = u.shape
        n = A.shape[1]
        if dout is None:
            dout = torch.zeros_like(u)
        dout = dout.to(u.dtype).contiguous()
        dlast = None if dlast is None else dlast.float().contiguous()
        du = torch.empty_like(u)
        ddelta = torch.empty_like(delta)
        dA = torch.empty_like(A)
        dB = torch.empty_like(B)
        dC = torch.empty_like(C)
        dD = torch.empty_like(D) if D is not None else None
        dz = torch.empty_like(z) if z is not None else None
        dbias = torch.empty_like(delta_bias) if delta_bias is not None else None
        dh0 = torch.empty_like(h0) if h0 is not None else None
        ws = _alloc_workspace(batch, length, dim, n, _io_dtype(u), u.device)
        fused_backward_into(u, delta, A, B, C, D, z, delta_bias, ctx.delta_softplus,
                            h0, seq_lens, cs, dout, dlast, du, ddelta, dA, dB, dC,
                            dD, dz, dbias, dh0, ws, ctx.zoh, pre)
        return du, ddelta, dA, dB, dC, dD, dz, dbias, dh0, None, None, None


def selective_scan_fn(u, delta, A, B, C, D=None, z=None, delta_bias=None,
                      delta_softplus=False, return_last_state=False, *,
                      initial_state=None, use_euler_barB_approx=True,
                      seq_lens=None):
    """Fused selective scan on the sm_100a kernels.

    Layouts: u, delta, z (B, D, L); A (D, N); B, C (B, N, L); D, delta_bias
    (D,); initial_state (B, D, N) fp32; seq_lens (B,) int32 (steps at or past
    seq_lens[b] are padding: their output and input gradients are zero).
    Returns out (B, D, L) in u's dtype, and last_state (B, D, N) fp32 when
    ``return_last_state``.
    """
    _check_fused(u, delta, A, B, C, D, z, delta_bias, initial_state, seq_lens)
    out, last = _FusedScan.apply(u, delta, A, B, C, D, z, delta_bias, initial_state,
                                 bool(delta_softplus), not use_euler_barB_approx,
                                 seq_lens)
    return (out, last) if return_last_state else out


# --------------------------------------------------------------------------
# Recurrent decode step (S6.step / Mamba.step, mamba/mamba1.py:200-214)
# --------------------------------------------------------------------------
def selective_state_update(state, u, delta, A, B, C, D=None, z=None, delta_bias=None,
                           delta_softplus=False, *, use_euler_barB_approx=True):
    """One decode step for one new token per sequence on the sm_100a kernel.

    state (B, D, N) fp32 is updated in place; u, delta, z are (B, D) and B, C
    (B, N) in fp32 or bf16; returns out (B, D) = (C . h + D u) * silu(z).
    """
    if state.ndim != 3 or state.dtype != torch.float32:
        raise ValueError("state must be a float32 tensor of shape (B, D, N)")
    batch, dim, n = state.shape
    if n not in _VALID_N:
        raise ValueError("N must be one of 1, 2, 4, 8, or 16")
    io = u.dtype
    for name, t, shape in (("u", u, (batch, dim)), ("delta", delta, (batch, dim)),
                           ("B", B, (batch, n)), ("C", C, (batch, n)), ("z", z, (batch, dim))):
        if t is None:
            continue
        if tuple(t.shape) != shape:
            raise ValueError(f"{name} must have shape {shape}, got {tuple(t.shape)}")
        if t.dtype != io:
            raise TypeError(f"{name} must have dtype {io}")
    for t in (state, u, delta, A, B, C, D, z, delta_bias):
        if t is not None and not t.is_cuda:
            raise ValueError("selective_state_update needs CUDA tensors")
    if not state.is_contiguous():
        raise ValueError("state must be contiguous (it is updated in place)")
    c = lambda t: None if t is None else t.contiguous()
    u, delta, A, B, C, D, z, delta_bias = map(c, (u, delta, A, B, C, D, z, delta_bias))
    out = torch.empty_like(u)
    fused_step_into(state, u, delta, A, B, C, D, z, delta_bias, delta_softplus, out,
                    zoh=not use_euler_barB_approx)
    return out


def fused_step_into(state, u, delta, A, B, C, D, z, delta_bias, delta_softplus, out,
                    zoh=False):
    """Launch one decode step on the current stream into a given `out`
    (contiguous CUDA tensors, no checks beyond the C ABI's)."""
    lib = _lib()
    batch, dim, n = state.shape
    st = lib.mamba_ss_fused_step(
        _stream(u.device), _io_dtype(u), int(zoh), batch, dim, n,
        _ptr(state), _ptr(u), _ptr(delta), _ptr(A), _ptr(B), _ptr(C), _ptr(D), _ptr(z),
        _ptr(delta_bias), int(bool(delta_softplus)), _ptr(out))
    _native.check(lib, st)


# --------------------------------------------------------------------------
# Reference contract (reference :217-308)
# --------------------------------------------------------------------------
class _SelectiveScanCuda(torch.autograd.Function):
    """Forward/backward pair of the reference's ``_selective_scan_cuda``
    custom_vjp (reference :217-259), on the sm_100a kernels for both
    discretizations."""

    @staticmethod
    def forward(ctx, A, deltas, Bs, Cs, u, initial_x, use_euler_barB_approx):
        lib = _lib()
        batch, length, dim = u.shape
        n = A.shape[1]
        # physical layouts of the reference FFI call (reference :138-146)
        d_p = deltas.transpose(1, 2).contiguous()
        u_p = u.transpose(1, 2).contiguous()
        B_p = Bs.transpose(1, 2).contiguous()
        C_p = Cs.transpose(1, 2).contiguous()
        A_c = A.contiguous()
        h0 = initial_x.contiguous()
        y_p = torch.empty_like(u_p)
        final = torch.empty((batch, dim, n), dtype=torch.float32, device=u.device)
        cs = torch.empty(chunk_states_elems(batch, length, dim, n),
                         dtype=torch.float32, device=u.device)
        st = lib.mamba_ss_fwd(_stream(u.device), 0 if use_euler_barB_approx else 1,
                              batch, length, dim, n, _ptr(A_c), _ptr(d_p), _ptr(B_p),
                              _ptr(C_p), _ptr(u_p), _ptr(h0), _ptr(y_p), _ptr(final),
                              _ptr(cs))
        _native.check(lib, st)
        ctx.save_for_backward(A_c, d_p, B_p, C_p, u_p, h0, cs)
        ctx.euler = use_euler_barB_approx
        return y_p.transpose(1, 2), final

    @staticmethod
    def backward(ctx, dy, dfinal):
        lib = _lib()
        A, d_p, B_p, C_p, u_p, h0, cs = ctx.saved_tensors
        batch, dim, length = u_p.shape
        n = A.shape[1]
        dy_p = (torch.zeros_like(u_p) if dy is None
                else dy.transpose(1, 2).contiguous())
        dfinal = (torch.zeros_like(h0) if dfinal is None else dfinal.contiguous())
        dA = torch.empty_like(A)
        dd = torch.empty_like(d_p)
        dB = torch.empty_like(B_p)
        dC = torch.empty_like(C_p)
        du = torch.empty_like(u_p)
        dh0 = torch.empty_like(h0)
        ws = _alloc_workspace(batch, length, dim, n, _native.MSS_F32, u_p.device)
        st = lib.mamba_ss_bwd(_stream(u_p.device), 0 if ctx.euler else 1, batch,
                              length, dim, n, _ptr(A), _ptr(d_p), _ptr(B_p),
                              _ptr(C_p), _ptr(u_p), _ptr(h0), _ptr(cs), _ptr(dy_p),
                              _ptr(dfinal), _ptr(dA), _ptr(dd), _ptr(dB), _ptr(dC),
                              _ptr(du), _ptr(dh0), _ptr(ws), ws.numel())
        _native.check(lib, st)
        return (dA, dd.transpose(1, 2), dB.transpose(1, 2), dC.transpose(1, 2),
                du.transpose(1, 2), dh0, None)


def _selective_scan_cuda(A, deltas, Bs, Cs, u, initial_x, use_euler_barB_approx):
    register_cuda_kernel()
    _validate_inputs(A, deltas, Bs, Cs, u, initial_x)
    return _SelectiveScanCuda.apply(A, deltas, Bs, Cs, u, initial_x,
                                    bool(use_euler_barB_approx))


def selective_scan(A, deltas, Bs, Cs, u, initial_x=None, *,
                   use_euler_barB_approx=True, use_cuda=False, remat=False):
    """Run the reference scan or the sm_100a CUDA implementation.

    ``remat`` applies only to the reference formulation: it checkpoints the
    whole scan-and-output computation so the backward recomputes the
    per-step states instead of keeping them (reference :274-299).
    """
    if initial_x is None:
        initial_x = torch.zeros((u.shape[0], u.shape[2], A.shape[1]),
                                dtype=torch.result_type(A, u), device=u.device)
    if use_cuda:
        return _selective_scan_cuda(A, deltas, Bs, Cs, u, initial_x,
                                    use_euler_barB_approx)
    if remat:
        from torch.utils.checkpoint import checkpoint

        return checkpoint(
            lambda *xs: selective_scan_reference(
                *xs, use_euler_barB_approx=use_euler_barB_approx),
            A, deltas, Bs, Cs, u, initial_x, use_reentrant=False)
    return selective_scan_reference(A, deltas, Bs, Cs, u, initial_x,
                                    use_euler_barB_approx=use_euler_barB_approx)
