"""Complex selective scan (S6 with ``complex_ssm=True``) on the B200 kernels.

The reference evaluates this path in pure JAX (mamba/mamba1.py:170-176, 196):
``A`` (D, N), ``B``, ``C`` (B, N, L) and the state are complex, ``delta`` and
``u`` real, and the output is ``Re(C . h) + D u``. ``selective_scan_complex_fn``
adds the fused softplus(delta + bias), padding mask and silu(z) gate of
``selective_scan_fn``. Complex tensors are torch.complex64; their gradients
follow torch's convention (dL/dRe + i dL/dIm; JAX's cotangent is the
conjugate). There is no fallback: without the built library the calls raise.
"""
from __future__ import annotations

import torch

from . import _native
from .selective_scan_cuda import _lib, _ptr, _stream


def complex_chunk_states_elems(batch, length, dim, dstate):
    return int(_lib().mamba_ss_complex_chunk_states_elems(batch, length, dim, dstate))


def complex_bwd_workspace_bytes(batch, length, dim, dstate):
    return int(_lib().mamba_ss_complex_bwd_workspace_bytes(batch, length, dim, dstate))


def _workspace(batch, length, dim, dstate, device):
    nbytes = complex_bwd_workspace_bytes(batch, length, dim, dstate)
    ws = torch.empty(nbytes + 256, dtype=torch.uint8, device=device)
    off = (-ws.data_ptr()) % 256
    return ws[off:off + nbytes]


def _c(t):
    return None if t is None else t.contiguous()


class _ComplexScan(torch.autograd.Function):
    @staticmethod
    def forward(ctx, u, delta, A, B, C, D, z, delta_bias, initial_state, seq_lens,
                delta_softplus, zoh):
        u, delta, A, B, C, D, z, delta_bias, initial_state = map(
            _c, (u, delta, A, B, C, D, z, delta_bias, initial_state))
        batch, dim, length = u.shape
        n = A.shape[1]
        out = torch.empty_like(u)
        pre = torch.empty_like(u) if z is not None else None
        last = torch.empty(batch, dim, n, dtype=torch.complex64, device=u.device)
        cs = torch.empty(complex_chunk_states_elems(batch, length, dim, n), device=u.device)
        lib = _lib()
        st = lib.mamba_ss_complex_fwd(
            _stream(u.device), int(zoh), batch, length, dim, n, _ptr(u), _ptr(delta), _ptr(A),
            _ptr(B), _ptr(C), _ptr(D), _ptr(z), _ptr(delta_bias), int(bool(delta_softplus)),
            _ptr(initial_state), _ptr(seq_lens), _ptr(out), _ptr(pre), _ptr(last), _ptr(cs))
        _native.check(lib, st)
        ctx.save_for_backward(u, delta, A, B, C, D, z, delta_bias, initial_state, seq_lens, cs,
                              pre)
        ctx.flags = (bool(delta_softplus), bool(zoh))
        return out, last

    @staticmethod
    def backward(ctx, dout, dlast):
        u, delta, A, B, C, D, z, delta_bias, initial_state, seq_lens, cs, pre = ctx.saved_tensors
        delta_softplus, zoh = ctx.flags
        batch, dim, length = u.shape
        n = A.shape[1]
        dout = dout.contiguous()
        dlast = dlast.contiguous() if dlast is not None else None
        du, dd = torch.empty_like(u), torch.empty_like(delta)
        dA, dB, dC = torch.empty_like(A), torch.empty_like(B), torch.empty_like(C)
        dD = torch.empty_like(D) if D is not None else None
        dz = torch.empty_like(z) if z is not None else None
        dbias = torch.empty_like(delta_bias) if delta_bias is not None else None
        dh0 = torch.empty_like(initial_state) if initial_state is not None else None
        ws = _workspace(batch, length, dim, n, u.device)
        lib = _lib()
        st = lib.mamba_ss_complex_bwd(
            _stream(u.device), int(zoh), batch, length, dim, n, _ptr(u), _ptr(delta), _ptr(A),
            _ptr(B), _ptr(C), _ptr(D), _ptr(z), _ptr(delta_bias), int(delta_softplus),
            _ptr(initial_state), _ptr(seq_lens), _ptr(cs), _ptr(pre), _ptr(dout), _ptr(dlast),
            _ptr(du), _ptr(dd), _ptr(dA), _ptr(dB), _ptr(dC), _ptr(dD), _ptr(dz), _ptr(dbias),
            _ptr(dh0), _ptr(ws), ws.numel())
        _native.check(lib, st)
        return du, dd, dA, dB, dC, dD, dz, dbias, dh0, None, None, None


def selective_scan_complex_fn(u, delta, A, B, C, D=None, z=None, delta_bias=None,
                              delta_softplus=False, return_last_state=False, *,
                              initial_state=None, use_euler_barB_approx=True, seq_lens=None):
    """out = (Re(C . h) + D u) * silu(z) of the complex scan, (B, D, L) float32.

    A (D, N), B, C (B, N, L) and initial_state (B, D, N) are complex64; u,
    delta, z float32 (B, D, L); D, delta_bias float32 (D,); seq_lens int32 (B,).
    """
    if not u.is_cuda:
        raise ValueError("selective_scan_complex_fn needs CUDA tensors")
    if u.dtype != torch.float32 or delta.dtype != torch.float32:
        raise TypeError("u and delta must be float32")
    for name, t in (("A", A), ("B", B), ("C", C), ("initial_state", initial_state)):
        if t is not None and t.dtype != torch.complex64:
            raise TypeError(f"{name} must be complex64")
    batch, dim, length = u.shape
    n = A.shape[1]
    if A.shape != (dim, n) or B.shape != (batch, n, length) or C.shape != (batch, n, length):
        raise ValueError("A must be (D, N) and B, C (B, N, L)")
    if n not in (1, 2, 4, 8, 16):
        raise ValueError("N must be one of 1, 2, 4, 8, 16")
    out, last = _ComplexScan.apply(u, delta, A, B, C, D, z, delta_bias, initial_state, seq_lens,
                                   delta_softplus, not use_euler_barB_approx)
    return (out, last) if return_last_state else out
