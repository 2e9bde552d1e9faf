"""Causal depthwise conv1d + bias + SiLU + padding mask on the B200 kernels.

The operation between the input projection and the selective scan in the
reference's ``Mamba.__call__`` (mamba/mamba1.py:313-329)::

    projed *= padding_mask
    conved = silu(nnx.Conv(d_inner, d_inner, kernel_size=k,
                           feature_group_count=d_inner, padding="CAUSAL")
                  (cache ++ projed))[:, -L:] * padding_mask

(the conv is built at mamba1.py:250-255), evaluated here in the scan's
``(B, D, L)`` layout by ``mamba_ss_conv1d_fwd`` / ``mamba_ss_conv1d_bwd``.
``weight`` is flax's ``(k, 1, D)`` kernel squeezed to ``(k, D)``; the conv
state (the reference's cache, ``(B, k-1, D)`` there) is ``(B, D, k-1)``.
There is no fallback: without the built library the calls raise.
"""
from __future__ import annotations

import torch

from . import _native
from .selective_scan_cuda import _io_dtype, _lib, _ptr, _stream


def conv1d_bwd_workspace_bytes(batch, length, dim, kwidth):
    return int(_lib().mamba_ss_conv1d_bwd_workspace_bytes(batch, length, dim, kwidth))


def conv1d_forward_into(x, weight, bias, seq_lens, conv_state, u, final_state=None):
    """Launch the forward on the current stream into given buffers."""
    lib = _lib()
    batch, dim, length = x.shape
    st = lib.mamba_ss_conv1d_fwd(
        _stream(x.device), _io_dtype(x), batch, length, dim, weight.shape[0], _ptr(x),
        _ptr(weight), _ptr(bias), _ptr(seq_lens), _ptr(conv_state), _ptr(u), _ptr(final_state))
    _native.check(lib, st)


def conv1d_backward_into(x, weight, bias, seq_lens, conv_state, du, dx, dweight, dbias,
                         dconv_state, workspace):
    """Launch the backward on the current stream into given buffers."""
    lib = _lib()
    batch, dim, length = x.shape
    st = lib.mamba_ss_conv1d_bwd(
        _stream(x.device), _io_dtype(x), batch, length, dim, weight.shape[0], _ptr(x),
        _ptr(weight), _ptr(bias), _ptr(seq_lens), _ptr(conv_state), _ptr(du), _ptr(dx),
        _ptr(dweight), _ptr(dbias), _ptr(dconv_state), _ptr(workspace),
        0 if workspace is None else workspace.numel())
    _native.check(lib, st)


def _workspace(batch, length, dim, kwidth, device):
    nbytes = conv1d_bwd_workspace_bytes(batch, length, dim, kwidth)
    ws = torch.empty(nbytes + 256, dtype=torch.uint8, device=device)
    off = (-ws.data_ptr()) % 256
    return ws[off:off + nbytes]


def _check(x, weight, bias, seq_lens, conv_state):
    if not x.is_cuda:
        raise ValueError("causal_conv1d_fn needs CUDA tensors")
    if x.ndim != 3:
        raise ValueError("x must have shape (B, D, L)")
    batch, dim, _ = x.shape
    if weight.ndim != 2 or weight.shape[1] != dim or not 1 <= weight.shape[0] <= 4:
        raise ValueError("weight must have shape (k, D) with 1 <= k <= 4")
    if weight.dtype != torch.float32 or (bias is not None and bias.dtype != torch.float32):
        raise TypeError("weight and bias must be float32")
    if bias is not None and bias.shape != (dim,):
        raise ValueError("bias must have shape (D,)")
    if seq_lens is not None and (seq_lens.shape != (batch,) or seq_lens.dtype != torch.int32):
        raise ValueError("seq_lens must be an int32 tensor of shape (B,)")
    k = weight.shape[0]
    if conv_state is not None and conv_state.shape != (batch, dim, k - 1):
        raise ValueError("conv_state must have shape (B, D, k - 1)")


class _CausalConv1d(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, bias, seq_lens, conv_state, return_final_state):
        x, weight = x.contiguous(), weight.contiguous()
        bias = bias.contiguous() if bias is not None else None
        conv_state = conv_state.contiguous() if conv_state is not None else None
        batch, dim, _ = x.shape
        k = weight.shape[0]
        u = torch.empty_like(x)
        final = (torch.empty(batch, dim, k - 1, dtype=x.dtype, device=x.device)
                 if return_final_state else None)
        conv1d_forward_into(x, weight, bias, seq_lens, conv_state, u, final)
        ctx.save_for_backward(x, weight, bias, seq_lens, conv_state)
        if return_final_state:
            ctx.mark_non_differentiable(final)
        return u, final

    @staticmethod
    def backward(ctx, du, dfinal):
        x, weight, bias, seq_lens, conv_state = ctx.saved_tensors
        batch, dim, _ = x.shape
        k = weight.shape[0]
        du = du.contiguous()
        dx = torch.empty_like(x)
        dweight = torch.empty_like(weight)
        dbias = torch.empty_like(bias) if bias is not None else None
        dstate = torch.empty_like(conv_state) if conv_state is not None else None
        conv1d_backward_into(x, weight, bias, seq_lens, conv_state, du, dx, dweight, dbias,
                             dstate, _workspace(batch, x.shape[2], dim, k, x.device))
        return dx, dweight, dbias, None, dstate, None


def causal_conv1d_fn(x, weight, bias=None, seq_lens=None, conv_state=None,
                     return_final_state=False):
    """u = mask * silu(causal depthwise conv(mask * x) + bias), (B, D, L).

    x: (B, D, L) float32 or bfloat16; weight (k, D) and bias (D,) float32;
    seq_lens (B,) int32 masks steps at or past each length; conv_state
    (B, D, k-1) holds the inputs before t = 0. Returns u, or (u, final_state)
    with the last k - 1 masked inputs when return_final_state.
    """
    _check(x, weight, bias, seq_lens, conv_state)
    u, final = _CausalConv1d.apply(x, weight, bias, seq_lens, conv_state, return_final_state)
    return (u, final) if return_final_state else u


def causal_conv1d_update(x, conv_state, weight, bias=None):
    """One decode token (Mamba.step, mamba/mamba1.py:339-355): x (B, D) ->
    u = silu(bias + sum_k weight[k] * (conv_state ++ x)[k]); conv_state
    (B, D, k-1) is shifted in place. Returns u."""
    if x.ndim != 2 or not x.is_cuda:
        raise ValueError("x must be a CUDA tensor of shape (B, D)")
    batch, dim = x.shape
    k = weight.shape[0]
    if weight.shape != (k, dim) or weight.dtype != torch.float32:
        raise ValueError("weight must be float32 of shape (k, D)")
    if k > 1 and (conv_state is None or conv_state.shape != (batch, dim, k - 1)
                  or conv_state.dtype != x.dtype or not conv_state.is_contiguous()):
        raise ValueError("conv_state must be a contiguous (B, D, k - 1) tensor of x's dtype")
    x = x.contiguous()
    u = torch.empty_like(x)
    lib = _lib()
    st = lib.mamba_ss_conv1d_step(_stream(x.device), _io_dtype(x), batch, dim, k, _ptr(x),
                                  _ptr(weight.contiguous()), _ptr(bias), _ptr(conv_state), _ptr(u))
    _native.check(lib, st)
    return u
