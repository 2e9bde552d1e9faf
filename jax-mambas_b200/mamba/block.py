"""The Mamba block around the selective scan, on the B200 kernels.

Mirrors the reference's ``Mamba`` module (mamba/mamba1.py:217-337) with its
``S6`` (mamba1.py:23-198) for the real, Euler case: norm, input projections,
padding mask, causal depthwise conv + SiLU, the x / dt projections, the
selective scan with the D skip, the silu(skip) gate, the output projection and
the residual. Parameter shapes, initialisation and dt_rank follow the
reference (mamba1.py:9-20, 40-131, 228-283).

Everything between the projections stays in the scan's (B, D, L) layout: the
projections are plain GEMMs (cuBLAS) that read and write that layout through
transposed operands, so no transpose pass runs around the kernels; the conv
(``causal_conv1d_fn``) and the fused scan (``selective_scan_fn``: softplus of
dt_proj + bias, D skip, silu(skip) gate) are the sm_100a kernels.
"""
from __future__ import annotations

import math

import torch
from torch import nn

from .causal_conv1d import causal_conv1d_fn
from .selective_scan_cuda import selective_scan_fn


# The projections are batched GEMMs (torch.bmm -> cuBLAS) against weights
# expanded over the batch with stride 0, so that transposed operands reach
# cuBLAS as transposed views instead of being copied (torch.matmul folds a
# 3-D @ 2-D product into one 2-D GEMM and copies a transposed view first).
def _bw(w, batch):
    return w.expand(batch, *w.shape)


class _ProjIn(torch.autograd.Function):
    """projed, zpre (B, d_inner, L) = W_main x^T, W_skip x^T for x (B, L, d_model);
    the backward writes dx in x's layout (the second product accumulates in the
    GEMM)."""

    @staticmethod
    def forward(ctx, x, w_main, w_skip):
        b = x.shape[0]
        xt = x.transpose(1, 2)
        ctx.save_for_backward(x, w_main, w_skip)
        return torch.bmm(_bw(w_main, b), xt), torch.bmm(_bw(w_skip, b), xt)

    @staticmethod
    def backward(ctx, dp, dz):
        x, w_main, w_skip = ctx.saved_tensors
        b = x.shape[0]
        dx = torch.bmm(dp.transpose(1, 2), _bw(w_main, b))
        dx = torch.baddbmm(dx, dz.transpose(1, 2), _bw(w_skip, b))
        return dx, torch.bmm(dp, x).sum(0), torch.bmm(dz, x).sum(0)


class _ProjX(torch.autograd.Function):
    """x_proj of S6 as one GEMM: (dt_r, B, C) = (W_r, W_B, W_C) u for u
    (B, d_inner, L); B and C come out contiguous (B, N, L), and the backward's
    du is one GEMM."""

    @staticmethod
    def forward(ctx, u, w_x, r, n):
        xp = torch.bmm(_bw(w_x, u.shape[0]), u)
        ctx.save_for_backward(u, w_x)
        ctx.rn = (r, n)
        return xp[:, :r], xp[:, r:r + n].contiguous(), xp[:, r + n:].contiguous()

    @staticmethod
    def backward(ctx, dr, dB, dC):
        u, w_x = ctx.saved_tensors
        dxp = torch.cat([dr, dB, dC], dim=1)
        du = torch.bmm(_bw(w_x.t(), u.shape[0]), dxp)
        return du, torch.bmm(dxp, u.transpose(1, 2)).sum(0), None, None


class _ProjOut(torch.autograd.Function):
    """out (B, L, d_model) = y^T W_out^T for y (B, d_inner, L); the backward
    writes dy in the scan's (B, d_inner, L) layout."""

    @staticmethod
    def forward(ctx, y, w_out):
        ctx.save_for_backward(y, w_out)
        return torch.bmm(y.transpose(1, 2), _bw(w_out.t(), y.shape[0]))

    @staticmethod
    def backward(ctx, dout):
        y, w_out = ctx.saved_tensors
        dt = dout.transpose(1, 2)  # (B, d_model, L) view
        dy = torch.bmm(_bw(w_out.t(), y.shape[0]), dt)
        return dy, torch.bmm(dt, y.transpose(1, 2)).sum(0)


def _uniform(t, bound, gen):
    with torch.no_grad():
        t.uniform_(-bound, bound, generator=gen)
    return t


class MambaBlock(nn.Module):
    """One Mamba-1 block: x (B, L, d_model) -> x + mamba(norm(x)).

    d_inner = expand * d_model; dt_rank "auto" = max(1, ceil(d_model / 16))
    (the reference computes it from d_model, mamba1.py:229-231); norm_type
    "layernorm" or "rmsnorm" (eps 1e-5); dtype float32 or bfloat16 for the
    activations and projection weights (A_log, D and the dt bias stay float32,
    as in the reference, mamba1.py:44-46, 72-73).
    """

    def __init__(self, d_model, expand=2, d_state=16, dt_rank="auto", conv_kernel=4,
                 use_norm=True, norm_type="layernorm", num_layers=1, dtype=torch.float32,
                 device="cuda", seed=0):
        super().__init__()
        g = torch.Generator(device="cpu").manual_seed(seed)
        di = expand * d_model
        r = max(1, (d_model + 15) // 16) if dt_rank == "auto" else int(dt_rank)
        self.d_model, self.d_inner, self.d_state, self.dt_rank = d_model, di, d_state, r
        self.kw = conv_kernel
        f32 = dict(dtype=torch.float32)
        P = lambda *s: nn.Parameter(torch.empty(*s, **f32))
        # projections as (out, in) matrices
        self.w_main = P(di, d_model)
        self.w_skip = P(di, d_model)
        _uniform(self.w_main, d_model ** -0.5, g)
        _uniform(self.w_skip, d_model ** -0.5, g)
        self.conv_w = P(conv_kernel, di)  # flax's (k, 1, d_inner) kernel
        self.conv_b = P(di)
        _uniform(self.conv_w, conv_kernel ** -0.5, g)
        _uniform(self.conv_b, conv_kernel ** -0.5, g)
        self.w_r = P(r, di)
        self.w_B = P(d_state, di)
        self.w_C = P(d_state, di)
        for w in (self.w_r, self.w_B, self.w_C):
            _uniform(w, di ** -0.5, g)
        self.w_dt = P(di, r)
        _uniform(self.w_dt, r ** -0.5, g)
        # dt bias: inverse softplus of dt ~ exp(U(log 1e-3, log 1e-1)), dt >= 1e-4
        dt = torch.exp(torch.empty(di, **f32).uniform_(math.log(1e-3), math.log(1e-1), generator=g))
        dt = dt.clamp(min=1e-4)
        self.dt_bias = nn.Parameter(dt + torch.log(-torch.expm1(-dt)))
        # A = -exp(A_log), A_log = log(n + 1) (the stability trick, mamba1.py:40-46)
        self.A_log = nn.Parameter(torch.log(torch.arange(1, d_state + 1, **f32)).repeat(di, 1))
        self.D = nn.Parameter(torch.ones(di, **f32))
        self.w_out = P(d_model, di)
        _uniform(self.w_out, di ** -0.5 * num_layers ** -0.5, g)
        self.use_norm = use_norm
        if use_norm:
            self.norm = (nn.LayerNorm(d_model, eps=1e-5) if norm_type == "layernorm"
                         else nn.RMSNorm(d_model, eps=1e-5))
        self.act_dtype = dtype
        self.to(device)

    def forward(self, x, seq_lens=None):
        """x (B, L, d_model); seq_lens (B,) int32 for right padding (the
        reference's padding_mask for that case: mamba1.py:309-311, 328-329)."""
        res = x
        dt = self.act_dtype
        if self.use_norm:
            x = self.norm(x.float()).to(dt)
        projed, zpre = _ProjIn.apply(x.to(dt), self.w_main.to(dt),
                                     self.w_skip.to(dt))   # (B, d_inner, L)
        # mask * silu(conv(mask * projed)) (the conv masks by seq_lens)
        u = causal_conv1d_fn(projed, self.conv_w, self.conv_b, seq_lens)
        w_x = torch.cat([self.w_r, self.w_B, self.w_C], dim=0).to(dt)
        dtr, Bm, Cm = _ProjX.apply(u, w_x, self.dt_rank, self.d_state)  # (B, r / N / N, L)
        delta = torch.bmm(_bw(self.w_dt.to(dt), u.shape[0]), dtr)  # (B, d_inner, L); bias in the scan
        A = -torch.exp(self.A_log)
        y = selective_scan_fn(u, delta, A, Bm, Cm, self.D, zpre, self.dt_bias, True,
                              seq_lens=seq_lens)             # (scan + D u) * silu(skip)
        out = _ProjOut.apply(y, self.w_out.to(dt))         # (B, L, d_model)
        return res + out.to(res.dtype)


class MambaStack(nn.Module):
    """Embedding, n MambaBlocks, final norm and an output head: the model of
    the reference's induction-heads experiment (configs[3]: 2 layers,
    d_model 64, expand 2, d_state 16, conv 4, RMSNorm, vocab 16)."""

    def __init__(self, vocab, d_model, n_layers, norm_type="rmsnorm", dtype=torch.float32,
                 device="cuda", seed=0, **kw):
        super().__init__()
        g = torch.Generator(device="cpu").manual_seed(seed)
        self.embed = nn.Parameter(torch.randn(vocab, d_model, generator=g) * d_model ** -0.5)
        self.layers = nn.ModuleList(
            MambaBlock(d_model, norm_type=norm_type, num_layers=n_layers, dtype=dtype,
                       device=device, seed=seed + 1 + i, **kw) for i in range(n_layers))
        self.norm = nn.RMSNorm(d_model, eps=1e-5) if norm_type == "rmsnorm" else \
            nn.LayerNorm(d_model, eps=1e-5)
        self.head = nn.Parameter(torch.randn(vocab, d_model, generator=g) * d_model ** -0.5)
        self.to(device)

    def forward(self, tokens, seq_lens=None):
        x = self.embed[tokens]
        for layer in self.layers:
            x = layer(x, seq_lens)
        return self.norm(x) @ self.head.t()
