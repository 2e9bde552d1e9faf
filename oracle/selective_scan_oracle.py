"""CPU oracle of the Mamba-1 selective scan — TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg may import this module, and only as the checker or the timed CPU
reference. The product (``jax-mambas_b200/``) never calls it.

It restates, in NumPy, the math of the JAX-Mambas reference:

* ``selective_scan_reference`` follows ``mamba/selective_scan_cuda.py:56-90``
  (discretise, fold ``initial_x`` into step 0, associative scan with
  ``compose(l, r) = (r_a*l_a, r_a*l_h + r_h)``, contract with C).
* ``sequential_recurrence`` follows the known-answer loop of
  ``tests/test_selective_scan_cuda.py:35-49``.
* ``fused_forward`` adds the caller-side math of ``S6.__call__`` /
  ``Mamba.__call__`` (``mamba/mamba1.py:162-198, 308, 332``): softplus of
  delta (+ bias), padding mask on delta and u (``mamba1.py:167-168``), the D
  skip and the silu(z) gate, in the (batch, dim, length) layout the kernels use.
* ``fused_backward`` is the analytic adjoint of ``fused_forward`` (the
  reference gets it from ``jax.vjp``, ``mamba/selective_scan_cuda.py:255``);
  the CPU tests pin it against torch.autograd in float64.
* ``causal_conv1d_forward`` / ``causal_conv1d_backward`` restate the conv
  step of ``Mamba.__call__`` (``mamba/mamba1.py:313-329`` with the conv of
  ``mamba1.py:250-255``: mask, causal depthwise flax conv over
  ``cache ++ projed``, silu, mask) and its adjoint; the CPU tests pin them
  against torch's grouped conv1d under autograd in float64.

Parity pinning: the reference ships no golden vectors and JAX is not
installed on this image or on the GPU box, so the reference's own functions
were executed here instead: tests/golden/make_ref_golden.py lifts
``selective_scan_reference`` (``mamba/selective_scan_cuda.py:56-90``) and
``S6.discretize`` / ``S6.binary_operator`` (``mamba/mamba1.py:143-158``) out
of the reference source unmodified and runs them in float64 under a
torch-backed stand-in for ``jax.numpy`` / ``lax.associative_scan``, with
torch.autograd for the vector-Jacobian products. tests/test_ref_golden.py
checks this oracle against those fixtures (tests/golden/ref_*.npz) to 1e-6:
the reference test recipe at six lengths and both discretizations, configs[0]
with the fused layer math, mask-style padding and the complex branch. The
restated known-answer test (associative scan vs sequential recurrence,
``tests/test_selective_scan_cuda.py:22-52``) and autograd cross-checks of the
analytic backward stay in ``tests/test_oracle.py``.
"""
from __future__ import annotations

import numpy as np


# --------------------------------------------------------------------------
# Reference contract: logical layouts u/deltas (B, L, D), Bs/Cs (B, L, N),
# A (D, N), initial_x (B, D, N).
# --------------------------------------------------------------------------
def _associative_scan(a: np.ndarray, h: np.ndarray, axis: int = 1):
    """Inclusive scan of affine maps along ``axis`` (Hillis-Steele doubling).

    Element i after the scan is compose(e_0, ..., e_i) with
    compose(left, right) = (right_a * left_a, right_a * left_h + right_h),
    the operator of ``mamba/selective_scan_cuda.py:83-86``.
    """
    a = np.moveaxis(a, axis, 0).copy()
    h = np.moveaxis(h, axis, 0).copy()
    n = a.shape[0]
    s = 1
    while s < n:
        a_new = a.copy()
        h_new = h.copy()
        a_new[s:] = a[s:] * a[:-s]
        h_new[s:] = a[s:] * h[:-s] + h[s:]
        a, h = a_new, h_new
        s *= 2
    return np.moveaxis(a, 0, axis), np.moveaxis(h, 0, axis)


def discretize(A, deltas, Bs, use_euler_barB_approx=True):
    """a_bar, b_bar of ``mamba/selective_scan_cuda.py:72-79`` (B, L, D, N)."""
    delta_a = np.einsum("bld,dn->bldn", deltas, A)
    a_bars = np.exp(delta_a)
    if use_euler_barB_approx:
        b_bars = np.einsum("bld,bln->bldn", deltas, Bs)
    else:
        b_bars = np.expm1(delta_a) * np.einsum("dn,bln->bldn", np.reciprocal(A), Bs)
    return a_bars, b_bars


def selective_scan_reference(A, deltas, Bs, Cs, u, initial_x=None, *,
                             use_euler_barB_approx=True, dtype=np.float64):
    """Restatement of ``selective_scan_reference`` (selective_scan_cuda.py:56-90)."""
    A, deltas, Bs, Cs, u = (np.asarray(x, dtype=dtype) for x in (A, deltas, Bs, Cs, u))
    if initial_x is None:
        initial_x = np.zeros((u.shape[0], u.shape[2], A.shape[1]), dtype=dtype)
    initial_x = np.asarray(initial_x, dtype=dtype)
    a_bars, b_bars = discretize(A, deltas, Bs, use_euler_barB_approx)
    bu = b_bars * u[..., None]
    bu[:, 0] += a_bars[:, 0] * initial_x
    _, states = _associative_scan(a_bars, bu, axis=1)
    y = np.einsum("bln,bldn->bld", Cs, states)
    return y, states[:, -1]


def sequential_recurrence(A, deltas, Bs, Cs, u, initial_x, *,
                          use_euler_barB_approx=True, dtype=np.float64):
    """The known-answer loop of ``tests/test_selective_scan_cuda.py:35-49``."""
    A, deltas, Bs, Cs, u, initial_x = (
        np.asarray(x, dtype=dtype) for x in (A, deltas, Bs, Cs, u, initial_x))
    a_bars, b_bars = discretize(A, deltas, Bs, use_euler_barB_approx)
    state = initial_x
    outputs = []
    for step in range(u.shape[1]):
        state = a_bars[:, step] * state + b_bars[:, step] * u[:, step, :, None]
        outputs.append(np.einsum("bn,bdn->bd", Cs[:, step], state))
    return np.stack(outputs, axis=1), state


# --------------------------------------------------------------------------
# Fused contract in kernel layout: u, delta, z, out (B, D, L); B, C (B, N, L);
# A (D, N); D, delta_bias (D,); initial_state (B, D, N); seq_lens (B,).
# --------------------------------------------------------------------------
def _softplus(x):
    # jax.nn.softplus(x) == logaddexp(x, 0)
    return np.logaddexp(x, 0.0)


def _sigmoid(x):
    return 1.0 / (1.0 + np.exp(-x))


def _prepare(u, delta, A, B, C, D, z, delta_bias, delta_softplus, seq_lens, dtype):
    f = lambda x: None if x is None else np.asarray(x, dtype=dtype)
    u, delta, A, B, C, D, z, delta_bias = map(f, (u, delta, A, B, C, D, z, delta_bias))
    pre = delta + (delta_bias[None, :, None] if delta_bias is not None else 0.0)
    dlt = _softplus(pre) if delta_softplus else pre
    batch, _, L = u.shape
    if seq_lens is not None:
        mask = (np.arange(L)[None, :] < np.asarray(seq_lens)[:, None]).astype(dtype)
    else:
        mask = np.ones((batch, L), dtype=dtype)
    m = mask[:, None, :]
    return u * m, dlt * m, pre, A, B, C, D, z, mask


def fused_forward(u, delta, A, B, C, D=None, z=None, delta_bias=None,
                  delta_softplus=False, initial_state=None,
                  use_euler_barB_approx=True, seq_lens=None, dtype=np.float64):
    """out, last_state of the fused selective scan (sequential, exact order)."""
    um, dl, _, A, B, C, D, z, mask = _prepare(
        u, delta, A, B, C, D, z, delta_bias, delta_softplus, seq_lens, dtype)
    batch, dim, L = um.shape
    N = A.shape[1]
    h = (np.zeros((batch, dim, N), dtype=dtype) if initial_state is None
         else np.asarray(initial_state, dtype=dtype).copy())
    y = np.empty((batch, dim, L), dtype=dtype)
    for t in range(L):
        dA = dl[:, :, t, None] * A[None]
        a = np.exp(dA)
        if use_euler_barB_approx:
            bbar = dl[:, :, t, None] * B[:, None, :, t]
        else:
            bbar = np.expm1(dA) / A[None] * B[:, None, :, t]
        h = a * h + bbar * um[:, :, t, None]
        y[:, :, t] = np.einsum("bn,bdn->bd", C[:, :, t], h)
    out = y
    if D is not None:
        out = out + D[None, :, None] * um
    if z is not None:
        out = out * (z * _sigmoid(z))
    if seq_lens is not None:
        out = out * mask[:, None, :]
    return out, h


def fused_backward(u, delta, A, B, C, D=None, z=None, delta_bias=None,
                   delta_softplus=False, initial_state=None,
                   use_euler_barB_approx=True, seq_lens=None, dout=None,
                   dlast_state=None, dtype=np.float64):
    """Gradients of ``fused_forward`` w.r.t. every input.

    Returns a dict with du, ddelta, dA, dB, dC, dD, dz, ddelta_bias,
    dinitial_state (None where the input is None).
    """
    um, dl, pre, A, B, C, D, z, mask = _prepare(
        u, delta, A, B, C, D, z, delta_bias, delta_softplus, seq_lens, dtype)
    zero_state = initial_state is None
    batch, dim, L = um.shape
    N = A.shape[1]
    h0 = (np.zeros((batch, dim, N), dtype=dtype) if zero_state
          else np.asarray(initial_state, dtype=dtype))
    dout = np.asarray(dout, dtype=dtype) * mask[:, None, :]
    euler = use_euler_barB_approx

    # forward pass, keeping every state
    hs = np.empty((L + 1, batch, dim, N), dtype=dtype)
    hs[0] = h0
    a_all = np.empty((L, batch, dim, N), dtype=dtype)
    y = np.empty((batch, dim, L), dtype=dtype)
    for t in range(L):
        dA = dl[:, :, t, None] * A[None]
        a = np.exp(dA)
        bbar = (dl[:, :, t, None] * B[:, None, :, t] if euler
                else np.expm1(dA) / A[None] * B[:, None, :, t])
        hs[t + 1] = a * hs[t] + bbar * um[:, :, t, None]
        a_all[t] = a
        y[:, :, t] = np.einsum("bn,bdn->bd", C[:, :, t], hs[t + 1])

    pre_gate = y + (D[None, :, None] * um if D is not None else 0.0)
    if z is not None:
        sg = _sigmoid(z)
        dz = dout * pre_gate * sg * (1.0 + z * (1.0 - sg))
        dy = dout * z * sg
    else:
        dz = None
        dy = dout
    dD = np.einsum("bdl,bdl->d", dy, um) if D is not None else None

    g = (np.zeros((batch, dim, N), dtype=dtype) if dlast_state is None
         else np.asarray(dlast_state, dtype=dtype).copy())
    d_dl = np.zeros((batch, dim, L), dtype=dtype)
    d_um = np.zeros((batch, dim, L), dtype=dtype)
    dA_tot = np.zeros_like(A)
    dB = np.zeros_like(B)
    dC = np.zeros_like(C)
    for t in range(L - 1, -1, -1):
        g = g + dy[:, :, t, None] * C[:, None, :, t]          # dL/dh_t
        dC[:, :, t] = np.einsum("bd,bdn->bn", dy[:, :, t], hs[t + 1])
        a = a_all[t]
        dt = dl[:, :, t, None]
        w = g * a * hs[t]                                      # g a h_{t-1}
        d_dl[:, :, t] += np.einsum("bdn,dn->bd", w, A)
        dA_tot += np.einsum("bdn,bd->dn", w, dl[:, :, t])
        ut = um[:, :, t, None]
        if euler:
            d_dl[:, :, t] += np.einsum("bdn,bn->bd", g, B[:, :, t]) * um[:, :, t]
            d_um[:, :, t] += np.einsum("bdn,bn->bd", g, B[:, :, t]) * dl[:, :, t]
            dB[:, :, t] += np.einsum("bdn,bd->bn", g, dl[:, :, t] * um[:, :, t])
        else:
            em1 = np.expm1(dt * A[None])
            bb = em1 / A[None]
            Bt = B[:, None, :, t]
            d_dl[:, :, t] += np.einsum("bdn->bd", g * a * Bt * ut)
            d_um[:, :, t] += np.einsum("bdn->bd", g * bb * Bt)
            dB[:, :, t] += np.einsum("bdn->bn", g * bb * ut)
            dA_tot += np.einsum("bdn->dn", g * Bt * ut * (dt * a / A[None] - em1 / A[None] ** 2))
        g = g * a                                              # -> dL/dh_{t-1}
    if D is not None:
        d_um += D[None, :, None] * dy
    # masked inputs: the mask multiplies u and the activated delta
    du = d_um * mask[:, None, :]
    d_dl = d_dl * mask[:, None, :]
    ddelta = d_dl * _sigmoid(pre) if delta_softplus else d_dl
    ddelta_bias = ddelta.sum(axis=(0, 2)) if delta_bias is not None else None
    return {
        "du": du,
        "ddelta": ddelta,
        "dA": dA_tot,
        "dB": dB,
        "dC": dC,
        "dD": dD,
        "dz": dz,
        "ddelta_bias": ddelta_bias,
        "dinitial_state": None if zero_state else g,
        "out": (pre_gate * (z * _sigmoid(z)) if z is not None else pre_gate)
               * (mask[:, None, :] if seq_lens is not None else 1.0),
        "last_state": hs[L],
    }


def fused_step(state, u, delta, A, B, C, D=None, z=None, delta_bias=None,
               delta_softplus=False, use_euler_barB_approx=True, dtype=np.float64):
    """One decode step, restating S6.step (mamba/mamba1.py:200-214) plus the
    fused gate: returns (out (B, D), new_state (B, D, N))."""
    f = lambda x: None if x is None else np.asarray(x, dtype=dtype)
    state, u, delta, A, B, C, D, z, delta_bias = map(
        f, (state, u, delta, A, B, C, D, z, delta_bias))
    pre = delta + (delta_bias[None, :] if delta_bias is not None else 0.0)
    dl = _softplus(pre) if delta_softplus else pre
    dA = dl[:, :, None] * A[None]
    a = np.exp(dA)
    if use_euler_barB_approx:
        bbar = dl[:, :, None] * B[:, None, :]
    else:
        bbar = np.expm1(dA) / A[None] * B[:, None, :]
    h = a * state + bbar * u[:, :, None]
    y = np.einsum("bn,bdn->bd", C, h)
    if D is not None:
        y = y + D[None, :] * u
    if z is not None:
        y = y * z * _sigmoid(z)
    return y, h


# --------------------------------------------------------------------------
# Complex SSM (S6 with complex_ssm=True, mamba/mamba1.py:170-176, 196): A, B,
# C and the state complex, delta and u real; y = Re(C . h) + D u. Gradients of
# complex arguments are dL/dRe + i dL/dIm (torch's convention; JAX's
# cotangent is the conjugate).
# --------------------------------------------------------------------------
def complex_fused_forward(u, delta, A, B, C, D=None, z=None, delta_bias=None,
                          delta_softplus=False, initial_state=None,
                          use_euler_barB_approx=True, seq_lens=None):
    """out (real), last_state (complex) of the complex fused scan."""
    um, dl, _, _, _, _, D, z, mask = _prepare(
        u, delta, None, None, None, D, z, delta_bias, delta_softplus, seq_lens, np.float64)
    A = np.asarray(A, dtype=np.complex128)
    B = np.asarray(B, dtype=np.complex128)
    C = np.asarray(C, dtype=np.complex128)
    batch, dim, L = um.shape
    N = A.shape[1]
    h = (np.zeros((batch, dim, N), dtype=np.complex128) if initial_state is None
         else np.asarray(initial_state, dtype=np.complex128).copy())
    y = np.empty((batch, dim, L))
    for t in range(L):
        dA = dl[:, :, t, None] * A[None]
        a = np.exp(dA)
        if use_euler_barB_approx:
            bbar = dl[:, :, t, None] * B[:, None, :, t]
        else:
            bbar = np.expm1(dA) / A[None] * B[:, None, :, t]
        h = a * h + bbar * um[:, :, t, None]
        y[:, :, t] = np.einsum("bn,bdn->bd", C[:, :, t], h).real
    out = y
    if D is not None:
        out = out + D[None, :, None] * um
    if z is not None:
        out = out * (z * _sigmoid(z))
    if seq_lens is not None:
        out = out * mask[:, None, :]
    return out, h


def complex_fused_backward(u, delta, A, B, C, D=None, z=None, delta_bias=None,
                           delta_softplus=False, initial_state=None,
                           use_euler_barB_approx=True, seq_lens=None, dout=None,
                           dlast=None):
    """Analytic adjoint of complex_fused_forward: dict of gradients (complex
    ones as dL/dRe + i dL/dIm). The adjoint state G = dL/dRe h + i dL/dIm h
    obeys G_t = dy_t conj(C_t) + conj(a_{t+1}) G_{t+1}."""
    um, dl, pre, _, _, _, D, z, mask = _prepare(
        u, delta, None, None, None, D, z, delta_bias, delta_softplus, seq_lens, np.float64)
    A = np.asarray(A, dtype=np.complex128)
    B = np.asarray(B, dtype=np.complex128)
    C = np.asarray(C, dtype=np.complex128)
    batch, dim, L = um.shape
    N = A.shape[1]
    m = mask[:, None, :]
    dout = np.asarray(dout, dtype=np.float64)
    h = [None] * (L + 1)
    h[0] = (np.zeros((batch, dim, N), dtype=np.complex128) if initial_state is None
            else np.asarray(initial_state, dtype=np.complex128).copy())
    avals, bvals = [], []
    for t in range(L):
        dA = dl[:, :, t, None] * A[None]
        a = np.exp(dA)
        bb = (dl[:, :, t, None] + 0j) if use_euler_barB_approx else np.expm1(dA) / A[None]
        bvals.append(bb)
        avals.append(a)
        h[t + 1] = a * h[t] + bb * B[:, None, :, t] * um[:, :, t, None]
    y = np.stack([np.einsum("bn,bdn->bd", C[:, :, t], h[t + 1]).real for t in range(L)], axis=2)
    pre_gate = y + (D[None, :, None] * um if D is not None else 0.0)
    if z is not None:
        sz = _sigmoid(z)
        dz = dout * pre_gate * sz * (1.0 + z * (1.0 - sz)) * m
        dy = dout * z * sz * m
    else:
        dz = None
        dy = dout * m
    G = (np.zeros((batch, dim, N), dtype=np.complex128) if dlast is None
         else np.asarray(dlast, dtype=np.complex128).copy())
    du = np.zeros((batch, dim, L))
    ddl = np.zeros((batch, dim, L))
    dA = np.zeros((dim, N), dtype=np.complex128)
    dB = np.zeros((batch, N, L), dtype=np.complex128)
    dC = np.zeros((batch, N, L), dtype=np.complex128)
    for t in range(L - 1, -1, -1):
        if t + 1 < L:
            G = np.conj(avals[t + 1]) * G
        G = G + dy[:, :, t, None] * np.conj(C[:, None, :, t])
        a, bb, hp = avals[t], bvals[t], h[t]
        Bt = B[:, None, :, t]
        ut = um[:, :, t, None]
        dC[:, :, t] = np.einsum("bd,bdn->bn", dy[:, :, t], np.conj(h[t + 1]))
        # b_t u_t = bb B u
        du[:, :, t] = np.sum((G * np.conj(bb * Bt)).real, axis=2)
        dB[:, :, t] = np.einsum("bdn->bn", G * np.conj(bb) * ut)
        ga = G * np.conj(hp)  # dL/da
        Ad = A[None]
        # a = exp(delta A): da/ddelta = A a, da/dA = delta a
        ddl[:, :, t] = np.sum((ga * np.conj(Ad * a)).real, axis=2)
        dA += np.einsum("bdn->dn", ga * np.conj(dl[:, :, t, None] * a))
        if use_euler_barB_approx:
            ddl[:, :, t] += np.sum((G * np.conj(Bt * ut)).real, axis=2)
        else:
            # bb = expm1(delta A) / A: dbb/ddelta = a, dbb/dA = (delta a - bb) / A
            gbb = G * np.conj(Bt * ut)
            ddl[:, :, t] += np.sum((gbb * np.conj(a)).real, axis=2)
            dA += np.einsum("bdn->dn", gbb * np.conj((dl[:, :, t, None] * a - bb) / Ad))
    dh0 = np.conj(avals[0]) * G if L > 0 else G
    du = du + (D[None, :, None] * dy if D is not None else 0.0)
    du = du * m
    ddl = ddl * m
    if delta_softplus:
        ddl = ddl * _sigmoid(pre)
    res = {"du": du, "ddelta": ddl, "dA": dA, "dB": dB, "dC": dC,
           "dD": np.sum(dy * um, axis=(0, 2)) if D is not None else None,
           "dz": dz, "ddelta_bias": np.sum(ddl, axis=(0, 2)) if delta_bias is not None else None,
           "dinitial_state": dh0}
    return res


# --------------------------------------------------------------------------
# Causal depthwise conv1d + SiLU of the Mamba block, (B, D, L) layout.
# --------------------------------------------------------------------------
def _conv_prepare(x, weight, bias, seq_lens, conv_state, dtype):
    x = np.asarray(x, dtype=dtype)
    Bn, Dn, L = x.shape
    K = weight.shape[0]
    mask = np.ones((Bn, 1, L), dtype=dtype)
    if seq_lens is not None:
        mask = (np.arange(L)[None, None, :] < np.asarray(seq_lens)[:, None, None]).astype(dtype)
    prev = (np.zeros((Bn, Dn, K - 1), dtype=dtype) if conv_state is None
            else np.asarray(conv_state, dtype=dtype))
    # projed *= padding_mask; conv input = cache ++ projed (mamba1.py:308-322)
    xc = np.concatenate([prev, x * mask], axis=2)
    w = np.asarray(weight, dtype=dtype)
    pre = np.zeros_like(x) if bias is None else np.broadcast_to(
        np.asarray(bias, dtype=dtype)[None, :, None], x.shape).copy()
    # flax CAUSAL conv: out[t] = sum_k w[k] * in[t - (K-1) + k]
    for k in range(K):
        pre = pre + w[k][None, :, None] * xc[:, :, k:k + L]
    return x, mask, xc, pre


def causal_conv1d_forward(x, weight, bias=None, seq_lens=None, conv_state=None,
                          dtype=np.float64):
    """u = mask * silu(conv(cache ++ mask * x) + bias), the new conv state
    (the last K - 1 conv inputs) and the pre-activation; x (B, D, L), weight
    (K, D) (flax's (K, 1, D) kernel), conv_state (B, D, K - 1)."""
    x, mask, xc, pre = _conv_prepare(x, weight, bias, seq_lens, conv_state, dtype)
    K = weight.shape[0]
    u = pre * _sigmoid(pre) * mask  # silu, then conved *= padding_mask
    final = xc[:, :, xc.shape[2] - (K - 1):]
    return u, final


def causal_conv1d_backward(x, weight, bias, seq_lens, conv_state, du, dtype=np.float64):
    """Adjoint of causal_conv1d_forward for the cotangent du of u:
    (dx, dweight (K, D), dbias (D,), dconv_state (B, D, K - 1))."""
    x, mask, xc, pre = _conv_prepare(x, weight, bias, seq_lens, conv_state, dtype)
    K = weight.shape[0]
    L = x.shape[2]
    s = _sigmoid(pre)
    g = np.asarray(du, dtype=dtype) * mask * s * (1.0 + pre * (1.0 - s))
    w = np.asarray(weight, dtype=dtype)
    dxc = np.zeros_like(xc)
    dweight = np.zeros_like(w)
    for k in range(K):
        dxc[:, :, k:k + L] += w[k][None, :, None] * g
        dweight[k] = np.sum(g * xc[:, :, k:k + L], axis=(0, 2))
    dx = dxc[:, :, K - 1:] * mask
    return dx, dweight, g.sum(axis=(0, 2)), dxc[:, :, :K - 1]


# --------------------------------------------------------------------------
# Seeded inputs with the distributions of the benchmark configurations.
# --------------------------------------------------------------------------
def make_inputs(batch, dim, length, dstate, *, seed=0, with_D=True, with_z=True,
                with_bias=True, delta_softplus=True, initial_state=False,
                valid_lengths=None, dtype=np.float32):
    """Inputs of configs[0]/[1]: u, z ~ N(0,1); delta ~ N(0,1) with
    delta_bias ~ U(-4,-2) and softplus; A[d, n] = -exp(log(n+1)); B, C ~ N(0,1)
    in (B, N, L); D ~ N(0,1). One PCG64 stream per tensor."""
    ss = np.random.SeedSequence(seed)
    rngs = [np.random.Generator(np.random.PCG64(s)) for s in ss.spawn(10)]
    u = rngs[0].standard_normal((batch, dim, length)).astype(dtype)
    delta = rngs[1].standard_normal((batch, dim, length)).astype(dtype)
    A = np.broadcast_to(-np.exp(np.log(np.arange(1, dstate + 1, dtype=np.float64))),
                        (dim, dstate)).astype(np.float32).copy()
    Bm = rngs[2].standard_normal((batch, dstate, length)).astype(dtype)
    Cm = rngs[3].standard_normal((batch, dstate, length)).astype(dtype)
    D = rngs[4].standard_normal(dim).astype(np.float32) if with_D else None
    z = rngs[5].standard_normal((batch, dim, length)).astype(dtype) if with_z else None
    bias = rngs[6].uniform(-4.0, -2.0, dim).astype(np.float32) if with_bias else None
    h0 = (rngs[7].standard_normal((batch, dim, dstate)).astype(np.float32)
          if initial_state else None)
    dout = rngs[8].standard_normal((batch, dim, length)).astype(dtype)
    seq_lens = None
    if valid_lengths is not None:
        lo, hi = valid_lengths
        seq_lens = rngs[9].integers(lo, hi + 1, batch).astype(np.int32)
    return {
        "u": u, "delta": delta, "A": A, "B": Bm, "C": Cm, "D": D, "z": z,
        "delta_bias": bias, "delta_softplus": delta_softplus,
        "initial_state": h0, "seq_lens": seq_lens, "dout": dout,
    }
