"""Plain PyTorch float64 restatement of the reference's Mamba block
(mamba/mamba1.py:301-337 with S6.__call__, mamba1.py:161-198; real, Euler,
no cache) for the block parity test: the same parameters as
mamba.block.MambaBlock, evaluated with the sequential recurrence."""
import torch


def block_reference(P, x, use_norm=True, dtype=torch.float64):
    """P: the block's parameters by name (float64 leaves); x (B, L, d_model)."""
    res = x.to(dtype)
    h = res
    d_model = x.shape[-1]
    if use_norm:
        h = torch.nn.functional.layer_norm(h, (d_model,), P["norm.weight"], P["norm.bias"],
                                           eps=1e-5) if "norm.bias" in P else \
            torch.nn.functional.rms_norm(h, (d_model,), P["norm.weight"], eps=1e-5)
    projed = h @ P["w_main"].t()                       # (B, L, Di)
    skip = torch.nn.functional.silu(h @ P["w_skip"].t())
    K = P["conv_w"].shape[0]
    pad = torch.nn.functional.pad(projed, (0, 0, K - 1, 0))  # causal: K-1 zeros before
    L = projed.shape[1]
    conv = P["conv_b"] + sum(P["conv_w"][k] * pad[:, k:k + L] for k in range(K))
    u = torch.nn.functional.silu(conv)                 # (B, L, Di)
    Bs = u @ P["w_B"].t()
    Cs = u @ P["w_C"].t()
    deltas = torch.nn.functional.softplus(u @ P["w_r"].t() @ P["w_dt"].t() + P["dt_bias"])
    A = -torch.exp(P["A_log"])
    state = torch.zeros(u.shape[0], u.shape[2], A.shape[1], dtype=dtype, device=u.device)
    ys = []
    for t in range(L):
        a = torch.exp(deltas[:, t, :, None] * A[None])
        state = a * state + deltas[:, t, :, None] * Bs[:, t, None, :] * u[:, t, :, None]
        ys.append(torch.einsum("bn,bdn->bd", Cs[:, t], state))
    y = torch.stack(ys, dim=1) + P["D"] * u
    return res + (y * skip) @ P["w_out"].t()
