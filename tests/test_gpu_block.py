"""The Mamba block around the kernels (mamba.block.MambaBlock: GEMMs in the
scan's (B, D, L) layout, the conv1d + SiLU kernel, the fused scan) against a
float64 PyTorch restatement of the reference block (mamba/mamba1.py:301-337):
output and every parameter and input gradient, fp32 within 1e-4 relative to
the largest magnitude (the block chains GEMMs, the conv and the scan)."""
import pytest
import torch

from _block_ref import block_reference
from _helpers import rel_err

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("norm_type", ["layernorm", "rmsnorm"])
@pytest.mark.parametrize("L", [33, 200])
def test_block_matches_reference(norm_type, L):
    from mamba.block import MambaBlock

    torch.backends.cuda.matmul.allow_tf32 = False
    blk = MambaBlock(24, expand=2, d_state=16, norm_type=norm_type, seed=3)
    g = torch.Generator(device="cpu").manual_seed(L)
    x = torch.randn(2, L, 24, generator=g).cuda().requires_grad_(True)
    dout = torch.randn(2, L, 24, generator=g).cuda()
    out = blk(x)
    (out * dout).sum().backward()

    xr = x.detach().double().requires_grad_(True)
    ref_params = {k: v.detach().double().requires_grad_(True) for k, v in blk.named_parameters()}
    ref = block_reference(ref_params, xr, use_norm=blk.use_norm)
    (ref * dout.double()).sum().backward()

    assert rel_err(out.detach().double().cpu().numpy(), ref.detach().cpu().numpy()) < 1e-4
    assert rel_err(x.grad.double().cpu().numpy(), xr.grad.cpu().numpy()) < 1e-4
    for name, p in blk.named_parameters():
        got = p.grad.double().cpu().numpy()
        want = ref_params[name].grad.cpu().numpy()
        assert rel_err(got, want) < 1e-4, (name, rel_err(got, want))


def test_stack_trains_one_step():
    """configs[3]'s model (2 layers, d_model 64, RMSNorm, vocab 16) runs a
    forward + backward + SGD step and lowers the loss on a fixed batch."""
    from mamba.block import MambaStack

    torch.backends.cuda.matmul.allow_tf32 = False
    model = MambaStack(16, 64, 2, seed=1)
    g = torch.Generator(device="cpu").manual_seed(0)
    tokens = torch.randint(1, 15, (8, 64), generator=g).cuda()
    labels = torch.randint(1, 15, (8,), generator=g).cuda()
    opt = torch.optim.SGD(model.parameters(), lr=0.1)
    losses = []
    for _ in range(3):
        opt.zero_grad()
        logits = model(tokens)[:, -1]
        loss = torch.nn.functional.cross_entropy(logits, labels)
        loss.backward()
        opt.step()
        losses.append(loss.item())
    assert all(torch.isfinite(torch.tensor(losses)))
    assert losses[-1] < losses[0]
