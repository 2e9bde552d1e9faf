"""Data-parallel plumbing for the selective scan (one process per GPU).

The scan's work partitions by sequence: each rank scans its own slice of the
batch with no exchange in the data path. The only collective is the sum over
ranks of the parameter gradients dA (D, N), dD (D) and ddelta_bias (D),
done as one all-reduce of a flat buffer (NCCL over NVLink on the GPU box,
gloo in the CPU tests). The reference has no distributed code; its
parameters would be reduced by XLA's psum under shard_map.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def batch_shard(global_batch: int, rank: int, world: int) -> slice:
    """Contiguous slice of the batch owned by `rank` (first ranks take the remainder)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} for world size {world}")
    base, extra = divmod(global_batch, world)
    start = rank * base + min(rank, extra)
    return slice(start, start + base + (1 if rank < extra else 0))


def flat_param_grads(dim: int, dstate: int, device=None, dtype=torch.float32):
    """One buffer [dA | dD | ddelta_bias] and its three views, so the kernels
    write straight into what the all-reduce sends."""
    buf = torch.empty(dim * dstate + 2 * dim, device=device, dtype=dtype)
    dA = buf[: dim * dstate].view(dim, dstate)
    dD = buf[dim * dstate: dim * dstate + dim]
    dbias = buf[dim * dstate + dim:]
    return buf, dA, dD, dbias


def allreduce_param_grads(buf: torch.Tensor, group=None, async_op=False):
    """Sum the flat parameter-gradient buffer over ranks, in place."""
    if not dist.is_available() or not dist.is_initialized() or dist.get_world_size(group) == 1:
        return None
    return dist.all_reduce(buf, op=dist.ReduceOp.SUM, group=group, async_op=async_op)
