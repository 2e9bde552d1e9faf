"""Multi-GPU plumbing for the selective scan (one process per GPU).

Two partitions of the scan's work:

* batch sharding: each rank scans its own sequences with no exchange in the
  data path; the only collective is the sum over ranks of the parameter
  gradients dA (D, N), dD (D) and ddelta_bias (D), one all-reduce of a flat
  buffer;
* channel sharding, for single long sequences: each rank owns a contiguous
  block of the d_inner channels (every channel's recurrence is independent),
  and B, C are shared; dA, dD and ddelta_bias are per channel and need no
  collective, but dB and dC are sums over all channels, so they are
  all-reduced.

The collectives are NCCL over NVLink on the GPU box and gloo in the CPU
tests. Both exchanges are small (D*N + 2D fp32 for the parameter gradients;
B*N*L per tensor for dB/dC), so launch latency, not bandwidth, sets their
cost: on 8 B200s NCCL's NVLink SHARP (NVLS) all-reduce measured about 2.5 ms
per call for the 110 KB parameter buffer, its ring/tree algorithms a few tens
of microseconds; set NCCL_NVLS_ENABLE=0 before creating the process group
(bench.py does). The reference has no distributed code; under JAX these would be
XLA psums inside shard_map.
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


def channel_shard(dim: int, rank: int, world: int) -> slice:
    """Contiguous block of channels owned by `rank` (same split as batch_shard)."""
    return batch_shard(dim, rank, world)


def token_balanced_shards(lengths, world: int):
    """Assign sequences to ranks, the same count each, balancing valid tokens.

    Right-padded batches cost each rank its valid steps, and every step waits
    for the slowest rank, so a data loader deals sequences out by length:
    sorted longest first, then dealt in a snake order (0, 1, .., w-1, w-1, ..,
    0, 0, 1, ..), which bounds any two ranks' token counts to within one
    sequence's length of each other. Returns one list of sequence indices per
    rank; ``len(lengths)`` must be a multiple of ``world``."""
    n = len(lengths)
    if world <= 0 or n % world:
        raise ValueError(f"{n} sequences do not split evenly over {world} ranks")
    order = sorted(range(n), key=lambda i: (-int(lengths[i]), i))
    shards = [[] for _ in range(world)]
    for k, i in enumerate(order):
        r, lap = k % world, k // world
        shards[r if lap % 2 == 0 else world - 1 - r].append(i)
    return shards


def allreduce_bc_grads(dB: torch.Tensor, dC: torch.Tensor, group=None, async_op=False):
    """Sum dB and dC over the channel shards, in place (one all-reduce each).
    With ``async_op`` the two work handles are returned (wait() on each makes
    the current stream wait for it)."""
    if not dist.is_available() or not dist.is_initialized() or dist.get_world_size(group) == 1:
        return []
    return [dist.all_reduce(t, op=dist.ReduceOp.SUM, group=group, async_op=async_op)
            for t in (dB, dC)]


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
