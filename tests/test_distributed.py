"""Data-parallel host logic on CPU: two gloo ranks each take a batch shard,
compute the parameter gradients of their shard (CPU oracle standing in for
the kernels), sum them with mamba.distributed.allreduce_param_grads, and must
match the gradients of the whole batch."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from mamba.distributed import allreduce_param_grads, batch_shard, flat_param_grads


def test_batch_shard_covers_batch():
    for gb in (1, 5, 8, 16):
        for world in (1, 2, 3, 8):
            parts = [batch_shard(gb, r, world) for r in range(world)]
            idx = [i for p in parts for i in range(gb)[p]]
            assert idx == list(range(gb))
    with pytest.raises(ValueError):
        batch_shard(8, 2, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle import selective_scan_oracle as orc

        x = orc.make_inputs(5, 6, 40, 4, seed=3, initial_state=True)
        sl = batch_shard(5, rank, world)
        sub = {k: (v[sl] if isinstance(v, np.ndarray) and v.shape[0] == 5 and k != "A" else v)
               for k, v in x.items()}
        g = orc.fused_backward(sub["u"], sub["delta"], x["A"], sub["B"], sub["C"], x["D"],
                               sub["z"], x["delta_bias"], True, sub["initial_state"], True,
                               None, dout=sub["dout"])
        buf, dA, dD, dbias = flat_param_grads(6, 4, dtype=torch.float64)
        dA.copy_(torch.from_numpy(g["dA"]))
        dD.copy_(torch.from_numpy(g["dD"]))
        dbias.copy_(torch.from_numpy(g["ddelta_bias"]))
        allreduce_param_grads(buf)
        if rank == 0:
            q.put((dA.numpy().copy(), dD.numpy().copy(), dbias.numpy().copy()))
    finally:
        dist.destroy_process_group()


def test_two_rank_gradient_allreduce_matches_full_batch():
    from oracle import selective_scan_oracle as orc

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    dA, dD, dbias = q.get(timeout=120)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    x = orc.make_inputs(5, 6, 40, 4, seed=3, initial_state=True)
    full = orc.fused_backward(x["u"], x["delta"], x["A"], x["B"], x["C"], x["D"], x["z"],
                              x["delta_bias"], True, x["initial_state"], True, None,
                              dout=x["dout"])
    np.testing.assert_allclose(dA, full["dA"], rtol=1e-12, atol=1e-12)
    np.testing.assert_allclose(dD, full["dD"], rtol=1e-12, atol=1e-12)
    np.testing.assert_allclose(dbias, full["ddelta_bias"], rtol=1e-12, atol=1e-12)


def _rank_channels(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from mamba.distributed import allreduce_bc_grads, channel_shard
        from oracle import selective_scan_oracle as orc

        x = orc.make_inputs(1, 10, 60, 8, seed=4, initial_state=True)
        sl = channel_shard(10, rank, world)
        ch = {"u", "delta", "z", "dout"}
        sub = {k: (v[:, sl] if k in ch else v) for k, v in x.items()}
        g = orc.fused_backward(sub["u"], sub["delta"], x["A"][sl], x["B"], x["C"], x["D"][sl],
                               sub["z"], x["delta_bias"][sl], True, x["initial_state"][:, sl],
                               True, None, dout=sub["dout"])
        dB = torch.from_numpy(g["dB"].copy())
        dC = torch.from_numpy(g["dC"].copy())
        allreduce_bc_grads(dB, dC)
        q.put((rank, dB.numpy(), dC.numpy(), g["dA"], g["du"]))
    finally:
        dist.destroy_process_group()


def test_two_rank_channel_sharding_matches_full_sequence():
    from mamba.distributed import channel_shard
    from oracle import selective_scan_oracle as orc

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_channels, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict((r[0], r[1:]) for r in (q.get(timeout=120), q.get(timeout=120)))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    x = orc.make_inputs(1, 10, 60, 8, seed=4, initial_state=True)
    full = orc.fused_backward(x["u"], x["delta"], x["A"], x["B"], x["C"], x["D"], x["z"],
                              x["delta_bias"], True, x["initial_state"], True, None,
                              dout=x["dout"])
    for r in (0, 1):
        dB, dC, dA, du = res[r]
        np.testing.assert_allclose(dB, full["dB"], rtol=1e-12, atol=1e-12)
        np.testing.assert_allclose(dC, full["dC"], rtol=1e-12, atol=1e-12)
        sl = channel_shard(10, r, 2)
        np.testing.assert_allclose(dA, full["dA"][sl], rtol=1e-12, atol=1e-12)
        np.testing.assert_allclose(du, full["du"][:, sl], rtol=1e-12, atol=1e-12)


def test_token_balanced_shards():
    from mamba.distributed import token_balanced_shards

    rng = np.random.default_rng(0)
    for world in (1, 2, 4, 8):
        lens = rng.integers(512, 4097, 16 * world)
        shards = token_balanced_shards(lens, world)
        assert sorted(i for s in shards for i in s) == list(range(16 * world))
        assert all(len(s) == 16 for s in shards)
        sums = [int(lens[s].sum()) for s in shards]
        assert max(sums) - min(sums) <= lens.max()
    with pytest.raises(ValueError):
        token_balanced_shards([1, 2, 3], 2)
