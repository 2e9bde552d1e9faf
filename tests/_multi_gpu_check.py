"""Multi-GPU parity check, one process per GPU (run under torch.distributed.run
by tests/test_gpu_multi_gpu.py; NCCL over NVLink).

Every rank builds the same seeded problem and also runs it whole on its own
GPU as the reference. Then:
  * batch sharding: the rank scans its slice of the batch; dA, dD and
    ddelta_bias, summed over the ranks by one NCCL all-reduce of the flat
    buffer (mamba.distributed.allreduce_param_grads), must equal the whole
    batch's; the per-sequence outputs must equal the whole run's slice;
  * channel sharding: the rank scans its block of d_inner channels with the
    shared B and C; dB and dC, summed by all-reduce
    (allreduce_bc_grads), must equal the whole run's; per-channel outputs and
    dA, dD, ddelta_bias must equal the whole run's block.
Tolerance 1e-4 (rtol and atol) for the all-reduced sums (the order of the
float additions differs from one GPU's), 1e-5 for the rest. Rank 0 prints
one line "MULTI_GPU_OK <world>" or raises."""
import os
import sys
from pathlib import Path

import numpy as np
import torch
import torch.distributed as dist

ROOT = Path(__file__).resolve().parents[1]
for p in (ROOT / "jax-mambas_b200", ROOT, ROOT / "tests"):
    sys.path.insert(0, str(p))

from mamba.distributed import (allreduce_bc_grads, allreduce_param_grads, batch_shard,  # noqa
                               channel_shard, flat_param_grads)
from mamba.selective_scan_cuda import selective_scan_fn  # noqa: E402
from oracle import selective_scan_oracle as orc  # noqa: E402

KEYS = ("u", "delta", "A", "B", "C", "D", "z", "delta_bias")


def run(x, dev):
    t = {k: torch.from_numpy(np.ascontiguousarray(x[k])).to(dev).requires_grad_(True)
         for k in KEYS}
    out = selective_scan_fn(t["u"], t["delta"], t["A"], t["B"], t["C"], t["D"], t["z"],
                            t["delta_bias"], True)
    out.backward(torch.from_numpy(np.ascontiguousarray(x["dout"])).to(dev))
    g = {k: t[k].grad for k in KEYS}
    g["out"] = out.detach()
    return g


def close(a, e, tol, name):
    a, e = a.detach().cpu().numpy(), e.detach().cpu().numpy()
    np.testing.assert_allclose(a, e, rtol=tol, atol=tol, err_msg=name)


def main():
    world = int(os.environ["WORLD_SIZE"])
    rank = int(os.environ["RANK"])
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", device_id=dev)
    batch, dim, L, n = 2 * world, 16 * world, 700, 16
    x = orc.make_inputs(batch, dim, L, n, seed=17)
    full = run(x, dev)

    # batch sharding
    sl = batch_shard(batch, rank, world)
    xb = {k: (v[sl] if k in ("u", "delta", "z", "B", "C", "dout") else v) for k, v in x.items()}
    gb = run(xb, dev)
    buf, dA, dD, dbias = flat_param_grads(dim, n, dev)
    dA.copy_(gb["A"])
    dD.copy_(gb["D"])
    dbias.copy_(gb["delta_bias"])
    allreduce_param_grads(buf)
    close(dA, full["A"], 1e-4, "batch: dA")
    close(dD, full["D"], 1e-4, "batch: dD")
    close(dbias, full["delta_bias"], 1e-4, "batch: ddelta_bias")
    for k in ("out", "u", "delta", "z", "B", "C"):
        close(gb[k], full[k][sl], 1e-5, f"batch: {k}")

    # channel sharding
    cs = channel_shard(dim, rank, world)
    xc = dict(x)
    for k in ("u", "delta", "z", "dout"):
        xc[k] = x[k][:, cs]
    for k in ("A", "D", "delta_bias"):
        xc[k] = x[k][cs]
    gc = run(xc, dev)
    dB, dC = gc["B"].contiguous(), gc["C"].contiguous()
    allreduce_bc_grads(dB, dC)
    close(dB, full["B"], 1e-4, "channel: dB")
    close(dC, full["C"], 1e-4, "channel: dC")
    for k in ("out", "u", "delta", "z"):
        close(gc[k], full[k][:, cs], 1e-5, f"channel: {k}")
    for k in ("A", "D", "delta_bias"):
        close(gc[k], full[k][cs], 1e-5, f"channel: d{k}")
    dist.barrier()
    if rank == 0:
        print(f"MULTI_GPU_OK {world}", flush=True)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
