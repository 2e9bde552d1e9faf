"""Selective-scan fwd+bwd throughput on B200 (B*D*L Gelem/s) — the metric of
BASELINE.json.

Default workload: configs[1] — B=8, D=1536, L=2048, N=16, fp32, fused
softplus(delta + bias), D skip and silu(z) gate, dy ~ N(0,1). One step = one
forward + one backward of the fused selective scan over one batch (plus, for
N>1 GPUs, the all-reduce of dA, dD and ddelta_bias across ranks: the batch is
sharded, each rank holds a full configs[1] batch, i.e. weak scaling).
``--config c2`` runs configs[2] (bf16 I/O, B=16, D=5120, L=4096, right-padded
valid lengths ~ U[512, 4096]).

``--impl reference`` times the reference's CPU path instead: JAX is not
installed on this image, so it runs the NumPy restatement of the reference's
math from oracle/ (forward + analytic backward) on all host cores, on a
bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "jax-mambas_b200"))
sys.path.insert(0, str(ROOT))

METRIC = "selective-scan fwd+bwd B*D*L elements/s"
UNIT = "Gelem/s"

CONFIGS = {
    "c1": dict(workload="configs[1]: fused selective scan fwd+bwd, Mamba-130M layer shape",
               batch=8, dim=1536, length=2048, dstate=16, dtype="f32", padded=False),
    "c2": dict(workload="configs[2]: fused selective scan fwd+bwd, Mamba-2.8B layer shape, "
                        "bf16 I/O, right padding",
               batch=16, dim=5120, length=4096, dstate=16, dtype="bf16", padded=True),
    "c4": dict(workload="configs[4] single-sequence variant: one Mamba-2.8B layer's scan, "
                        "B=1, L=131072, d_inner 5120 sharded over the GPUs (channel sharding)",
               batch=1, dim=5120, length=131072, dstate=16, dtype="bf16", padded=False,
               shard="channels"),
}


def _peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        j = json.loads(p.read_text())
        return float(j["hbm_gbs"]), float(j.get("sm_max_mhz", 1965.0)), "measured"
    return 6650.0, 1965.0, "fallback"


# ---------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "25", "-f", self.path],
                stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if self.proc is None or not self.path or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = []
        for line in Path(self.path).read_text().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append((float(parts[1]), float(parts[2]), float(parts[3]), parts[5:9]))
            except ValueError:
                continue
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        loaded = [r for r in rows if r[2] > 250.0] or rows
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in loaded for i, v in enumerate(r[3])
                          if v.lower() == "active"})
        return {"sm_mhz": statistics.median(r[0] for r in loaded),
                "sm_max_mhz": max(r[1] for r in rows), "samples": len(loaded),
                "reasons": reasons}


# ---------------------------------------------------------------- GPU arm
def _algorithmic(cfg, esize, d=None):
    b, L, n = cfg["batch"], cfg["length"], cfg["dstate"]
    d = cfg["dim"] if d is None else d
    elems = b * d * L
    bnl = b * n * L
    nch = math.ceil(L / 4)  # saved carries per row (one per 4 steps)
    # Algorithmic bytes (the minimum I/O of the fused op): forward u, delta,
    # z, B, C in, out and the pre-gate out (kept for dz) out; backward u,
    # delta, z, dy, pre-gate, B, C in, du, ddelta, dz, dB, dC out. The saved
    # carries (fp32 state every 4 steps, written by the forward and read by
    # the backward) are this design's own extra traffic, reported apart.
    fwd = elems * 5 * esize + 2 * bnl * esize
    bwd = elems * 8 * esize + 4 * bnl * esize
    carry = b * d * nch * n * 4
    # special-function-unit ops per element: N ex2 per pass, plus softplus
    # (exp, reciprocal) and sigmoid(z) (exp, reciprocal) in both kernels and
    # the softplus derivative (exp) in the backward
    mufu_fwd = n + 4
    mufu_bwd = n + 5
    return elems, fwd, bwd, carry, mufu_fwd, mufu_bwd


class _stdout_to_stderr:
    """Points file descriptor 1 at stderr for the duration of the block."""

    def __enter__(self):
        sys.stdout.flush()
        self._saved = os.dup(1)
        os.dup2(2, 1)

    def __exit__(self, *exc):
        sys.stdout.flush()
        os.dup2(self._saved, 1)
        os.close(self._saved)


def run_gpu(args, cfg):
    import torch
    import torch.distributed as dist

    from mamba import selective_scan_cuda as ssc
    from mamba.distributed import (allreduce_bc_grads, allreduce_param_grads, channel_shard,
                                   flat_param_grads)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        # NCCL prints its version banner on stdout when the communicator is
        # created; keep stdout for the one JSON line
        with _stdout_to_stderr():
            dist.init_process_group("nccl", device_id=dev)
            dist.barrier()

    b, d, L, n = cfg["batch"], cfg["dim"], cfg["length"], cfg["dstate"]
    chan = cfg.get("shard") == "channels"
    d_total = d
    if chan:  # this rank's block of channels; B and C are shared
        sl = channel_shard(d, rank, world)
        d = sl.stop - sl.start
    io = torch.bfloat16 if cfg["dtype"] == "bf16" else torch.float32
    esize = 2 if io == torch.bfloat16 else 4
    g = torch.Generator(device=dev)
    g.manual_seed(1234 + rank)

    def normal(*shape):
        return torch.randn(*shape, generator=g, device=dev, dtype=torch.float32).to(io)

    u, delta, z, dout = normal(b, d, L), normal(b, d, L), normal(b, d, L), normal(b, d, L)
    Bm, Cm = normal(b, n, L), normal(b, n, L)
    A = (-torch.arange(1, n + 1, device=dev, dtype=torch.float32)).expand(d, n).contiguous()
    Dp = torch.randn(d, generator=g, device=dev)
    bias = torch.rand(d, generator=g, device=dev) * 2.0 - 4.0
    seq_lens = None
    if cfg["padded"]:
        seq_lens = torch.randint(512, L + 1, (b,), generator=g, device=dev, dtype=torch.int32)
        t_idx = torch.arange(L, device=dev)
        m = (t_idx[None, :] < seq_lens[:, None].long())[:, None, :]
        delta.masked_fill_(~m, 0)
        u.masked_fill_(~m, 0)

    out = torch.empty_like(u)
    pre = torch.empty_like(u)
    last = torch.empty(b, d, n, device=dev)
    cs = torch.empty(ssc.chunk_states_elems(b, L, d, n), device=dev)
    du, ddl, dz = torch.empty_like(u), torch.empty_like(u), torch.empty_like(u)
    dB, dC = torch.empty_like(Bm), torch.empty_like(Cm)
    params, dA, dDp, dbias = flat_param_grads(d, n, dev)  # one all-reduce buffer
    ws = ssc._alloc_workspace(b, L, d, n, 1 if io == torch.bfloat16 else 0, dev)
    stream = torch.cuda.current_stream(dev)

    def fwd():
        ssc.fused_forward_into(u, delta, A, Bm, Cm, Dp, z, bias, True, None, seq_lens,
                               out, last, cs, out_pre=pre)

    def bwd():
        ssc.fused_backward_into(u, delta, A, Bm, Cm, Dp, z, bias, True, None, seq_lens, cs,
                                dout, None, du, ddl, dA, dB, dC, dDp, dz, dbias, None, ws,
                                out_pre=pre)

    def exchange():
        if chan:
            allreduce_bc_grads(dB, dC)  # dB, dC sum over every channel
        else:
            allreduce_param_grads(params)  # dA, dD, ddelta_bias sum over sequences

    def step():
        fwd()
        bwd()
        exchange()

    for _ in range(max(args.warmup, 0)):
        step()
    torch.cuda.synchronize()

    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    sampler = ClockSampler(local)
    with sampler:
        t_start = torch.cuda.Event(enable_timing=True)
        t_end = torch.cuda.Event(enable_timing=True)
        t_start.record(stream)
        for i in range(args.steps):
            ev[i][0].record(stream)
            fwd()
            ev[i][1].record(stream)
            bwd()
            ev[i][2].record(stream)
            exchange()
        t_end.record(stream)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
    total_ms = t_start.elapsed_time(t_end)
    fwd_ms = statistics.mean(e[0].elapsed_time(e[1]) for e in ev)
    bwd_ms = statistics.mean(e[1].elapsed_time(e[2]) for e in ev)
    clocks = sampler.summary()

    if world > 1:
        t = torch.tensor([total_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms = float(t.item())

    elems, fwd_bytes, bwd_bytes, carry_bytes, mufu_f, mufu_b = _algorithmic(cfg, esize, d)
    # padded steps are skipped by the kernels: the rooflines count
    # the valid steps only, the headline value counts every B*D*L position
    valid = 1.0
    if seq_lens is not None:
        valid = float(seq_lens.sum().item()) / (b * L)
    fwd_bytes, bwd_bytes, carry_bytes = fwd_bytes * valid, bwd_bytes * valid, carry_bytes * valid
    ms_per_step = total_ms / args.steps
    total_elems = b * d_total * L if chan else elems * world
    value = total_elems / (ms_per_step * 1e-3) / 1e9

    # ---- e2e through the public API with host buffers
    e2e = run_e2e(args, cfg, dev, io, rank, world) if args.e2e and not chan else None

    if rank != 0:
        if world > 1:
            dist.destroy_process_group()
        return None

    hbm, sm_max, peak_src = _peaks()
    bwd_gbs = bwd_bytes / (bwd_ms * 1e-3) / 1e9
    fwd_gbs = fwd_bytes / (fwd_ms * 1e-3) / 1e9
    f_mhz = clocks.get("sm_mhz") or sm_max
    mufu_peak = 148 * 16 * f_mhz * 1e6  # ops/s: 16 MUFU lanes per SM per clock
    mufu_bwd = elems * valid * mufu_b / (bwd_ms * 1e-3)
    mufu_fwd = elems * valid * mufu_f / (fwd_ms * 1e-3)
    traffic = args.traffic
    if traffic is None and args.config == "c1" and not args.batch:
        tf = ROOT / "profiles" / "ncu_traffic.json"
        if tf.exists():
            traffic = json.loads(tf.read_text()).get("c1", {}).get("ss_bwd_tile_kernel")
    res = {
        "metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4),
        "higher_is_better": True, "scaling": "strong" if chan else "weak", "vs_baseline": None,
        "dtype": cfg["dtype"], "data": "synthetic (seeded N(0,1)/U(-4,-2) inputs of the config)",
        "config": {"workload": cfg["workload"], "batch_per_gpu": b, "dim": d_total, "dim_per_gpu": d, "length": L,
                   "dstate": n, "global_batch": b * world,
                   "parallelism": (f"channel-sharded over {world} GPUs ({d} channels each)" if chan
                                   else f"batch-sharded dp{world}") if world > 1 else "single GPU",
                   "l2": "inputs larger than L2 (u, delta, z, dy: "
                         f"{elems * esize * 4 / 1e6:.0f} MB per step)",
                   "valid_fraction": round(valid, 4)},
        "kernels_ms": {"fwd": round(fwd_ms, 4), "bwd": round(bwd_ms, 4)},
        "roofline": {"bound": "hbm", "kernel": "ss_bwd_tile_kernel",
                     "achieved": round(bwd_gbs, 1), "peak": hbm, "unit": "GB/s",
                     "frac": round(bwd_gbs / hbm, 4), "traffic": traffic,
                     "peak_source": f"{peak_src} (MEASURED_PEAKS.json hbm_gbs)"
                     if peak_src == "measured" else "fallback 6.65 TB/s",
                     "algorithmic_bytes_per_launch": bwd_bytes,
                     "carry_bytes_per_launch": carry_bytes},
        "roofline_fwd": {"bound": "hbm", "kernel": "ss_fwd_kernel", "achieved": round(fwd_gbs, 1),
                         "peak": hbm, "unit": "GB/s", "frac": round(fwd_gbs / hbm, 4)},
        "roofline_sfu": {"bound": "sfu", "unit": "MUFU op/s",
                         "peak": mufu_peak, "clock_mhz": f_mhz,
                         "bwd_frac": round(mufu_bwd / mufu_peak, 4),
                         "fwd_frac": round(mufu_fwd / mufu_peak, 4),
                         "ops_per_elem": {"fwd": mufu_f, "bwd": mufu_b}},
        "clocks": clocks,
        "gpu_launches": args.steps * (3 if io == torch.float32 else 5),
    }
    if e2e is not None:
        res["e2e"] = e2e
    if args.cpu_baseline and world == 1:
        res["cpu_baseline"] = cpu_baseline(cfg, args.cpu_seconds)
    print(json.dumps(res), flush=True)
    if world > 1:
        dist.destroy_process_group()
    return res


def run_e2e(args, cfg, dev, io, rank, world):
    """Same metric through the public host-buffer API: pinned host inputs
    copied in and every result copied out, each step, by
    mamba.host_pipeline.HostScanPipeline (copy-in, kernels and copy-out of
    batch chunks overlapped on three streams). The unpipelined call
    (selective_scan_fn + autograd around whole-batch copies) is timed beside
    it and reported as ``autograd_value``."""
    import torch
    import torch.distributed as dist

    from mamba.host_pipeline import HostScanPipeline, alloc_host_outputs
    from mamba.selective_scan_cuda import selective_scan_fn

    b, d, L, n = cfg["batch"], cfg["dim"], cfg["length"], cfg["dstate"]
    g = torch.Generator()
    g.manual_seed(99 + rank)

    def host(*shape):
        return torch.randn(*shape, generator=g).to(io).pin_memory()

    h = {"u": host(b, d, L), "delta": host(b, d, L), "z": host(b, d, L),
         "dout": host(b, d, L), "B": host(b, n, L), "C": host(b, n, L)}
    h["A"] = (-torch.arange(1, n + 1, dtype=torch.float32)).expand(d, n).contiguous().pin_memory()
    h["D"] = torch.randn(d, generator=g).pin_memory()
    h["delta_bias"] = (torch.rand(d, generator=g) * 2 - 4).pin_memory()
    if cfg["padded"]:
        h["seq_lens"] = torch.randint(512, L + 1, (b,), generator=g,
                                      dtype=torch.int32).pin_memory()
    outs = alloc_host_outputs(b, d, L, n, io)
    h2d = sum(t.numel() * t.element_size() for t in h.values())
    d2h = sum(t.numel() * t.element_size() for t in outs.values())

    pipe = HostScanPipeline(b, d, L, n, io, device=dev)
    reduce = (lambda flat: dist.all_reduce(flat)) if world > 1 else None

    def step():
        pipe.run(h, outs, delta_softplus=True, reduce_params=reduce)

    def step_autograd():
        t = {k: h[k].to(dev, non_blocking=True) for k in ("u", "delta", "z", "dout", "B", "C")}
        A = h["A"].to(dev, non_blocking=True).requires_grad_(True)
        Dp = h["D"].to(dev, non_blocking=True).requires_grad_(True)
        bias = h["delta_bias"].to(dev, non_blocking=True).requires_grad_(True)
        seq = h["seq_lens"].to(dev, non_blocking=True) if "seq_lens" in h else None
        for k in ("u", "delta", "z", "B", "C"):
            t[k].requires_grad_(True)
        out = selective_scan_fn(t["u"], t["delta"], A, t["B"], t["C"], Dp, t["z"], bias,
                                delta_softplus=True, seq_lens=seq)
        out.backward(t["dout"])
        if world > 1:
            flat = torch.cat([A.grad.flatten(), Dp.grad, bias.grad])
            dist.all_reduce(flat)
        outs["out"].copy_(out.detach(), non_blocking=True)
        for k, src in (("du", "u"), ("ddelta", "delta"), ("dz", "z"), ("dB", "B"), ("dC", "C")):
            outs[k].copy_(t[src].grad, non_blocking=True)
        outs["dA"].copy_(A.grad, non_blocking=True)
        outs["dD"].copy_(Dp.grad, non_blocking=True)
        outs["ddelta_bias"].copy_(bias.grad, non_blocking=True)

    def timed(fn):
        for _ in range(max(1, min(args.warmup, 3))):
            fn()
        torch.cuda.synchronize()
        k = max(1, min(args.steps, 10))
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        if world > 1:
            dist.barrier()
        s.record()
        for _ in range(k):
            fn()
        e.record()
        torch.cuda.synchronize()
        ms = s.elapsed_time(e) / k
        if world > 1:
            t = torch.tensor([ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms, k

    ms_a, _ = timed(step_autograd)
    ms, k = timed(step)
    value = b * d * L * world / (ms * 1e-3) / 1e9
    return {"value": round(value, 3), "unit": UNIT, "ms_per_step": round(ms, 3),
            "steps": k, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "api": "mamba.host_pipeline.HostScanPipeline.run (pinned host buffers; "
                   "batch chunks copied in, scanned fwd+bwd and copied out on three streams)",
            "chunk_batch": pipe.chunk,
            "autograd_value": round(b * d * L * world / (ms_a * 1e-3) / 1e9, 3),
            "autograd_api": "selective_scan_fn + autograd backward around whole-batch copies"}


# ---------------------------------------------------------------- decode step
def run_step_bench(args):
    """--config step: one recurrent decode step (S6.step) of a Mamba-2.8B layer
    for a batch of 32 sequences: bf16 token inputs, fp32 state updated in
    place. HBM-bound; reported as channel-updates/s and GB/s of state +
    token traffic against the measured copy bandwidth."""
    import torch

    from mamba.selective_scan_cuda import fused_step_into

    dev = torch.device("cuda", 0)
    b, d, n = 32, 5120, 16
    g = torch.Generator(device=dev)
    g.manual_seed(7)
    bf = torch.bfloat16
    # several independent states, cycled, so that state traffic exceeds L2
    copies = 16
    states = [torch.randn(b, d, n, generator=g, device=dev) for _ in range(copies)]
    u, dl, z = (torch.randn(b, d, generator=g, device=dev).to(bf) for _ in range(3))
    Bm, Cm = (torch.randn(b, n, generator=g, device=dev).to(bf) for _ in range(2))
    A = (-torch.arange(1, n + 1, device=dev, dtype=torch.float32)).expand(d, n).contiguous()
    Dp = torch.randn(d, generator=g, device=dev)
    bias = torch.rand(d, generator=g, device=dev) * 2 - 4
    out = torch.empty_like(u)
    steps = max(args.steps, 64) // copies * copies

    def launch_all():
        for i in range(steps):
            fused_step_into(states[i % copies], u, dl, A, Bm, Cm, Dp, z, bias, True, out)

    # decode is launch-bound from Python: capture the steps in a CUDA graph
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        launch_all()  # warm-up outside the graph
    torch.cuda.current_stream(dev).wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        launch_all()
    for _ in range(max(args.warmup, 3)):
        graph.replay()
    torch.cuda.synchronize()
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s0.record()
    graph.replay()
    s1.record()
    torch.cuda.synchronize()
    ms = s0.elapsed_time(s1) / steps
    nbytes = b * d * n * 4 * 2 + b * d * 2 * 4 + 2 * b * n * 2 + d * n * 4 + 2 * d * 4
    hbm, _, src = _peaks()
    gbs = nbytes / (ms * 1e-3) / 1e9
    print(json.dumps({
        "metric": "selective-state-update (decode step) channel updates/s", "unit": "Gupd/s",
        "value": round(b * d / (ms * 1e-3) / 1e9, 3), "ms_per_step": round(ms, 5),
        "steps": steps, "higher_is_better": True, "dtype": "bf16 I/O, fp32 state",
        "data": "synthetic", "n_gpus": 1,
        "config": {"workload": "one decode token of a Mamba-2.8B layer (S6.step), "
                               "steps replayed from a CUDA graph", "batch": b,
                   "dim": d, "dstate": n, "l2": f"{copies} states cycled ({copies * b * d * n * 4 / 1e6:.0f} MB)"},
        "roofline": {"bound": "hbm", "kernel": "ss_step_kernel", "achieved": round(gbs, 1),
                     "peak": hbm, "unit": "GB/s", "frac": round(gbs / hbm, 4),
                     "peak_source": src, "algorithmic_bytes_per_launch": nbytes},
        "gpu_launches": steps}), flush=True)


def run_conv_bench(args):
    """--config conv: the Mamba block's causal conv1d + SiLU (kernel width 4)
    forward + backward at the configs[1] shape (B=8, D=1536, L=2048, fp32),
    one step = mamba_ss_conv1d_fwd + mamba_ss_conv1d_bwd. HBM-bound:
    algorithmic bytes per element are x read + u written (forward) and x, du
    read + dx written (backward), 20 B in fp32."""
    import torch

    from mamba.causal_conv1d import _workspace, conv1d_backward_into, conv1d_forward_into

    dev = torch.device("cuda", 0)
    b, d, L, k = 8, 1536, 2048, 4
    g = torch.Generator(device=dev)
    g.manual_seed(11)
    x = torch.randn(b, d, L, generator=g, device=dev)
    du = torch.randn(b, d, L, generator=g, device=dev)
    w = torch.randn(k, d, generator=g, device=dev) * 0.5
    bias = torch.randn(d, generator=g, device=dev)
    u, dx = torch.empty_like(x), torch.empty_like(x)
    dw, db = torch.empty_like(w), torch.empty_like(bias)
    ws = _workspace(b, L, d, k, dev)

    def step():
        conv1d_forward_into(x, w, bias, None, None, u)
        conv1d_backward_into(x, w, bias, None, None, du, dx, dw, db, None, ws)

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    sampler = ClockSampler(0)
    with sampler:
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record()
        for _ in range(args.steps):
            step()
        s1.record()
        torch.cuda.synchronize()
    ms = s0.elapsed_time(s1) / args.steps
    elems = b * d * L
    nbytes = elems * 4 * 5
    hbm, _, src = _peaks()
    gbs = nbytes / (ms * 1e-3) / 1e9
    print(json.dumps({
        "metric": "causal conv1d + SiLU fwd+bwd B*D*L elements/s", "unit": "Gelem/s",
        "value": round(elems / (ms * 1e-3) / 1e9, 3), "ms_per_step": round(ms, 4),
        "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "n_gpus": 1,
        "config": {"workload": "Mamba block conv step (kernel width 4) at the Mamba-130M "
                               "layer shape", "batch": b, "dim": d, "length": L, "kwidth": k,
                   "l2": f"inputs larger than L2 ({elems * 4 * 2 / 1e6:.0f} MB read per step)"},
        "roofline": {"bound": "hbm", "kernel": "ss_conv_fwd_kernel + ss_conv_bwd_kernel",
                     "achieved": round(gbs, 1), "peak": hbm, "unit": "GB/s",
                     "frac": round(gbs / hbm, 4), "peak_source": src,
                     "algorithmic_bytes_per_step": nbytes},
        "clocks": sampler.summary(),
        "gpu_launches": args.steps * 3}), flush=True)


def run_complex_bench(args):
    """--config complex: the complex SSM (complex_ssm=True) fused scan forward +
    backward at the configs[1] shape (B=8, D=1536, L=2048, N=16), fp32 real
    tensors and complex64 A, B, C. Reported like the real scan (B*D*L
    elements/s) with the SFU roofline: per state-step the forward evaluates
    exp and sin/cos of delta A, the backward recomputes them."""
    import torch

    from mamba.selective_scan_complex import selective_scan_complex_fn

    dev = torch.device("cuda", 0)
    b, d, L, n = 8, 1536, 2048, 16
    g = torch.Generator(device=dev)
    g.manual_seed(5)
    rnd = lambda *s: torch.randn(*s, generator=g, device=dev)
    u, dl, z, dout = (rnd(b, d, L) for _ in range(4))
    A = torch.complex(-0.5 * torch.ones(d, n, device=dev),
                      torch.arange(n, device=dev, dtype=torch.float32).expand(d, n).contiguous())
    B = torch.complex(rnd(b, n, L), rnd(b, n, L))
    C = torch.complex(rnd(b, n, L), rnd(b, n, L))
    Dp, bias = rnd(d), torch.rand(d, generator=g, device=dev) * 2 - 4
    leaves = [t.requires_grad_(True) for t in (u, dl, A, B, C, Dp, z, bias)]

    def step():
        for t in leaves:
            t.grad = None
        out = selective_scan_complex_fn(u, dl, A, B, C, Dp, z, bias, True)
        out.backward(dout)

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    steps = max(1, min(args.steps, 20))
    sampler = ClockSampler(0)
    with sampler:
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record()
        for _ in range(steps):
            step()
        s1.record()
        torch.cuda.synchronize()
    ms = s0.elapsed_time(s1) / steps
    elems = b * d * L
    print(json.dumps({
        "metric": "complex selective-scan fwd+bwd B*D*L elements/s", "unit": "Gelem/s",
        "value": round(elems / (ms * 1e-3) / 1e9, 3), "ms_per_step": round(ms, 4),
        "steps": steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32 / complex64", "data": "synthetic", "n_gpus": 1,
        "config": {"workload": "complex SSM scan at the Mamba-130M layer shape", "batch": b,
                   "dim": d, "length": L, "dstate": n},
        "clocks": sampler.summary(), "gpu_launches": steps * 10}), flush=True)


def run_block_bench(args):
    """--config block: one Mamba block of configs[4]'s 2.8B-shape stack
    (d_model 2560, d_inner 5120, N 16, dt_rank 160, conv 4, bf16, RMSNorm) on
    B=8 sequences of L=8192 tokens, forward + backward through
    mamba.block.MambaBlock (cuBLAS projections in the scan's layout, the conv
    and scan kernels). --config c3: configs[3]'s 2-layer induction-heads model
    (d_model 64, B=64, L=256, fp32), forward + backward of the stack.
    Reported as tokens/s."""
    import torch

    from mamba.block import MambaBlock, MambaStack

    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev)
    g.manual_seed(3)
    if args.config == "block":
        b, L, dm = 8, 8192, 2560
        model = MambaBlock(dm, expand=2, d_state=16, norm_type="rmsnorm", num_layers=64,
                           dtype=torch.bfloat16)
        x = torch.randn(b, L, dm, generator=g, device=dev, dtype=torch.bfloat16)
        dout = torch.randn(b, L, dm, generator=g, device=dev, dtype=torch.bfloat16)
        x.requires_grad_(True)

        def step():
            model.zero_grad(set_to_none=True)
            x.grad = None
            model(x).backward(dout)
        workload = ("one Mamba block of configs[4]'s 2.8B-shape stack (d_model 2560, "
                    "d_inner 5120, N 16, dt_rank 160, conv 4, RMSNorm), bf16")
        dtype = "bf16"
    else:
        b, L, vocab = 64, 256, 16
        model = MambaStack(vocab, 64, 2, expand=2, d_state=16)
        tokens = torch.randint(1, 15, (b, L), generator=g, device=dev)
        labels = torch.randint(1, 15, (b,), generator=g, device=dev)

        def step():
            model.zero_grad(set_to_none=True)
            loss = torch.nn.functional.cross_entropy(model(tokens)[:, -1], labels)
            loss.backward()
        workload = "configs[3]: 2-layer Mamba, d_model 64, induction-heads shape, fp32"
        dtype = "f32"
    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    steps = max(1, min(args.steps, 20))
    sampler = ClockSampler(0)
    with sampler:
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record()
        for _ in range(steps):
            step()
        s1.record()
        torch.cuda.synchronize()
    ms = s0.elapsed_time(s1) / steps
    print(json.dumps({
        "metric": "Mamba block fwd+bwd tokens/s", "unit": "tokens/s",
        "value": round(b * L / (ms * 1e-3), 1), "ms_per_step": round(ms, 3), "steps": steps,
        "warmup": args.warmup, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": dtype, "data": "synthetic", "n_gpus": 1,
        "config": {"workload": workload, "batch": b, "seq_len": L},
        "clocks": sampler.summary()}), flush=True)


# ---------------------------------------------------------------- CPU arm
def _cpu_sample_shape(cfg, seconds_target):
    # a bounded sample: full length and state size, a slice of the channels
    return 1, 128 * max(1, os.cpu_count() or 1), cfg["length"], cfg["dstate"]


def _cpu_slice(job):
    """One process' share of the CPU sample: channels [lo, hi) of a seeded case."""
    b, d, L, n, lo, hi = job
    import numpy as np

    from oracle import selective_scan_oracle as orc

    x = orc.make_inputs(b, hi - lo, L, n, seed=5 + lo, dtype=np.float32)
    t0 = time.perf_counter()
    orc.fused_backward(x["u"], x["delta"], x["A"], x["B"], x["C"], x["D"], x["z"],
                       x["delta_bias"], True, None, True, None, dout=x["dout"],
                       dtype=np.float32)
    return time.perf_counter() - t0


def _cpu_run(cfg, b, d, L, n, workers):
    """Wall time of the oracle port over a (b, d, L, n) sample split by
    channels across `workers` processes (inputs are generated in each worker
    before its clock starts; the slowest worker's time is returned)."""
    import multiprocessing as mp

    per = max(1, d // workers)
    jobs = [(b, d, L, n, i, min(d, i + per)) for i in range(0, d, per)]
    with mp.get_context("fork").Pool(workers) as pool:
        times = pool.map(_cpu_slice, jobs)
    return max(times)


def cpu_baseline(cfg, seconds=15.0):
    """Oracle port (NumPy forward + analytic backward, fp32) on a bounded
    sample: one sequence of the config's length and state size, a slice of its
    channels, split across host threads."""
    threads = os.cpu_count() or 1
    b, d, L, n = _cpu_sample_shape(cfg, seconds)
    dt = _cpu_run(cfg, b, d, L, n, threads)
    return {"value": round(b * d * L / dt / 1e9, 6), "unit": UNIT, "cores": threads,
            "kind": "port",
            "sample": f"B={b} D={d} L={L} N={n} (of B={cfg['batch']} D={cfg['dim']}), fp32, "
                      f"{dt:.2f} s, NumPy restatement of the reference math "
                      "(fwd + analytic bwd); JAX absent on this image"}


def run_reference(args, cfg):
    """--impl reference: the reference's CPU path (its NumPy restatement)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return None
    threads = os.cpu_count() or 1
    b, d, L, n = _cpu_sample_shape(cfg, args.cpu_seconds)
    for _ in range(max(0, min(args.warmup, 1))):
        _cpu_run(cfg, b, d, min(L, 256), n, threads)
    times = [_cpu_run(cfg, b, d, L, n, threads) for _ in range(max(1, min(args.steps, 3)))]
    dt = statistics.mean(times)
    value = b * d * L / dt / 1e9
    res = {"metric": METRIC, "value": round(value, 6), "unit": UNIT, "impl": "reference",
           "n_gpus": int(os.environ.get("WORLD_SIZE", "1")), "steps": len(times),
           "warmup": args.warmup, "ms_per_step": round(dt * 1e3, 3), "higher_is_better": True,
           "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
           "config": {"workload": cfg["workload"], "batch": cfg["batch"], "dim": cfg["dim"],
                      "length": cfg["length"], "dstate": cfg["dstate"]},
           "cpu_baseline": {"value": round(value, 6), "unit": UNIT, "cores": threads,
                            "kind": "port",
                            "sample": f"each step B={b} D={d} L={L} N={n}; NumPy restatement "
                                      "of the reference's pure-JAX math (JAX not installed)"},
           "e2e": {"value": round(value, 6), "unit": UNIT, "h2d_bytes_per_step": 0,
                   "d2h_bytes_per_step": 0}}
    print(json.dumps(res), flush=True)
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=600)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config",
                    choices=sorted(CONFIGS) + ["step", "conv", "complex", "block", "c3"],
                    default="c1")
    ap.add_argument("--no-e2e", dest="e2e", action="store_false")
    ap.add_argument("--no-cpu-baseline", dest="cpu_baseline", action="store_false")
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--batch", type=int, default=None,
                    help="sequences per GPU in place of the config's (small profiling cases)")
    ap.add_argument("--traffic", type=float, default=None,
                    help="ncu dram bytes per backward launch, if captured")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "ours":
        print("warning: fewer than 3 warm-up steps", file=sys.stderr)
    if args.config in ("step", "conv", "complex", "block", "c3"):
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": f"the {args.config} leg has no "
                              "CPU reference arm; see --config c1"}))
        else:
            {"step": run_step_bench, "conv": run_conv_bench, "complex": run_complex_bench,
             "block": run_block_bench, "c3": run_block_bench}[args.config](args)
        return
    cfg = CONFIGS[args.config]
    if args.batch:
        cfg = dict(cfg, batch=args.batch, workload=cfg["workload"] + f" (batch overridden: {args.batch})")
    if args.impl == "reference":
        run_reference(args, cfg)
    else:
        run_gpu(args, cfg)


if __name__ == "__main__":
    main()
