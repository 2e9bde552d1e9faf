"""Selective-scan fwd+bwd throughput on B200 (B*D*L Gelem/s) — the metric of
BASELINE.json.

Default workload: configs[2], the Mamba-2.8B layer shape the target is quoted
on — B=16, D=5120, L=4096, N=16, bf16 u/delta/z/B/C with fp32 A, D, bias and
state, fused softplus(delta + bias), D skip and silu(z) gate, dy ~ N(0,1),
right-padded valid lengths ~ U[512, 4096] (delta = u = 0 past them). One step
= one forward + one backward of the fused selective scan over one batch (plus,
for N>1 GPUs, the all-reduce of dA, dD and ddelta_bias across ranks: the
batch is sharded, each rank holds a full configs[2] batch, i.e. weak
scaling). ``value`` counts valid (sequence, channel, step) positions per
second; ``value_all_positions`` counts every B*D*L position.
The line also carries ``channel_sharded``: configs[4]'s single sequence
(B=1, L=131072, D=5120, bf16) with d_inner split over the N ranks (strong
scaling). ``--config c1`` runs configs[1] (fp32, B=8, D=1536, L=2048).

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
        # start timing only once the sampler is writing (nvidia-smi can take
        # a second or more to come up, longer than a short timed region)
        t_end = time.time() + 5.0
        while self.proc is not None and time.time() < t_end:
            if os.path.getsize(self.path) > 0:
                break
            time.sleep(0.05)
        time.sleep(0.1)
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


def _seq_lens(cfg, rank, world):
    """This rank's valid lengths for a right-padded config: the global batch's
    lengths ~ U[512, L] from one seeded generator (the same draw on every
    rank), dealt to the ranks token-balanced (longest first, snake order), as
    a length-aware data loader would. Returns (lengths of this rank, lengths
    of the global batch), int32 CPU tensors."""
    import torch

    from mamba.distributed import token_balanced_shards

    b, L = cfg["batch"], cfg["length"]
    g = torch.Generator()
    g.manual_seed(4321)
    lens = torch.randint(512, L + 1, (b * world,), generator=g, dtype=torch.int32)
    idx = token_balanced_shards(lens.tolist(), world)[rank]
    return lens[idx].contiguous(), lens


class ScanCase:
    """Device inputs and outputs of one rank's share of a config, and its step:
    fused forward, fused backward, and the exchange (batch sharding: the
    all-reduce of [dA | dD | ddelta_bias]; channel sharding: of dB and dC).

    The exchange is issued asynchronously on NCCL's stream right after the
    backward; only the next backward (which rewrites the reduced buffers)
    waits for it, so it runs under the next step's forward."""

    def __init__(self, cfg, rank, world, dev):
        import torch

        from mamba import selective_scan_cuda as ssc
        from mamba.distributed import channel_shard, flat_param_grads

        self.cfg, self.rank, self.world, self.dev = cfg, rank, world, dev
        b, d, L, n = cfg["batch"], cfg["dim"], cfg["length"], cfg["dstate"]
        self.chan = cfg.get("shard") == "channels"
        self.d_total = d
        if self.chan:  # this rank's block of channels; B and C are shared
            sl = channel_shard(d, rank, world)
            d = sl.stop - sl.start
        self.b, self.d, self.L, self.n = b, d, L, n
        io = torch.bfloat16 if cfg["dtype"] == "bf16" else torch.float32
        self.io, self.esize = io, (2 if io == torch.bfloat16 else 4)
        g = torch.Generator(device=dev)
        g.manual_seed(1234 + (0 if self.chan else rank))

        def normal(*shape):
            return torch.randn(*shape, generator=g, device=dev, dtype=torch.float32).to(io)

        self.u, self.delta, self.z, self.dout = (normal(b, d, L) for _ in range(4))
        self.B, self.C = normal(b, n, L), normal(b, n, L)
        self.A = (-torch.arange(1, n + 1, device=dev, dtype=torch.float32)).expand(d, n).contiguous()
        self.Dp = torch.randn(d, generator=g, device=dev)
        self.bias = torch.rand(d, generator=g, device=dev) * 2.0 - 4.0
        self.seq_lens = None
        self.valid_steps = b * L  # this rank's valid (sequence, step) pairs
        self.valid_steps_global = b * L * (1 if self.chan else world)
        if cfg["padded"]:
            lens, all_lens = _seq_lens(cfg, rank, world)
            self.seq_lens = lens.to(dev)
            self.valid_steps = int(lens.sum())
            self.valid_steps_global = int(all_lens.sum())
            m = (torch.arange(L, device=dev)[None, :] < self.seq_lens[:, None].long())[:, None, :]
            self.delta.masked_fill_(~m, 0)
            self.u.masked_fill_(~m, 0)
        self.out, self.pre = torch.empty_like(self.u), torch.empty_like(self.u)
        self.last = torch.empty(b, d, n, device=dev)
        self.cs = torch.empty(ssc.chunk_states_elems(b, L, d, n), device=dev)
        self.du, self.ddl, self.dz = (torch.empty_like(self.u) for _ in range(3))
        self.dB, self.dC = torch.empty_like(self.B), torch.empty_like(self.C)
        self.params, self.dA, self.dDp, self.dbias = flat_param_grads(d, n, dev)
        self.ws = ssc._alloc_workspace(b, L, d, n, 1 if io == torch.bfloat16 else 0, dev)
        self.work = []
        self.ssc = ssc

    def fwd(self):
        self.ssc.fused_forward_into(self.u, self.delta, self.A, self.B, self.C, self.Dp, self.z,
                                    self.bias, True, None, self.seq_lens, self.out, self.last,
                                    self.cs, out_pre=self.pre)

    def bwd(self):
        for w in self.work:  # the previous step's exchange reads the buffers rewritten here
            w.wait()
        self.work = []
        self.ssc.fused_backward_into(self.u, self.delta, self.A, self.B, self.C, self.Dp, self.z,
                                     self.bias, True, None, self.seq_lens, self.cs, self.dout,
                                     None, self.du, self.ddl, self.dA, self.dB, self.dC,
                                     self.dDp, self.dz, self.dbias, None, self.ws,
                                     out_pre=self.pre)

    def exchange(self):
        from mamba.distributed import allreduce_bc_grads, allreduce_param_grads

        if os.environ.get("MSS_BENCH_EXCHANGE") == "sync":  # diagnostics: blocking exchange
            if self.chan:
                allreduce_bc_grads(self.dB, self.dC)
            else:
                allreduce_param_grads(self.params)
            return
        if self.chan:
            self.work = allreduce_bc_grads(self.dB, self.dC, async_op=True)
        else:
            w = allreduce_param_grads(self.params, async_op=True)
            self.work = [w] if w is not None else []

    def finish(self):
        for w in self.work:
            w.wait()
        self.work = []

    def step(self):
        self.fwd()
        self.bwd()
        self.exchange()

    def time(self, steps, warmup, sampler=None):
        """(total ms over `steps`, mean forward ms, mean backward ms), CUDA
        events on the launching stream; total is the max over ranks."""
        import torch
        import torch.distributed as dist

        for _ in range(max(warmup, 0)):
            self.step()
        self.finish()
        torch.cuda.synchronize()
        stream = torch.cuda.current_stream(self.dev)
        ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(steps)]
        # the clock sampler (rank 0 only) comes up before the barrier: started
        # after it, its start-up delayed rank 0's first launch, and the other
        # ranks' clocks then counted their wait for rank 0 at the first exchange
        ctx = sampler if sampler is not None else _Null()
        with ctx:
            if self.world > 1:
                dist.barrier()
            torch.cuda.synchronize()
            t0 = torch.cuda.Event(enable_timing=True)
            t1 = torch.cuda.Event(enable_timing=True)
            t0.record(stream)
            for i in range(steps):
                ev[i][0].record(stream)
                self.fwd()
                ev[i][1].record(stream)
                self.bwd()
                ev[i][2].record(stream)
                self.exchange()
            self.finish()
            t1.record(stream)
            torch.cuda.synchronize()
            if self.world > 1:
                dist.barrier()
        total = t0.elapsed_time(t1)
        fwd_ms = statistics.mean(e[0].elapsed_time(e[1]) for e in ev)
        bwd_ms = statistics.mean(e[1].elapsed_time(e[2]) for e in ev)
        self.per_rank = None
        if self.world > 1:
            # every rank's own figures (its backward includes waiting for the
            # previous step's exchange, i.e. for the slowest rank)
            mine = torch.tensor([total, fwd_ms, bwd_ms, float(self.valid_steps)],
                                device=self.dev)
            allr = [torch.empty_like(mine) for _ in range(self.world)]
            dist.all_gather(allr, mine)
            self.per_rank = [[round(float(v), 4) for v in r.tolist()] for r in allr]
            t = torch.tensor([total], device=self.dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            total = float(t.item())
        return total, fwd_ms, bwd_ms

    def launches_per_step(self):
        """Kernels of this library per step: forward 1, backward 2 (tile +
        parameter reduction); bf16 I/O adds the widening of B and C and the
        two narrowings of dB/dC; time segments add the end-state pass and its
        combine (forward) and the adjoint pass and its combine (backward)."""
        k = 3 + (3 if self.esize == 2 else 0)
        if self.ssc._lib().mamba_ss_segments(self.b, self.L, self.d, self.n) > 1:
            k += 4
        return k


class _Null:
    def __enter__(self):
        return self

    def __exit__(self, *exc):
        return False


def _config_block(cfg, world):
    """The line's ``config`` object (the same for the GPU and reference arms)."""
    b, L, n = cfg["batch"], cfg["length"], cfg["dstate"]
    chan = cfg.get("shard") == "channels"
    d_rank = -(-cfg["dim"] // world) if chan else cfg["dim"]
    esize = 2 if cfg["dtype"] == "bf16" else 4
    valid = 1.0
    if cfg["padded"]:
        _, all_lens = _seq_lens(cfg, 0, world)
        valid = float(all_lens.sum()) / (b * world * L)
    return {"workload": cfg["workload"], "batch_per_gpu": b, "dim": cfg["dim"],
            "dim_per_gpu": d_rank, "length": L, "dstate": n, "io_dtype": cfg["dtype"],
            "global_batch": b * (1 if chan else world),
            "parallelism": (f"channel-sharded over {world} GPUs" if chan
                            else f"batch-sharded dp{world}") if world > 1 else "single GPU",
            "l2": "inputs larger than L2 (u, delta, z, dy: "
                  f"{b * d_rank * L * esize * 4 / 1e6:.0f} MB per step)",
            "valid_fraction": round(valid, 4),
            "valid_lengths": "U[512, L], global batch dealt to ranks token-balanced"
            if cfg["padded"] else None,
            "value_counts": "valid (sequence, channel, step) positions"}


def _ncu_counts(config):
    """Per valid element DRAM bytes and warp instructions of each scan kernel
    for `config`, from a committed ncu capture summary (profiles/)."""
    f = ROOT / "profiles" / "ncu_counts.json"
    if not f.exists():
        return None
    return json.loads(f.read_text()).get(config)


def run_gpu(args, cfg):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        # The exchanges are small (110 KB of parameter gradients; 8 MB of
        # dB/dC for configs[4]). NCCL's NVLink SHARP (NVLS) all-reduce took
        # about 2.5 ms per call on 8 B200s here (a configs[2] step 4.5 ->
        # 7.1 ms), its ring/tree algorithms a few tens of microseconds, so
        # NVLS is off (MSS_BENCH_NVLS=1 keeps the environment's setting; a
        # default from the environment is not trusted: the pool's boxes may
        # set one).
        if os.environ.get("MSS_BENCH_NVLS") != "1":
            os.environ["NCCL_NVLS_ENABLE"] = "0"
        print(f"rank {rank}: NCCL_NVLS_ENABLE={os.environ.get('NCCL_NVLS_ENABLE')}",
              file=sys.stderr)
        # NCCL prints its version banner on stdout when the communicator is
        # created; keep stdout for the one JSON line
        with _stdout_to_stderr():
            dist.init_process_group("nccl", device_id=dev)
            dist.barrier()

    if args.deterministic:
        from mamba.selective_scan_cuda import set_deterministic

        set_deterministic(True)
    case = ScanCase(cfg, rank, world, dev)
    sampler = ClockSampler(local)
    total_ms, fwd_ms, bwd_ms = case.time(args.steps, args.warmup, sampler)
    per_rank = case.per_rank
    clocks = sampler.summary()
    clocks_per_rank = None
    if world > 1:
        clocks_per_rank = [None] * world
        dist.all_gather_object(clocks_per_rank, {k: clocks.get(k) for k in ("sm_mhz", "reasons")})
    b, d, L, n, esize = case.b, case.d, case.L, case.n, case.esize
    launches = case.launches_per_step() * args.steps
    valid = case.valid_steps / (b * L)
    ms_per_step = total_ms / args.steps
    # throughput counts valid positions only (padded steps are skipped by the
    # kernels); the all-position figure is reported beside it
    total_valid = case.valid_steps_global * case.d_total
    total_all = b * L * case.d_total * (1 if case.chan else world)
    value = total_valid / (ms_per_step * 1e-3) / 1e9
    value_all = total_all / (ms_per_step * 1e-3) / 1e9
    del case
    torch.cuda.empty_cache()

    # ---- strong scaling: configs[4]'s single sequence, channels over the ranks
    strong = None
    if args.strong and args.config != "c4":
        c4 = ScanCase(CONFIGS["c4"], rank, world, dev)
        s_ms, s_f, s_b = c4.time(max(3, min(args.steps, 10)), 3)
        s_steps = max(3, min(args.steps, 10))
        strong = {"workload": CONFIGS["c4"]["workload"], "scaling": "strong",
                  "value": round(c4.b * c4.L * c4.d_total / (s_ms / s_steps * 1e-3) / 1e9, 3),
                  "unit": UNIT, "ms_per_step": round(s_ms / s_steps, 3), "steps": s_steps,
                  "dim_per_gpu": c4.d, "dtype": "bf16",
                  "segments": int(c4.ssc._lib().mamba_ss_segments(c4.b, c4.L, c4.d, c4.n)),
                  "kernels_ms": {"fwd": round(s_f, 3), "bwd": round(s_b, 3)},
                  "exchange": "async NCCL all-reduce of dB and dC (sums over all channels)"}
        launches += c4.launches_per_step() * s_steps
        del c4
        torch.cuda.empty_cache()

    # ---- e2e through the public API with host buffers
    e2e = run_e2e(args, cfg, dev, rank, world) if args.e2e and cfg.get("shard") != "channels" \
        else None

    if rank != 0:
        if world > 1:
            dist.destroy_process_group()
        return None

    elems, fwd_bytes, bwd_bytes, carry_bytes, mufu_f, mufu_b = _algorithmic(cfg, esize, d)
    fwd_bytes, bwd_bytes, carry_bytes = fwd_bytes * valid, bwd_bytes * valid, carry_bytes * valid
    valid_elems = elems * valid  # one launch's valid (sequence, channel, step) triples
    hbm, sm_max, peak_src = _peaks()
    bwd_gbs = bwd_bytes / (bwd_ms * 1e-3) / 1e9
    fwd_gbs = fwd_bytes / (fwd_ms * 1e-3) / 1e9
    f_mhz = clocks.get("sm_mhz") or sm_max
    mufu_peak = 148 * 16 * f_mhz * 1e6  # ops/s: 16 MUFU lanes per SM per clock
    issue_peak = 148 * 4 * f_mhz * 1e6  # warp instructions/s: one per SM sub-partition per clock
    mufu_bwd = valid_elems * mufu_b / (bwd_ms * 1e-3)
    mufu_fwd = valid_elems * mufu_f / (fwd_ms * 1e-3)
    counts = _ncu_counts(args.config) if not args.batch else None
    traffic = args.traffic
    issue = None
    if counts:
        kb, kf = counts["ss_bwd_tile_kernel"], counts["ss_fwd_kernel"]
        if traffic is None:
            traffic = round(kb["dram_bytes_per_valid_elem"] * valid_elems)
        ib = kb["warp_inst_per_valid_elem"] * valid_elems / (bwd_ms * 1e-3)
        i_f = kf["warp_inst_per_valid_elem"] * valid_elems / (fwd_ms * 1e-3)
        issue = {"bound": "issue", "unit": "warp inst/s", "peak": issue_peak,
                 "clock_mhz": f_mhz,
                 "inst_per_elem": {"fwd": kf["warp_inst_per_valid_elem"],
                                   "bwd": kb["warp_inst_per_valid_elem"]},
                 "bwd_frac": round(ib / issue_peak, 4), "fwd_frac": round(i_f / issue_peak, 4),
                 "source": counts.get("source", "profiles/ncu_counts.json")}
    fracs = {"bwd": {"hbm": bwd_gbs / hbm, "sfu": mufu_bwd / mufu_peak},
             "fwd": {"hbm": fwd_gbs / hbm, "sfu": mufu_fwd / mufu_peak}}
    fp32 = None
    if issue:
        fracs["bwd"]["issue"] = issue["bwd_frac"]
        fracs["fwd"]["issue"] = issue["fwd_frac"]
        if "fp32_ops_per_valid_elem" in kb:
            fp32_peak = 148 * 128 * f_mhz * 1e6  # fp32 lanes per SM per clock
            ob = kb["fp32_ops_per_valid_elem"] * valid_elems / (bwd_ms * 1e-3)
            of = kf["fp32_ops_per_valid_elem"] * valid_elems / (fwd_ms * 1e-3)
            fp32 = {"bound": "fp32", "unit": "fp32 op/s", "peak": fp32_peak, "clock_mhz": f_mhz,
                    "ops_per_elem": {"fwd": kf["fp32_ops_per_valid_elem"],
                                     "bwd": kb["fp32_ops_per_valid_elem"]},
                    "bwd_frac": round(ob / fp32_peak, 4), "fwd_frac": round(of / fp32_peak, 4)}
            fracs["bwd"]["fp32"] = fp32["bwd_frac"]
            fracs["fwd"]["fp32"] = fp32["fwd_frac"]
    # the binding ceiling of a kernel is the resource it uses the largest share of
    binding = {k: {"resource": max(v, key=v.get), "frac": round(max(v.values()), 4)}
               for k, v in fracs.items()}
    res = {
        "metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4),
        "higher_is_better": True, "scaling": "strong" if cfg.get("shard") else "weak",
        "vs_baseline": None, "dtype": cfg["dtype"],
        "data": "synthetic (seeded N(0,1)/U(-4,-2) inputs of the config)",
        "value_all_positions": round(value_all, 3),
        "config": dict(_config_block(cfg, world), deterministic_dBdC=bool(args.deterministic)),
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
        "roofline_issue": issue,
        "roofline_fp32": fp32,
        "binding": binding,
        "clocks": clocks,
        "clocks_per_rank": clocks_per_rank,
        "gpu_launches": launches,
    }
    if per_rank is not None:
        res["per_rank_ms"] = {"columns": ["total", "fwd", "bwd (incl. the wait for the "
                                          "previous exchange)", "valid_steps"],
                              "ranks": per_rank}
    if strong is not None:
        res["channel_sharded"] = strong
    if e2e is not None:
        res["e2e"] = e2e
    if args.cpu_baseline and world == 1:
        res["cpu_baseline"] = cpu_baseline(cfg, args.cpu_seconds)
    print(json.dumps(res), flush=True)
    if world > 1:
        dist.destroy_process_group()
    return res


def run_e2e(args, cfg, dev, rank, world):
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
    io = torch.bfloat16 if cfg["dtype"] == "bf16" else torch.float32
    g = torch.Generator()
    g.manual_seed(99 + rank)

    def host(*shape):
        return torch.randn(*shape, generator=g).to(io).pin_memory()

    h = {"u": host(b, d, L), "delta": host(b, d, L), "z": host(b, d, L),
         "dout": host(b, d, L), "B": host(b, n, L), "C": host(b, n, L)}
    h["A"] = (-torch.arange(1, n + 1, dtype=torch.float32)).expand(d, n).contiguous().pin_memory()
    h["D"] = torch.randn(d, generator=g).pin_memory()
    h["delta_bias"] = (torch.rand(d, generator=g) * 2 - 4).pin_memory()
    valid_global = b * L * world
    if cfg["padded"]:
        lens, all_lens = _seq_lens(cfg, rank, world)
        h["seq_lens"] = lens.pin_memory()
        valid_global = int(all_lens.sum())
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
    value = valid_global * d / (ms * 1e-3) / 1e9
    return {"value": round(value, 3), "unit": UNIT, "ms_per_step": round(ms, 3),
            "steps": k, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "api": "mamba.host_pipeline.HostScanPipeline.run (pinned host buffers; "
                   "batch chunks copied in, scanned fwd+bwd and copied out on three streams)",
            "chunk_batch": pipe.chunk,
            "autograd_value": round(valid_global * d / (ms_a * 1e-3) / 1e9, 3),
            "value_counts": "valid (sequence, channel, step) positions",
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
    """A bounded sample that is a real slice of the config: one full-length
    sequence (all steps valid) and its first min(D, 128 x cores) channels."""
    return 1, min(cfg["dim"], 128 * max(1, os.cpu_count() or 1)), cfg["length"], cfg["dstate"]


def _sample_label(cfg, b, d, L, n):
    return (f"B={b} D={d} L={L} N={n}: one full-length sequence and the first {d} of "
            f"{cfg['dim']} channels of the config (batch {cfg['batch']}), all steps valid; "
            "fp32 (NumPy has no bf16); NumPy restatement of the reference math "
            "(fwd + analytic bwd), JAX absent on this image; throughput per valid position")


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
            "sample": _sample_label(cfg, b, d, L, n) + f"; {dt:.2f} s"}


def run_reference(args, cfg):
    """--impl reference: the reference's CPU path (its NumPy restatement)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return None
    threads = os.cpu_count() or 1
    b, d, L, n = _cpu_sample_shape(cfg, args.cpu_seconds)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    for _ in range(max(0, min(args.warmup, 1))):
        _cpu_run(cfg, b, d, min(L, 256), n, threads)
    times = [_cpu_run(cfg, b, d, L, n, threads) for _ in range(max(1, args.steps))]
    dt = statistics.mean(times)
    value = b * d * L / dt / 1e9
    res = {"metric": METRIC, "value": round(value, 6), "unit": UNIT, "impl": "reference",
           "n_gpus": world, "steps": len(times),
           "warmup": args.warmup, "ms_per_step": round(dt * 1e3, 3), "higher_is_better": True,
           "scaling": "strong" if cfg.get("shard") else "weak", "vs_baseline": None,
           "dtype": "f32", "data": "synthetic (seeded N(0,1)/U(-4,-2) inputs of the config)",
           "config": _config_block(cfg, world),
           "cpu_baseline": {"value": round(value, 6), "unit": UNIT, "cores": threads,
                            "kind": "port", "sample": "each step " + _sample_label(cfg, b, d, L, n)},
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
                    default="c2")
    ap.add_argument("--no-e2e", dest="e2e", action="store_false")
    ap.add_argument("--no-cpu-baseline", dest="cpu_baseline", action="store_false")
    ap.add_argument("--no-strong", dest="strong", action="store_false",
                    help="skip the channel-sharded configs[4] single-sequence leg")
    ap.add_argument("--deterministic", action="store_true",
                    help="bitwise-reproducible dB/dC (partials summed in a fixed order)")
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
                              "CPU reference arm; see --config c2"}))
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
