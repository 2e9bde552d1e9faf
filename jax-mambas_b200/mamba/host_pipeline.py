"""Fused selective scan forward + backward on HOST buffers, pipelined.

The device-tensor op (``selective_scan_fn``) leaves the host<->device copies
to the caller; a caller whose activations live in host memory (the
reference's XLA path copies its inputs in and its results out around the
custom call) pays a PCIe transfer in and out that is an order of magnitude
longer than the kernels. This executor hides it: the batch is cut into
chunks along B (every sequence is independent), and three CUDA streams run

    copy-in (chunk i + 1)  |  forward + backward (chunk i)  |  copy-out (chunk i - 1)

over a ring of device buffer slots, so that the host->device and
device->host directions of the link run at the same time and the kernels
run in their shadow. The parameter gradients dA, dD and d(delta_bias) are
sums over the batch: each chunk's are added on the device and copied out
once at the end.

Results are those of one ``fused_forward_into`` + ``fused_backward_into``
over the whole batch except for the order of the batch sums of dA, dD and
d(delta_bias) (fp32, chunk by chunk).
"""
from __future__ import annotations

import torch

from .selective_scan_cuda import (_alloc_workspace, _io_dtype, chunk_states_elems,
                                  fused_backward_into, fused_forward_into)

_PER_SEQ_IN = ("u", "delta", "z", "dout")      # (B, D, L), io dtype
_PER_SEQ_BC = ("B", "C")                       # (B, N, L), io dtype
_PER_SEQ_OUT = ("out", "du", "ddelta", "dz")   # (B, D, L), io dtype
_PER_SEQ_DBC = ("dB", "dC")                    # (B, N, L), io dtype


class HostScanPipeline:
    """Pipelined fused forward + backward over pinned host tensors.

    Shapes are fixed at construction: batch, dim, length, dstate, the I/O
    dtype (float32 or bfloat16) and whether z is present; device buffers are
    allocated once (``depth`` slots of ``chunk`` sequences) and reused by
    every ``run``. ``chunk`` defaults to one sequence per slot for up to 8
    sequences, else batch // 8 (rounded up).
    """

    def __init__(self, batch, dim, length, dstate, dtype=torch.float32, *, with_z=True,
                 device="cuda", chunk=None, depth=3):
        if dtype not in (torch.float32, torch.bfloat16):
            raise TypeError("the I/O dtype must be float32 or bfloat16")
        if min(batch, dim, length, dstate) <= 0:
            raise ValueError("batch, dim, length and dstate must be positive")
        self.batch, self.dim, self.length, self.dstate = batch, dim, length, dstate
        self.dtype, self.with_z = dtype, with_z
        self.device = torch.device(device)
        self.chunk = chunk or max(1, -(-batch // 8))
        self.depth = max(2, depth)
        c, d, L, n = self.chunk, dim, length, dstate
        dev = self.device
        io = dict(dtype=dtype, device=dev)
        f32 = dict(dtype=torch.float32, device=dev)
        self.slots = []
        for _ in range(self.depth):
            s = {k: torch.empty((c, d, L), **io) for k in _PER_SEQ_IN + _PER_SEQ_OUT}
            s.update({k: torch.empty((c, n, L), **io) for k in _PER_SEQ_BC + _PER_SEQ_DBC})
            s["pre"] = torch.empty((c, d, L), **io)
            s["seq"] = torch.empty((c,), dtype=torch.int32, device=dev)
            s["last"] = torch.empty((c, d, n), **f32)
            s["cs"] = torch.empty(chunk_states_elems(c, L, d, n), **f32)
            s["ws"] = _alloc_workspace(c, L, d, n, _io_dtype(s["u"]), dev)
            s["dA"] = torch.empty((d, n), **f32)
            s["dD"] = torch.empty((d,), **f32)
            s["dbias"] = torch.empty((d,), **f32)
            s["in_ready"] = torch.cuda.Event()
            s["out_ready"] = torch.cuda.Event()
            s["free"] = torch.cuda.Event()
            self.slots.append(s)
        self.acc = {"dA": torch.zeros((d, n), **f32), "dD": torch.zeros((d,), **f32),
                    "dbias": torch.zeros((d,), **f32)}
        self.params = {"A": torch.empty((d, n), **f32), "D": torch.empty((d,), **f32),
                       "delta_bias": torch.empty((d,), **f32)}
        self.s_in = torch.cuda.Stream(dev)
        self.s_run = torch.cuda.Stream(dev)
        self.s_out = torch.cuda.Stream(dev)

    def _check_host(self, name, t, shape, dtype):
        if tuple(t.shape) != shape or t.dtype != dtype:
            raise ValueError(f"{name} must be a {dtype} tensor of shape {shape}, "
                             f"got {t.dtype} {tuple(t.shape)}")
        if t.is_cuda or not t.is_contiguous():
            raise ValueError(f"{name} must be a contiguous host tensor")

    def run(self, inputs, outputs, *, delta_softplus=True, zoh=False, reduce_params=None):
        """One fused forward + backward over host tensors.

        inputs: "u", "delta", "dout" and (if ``with_z``) "z" (B, D, L); "B",
        "C" (B, N, L) in the I/O dtype; "A" (D, N), "D", "delta_bias" (D,)
        float32; optional "seq_lens" (B,) int32. outputs: preallocated host
        tensors "out", "du", "ddelta" (and "dz") (B, D, L), "dB", "dC"
        (B, N, L) in the I/O dtype, "dA" (D, N), "dD", "ddelta_bias" (D,)
        float32. Host tensors should be pinned for the copies to overlap.
        ``reduce_params``, if given, is called on the compute stream with
        one flat float32 device tensor [dA, dD, d(delta_bias)] before it is
        copied out (a batch-sharded job passes an all-reduce here).
        Returns once every output is written (the host syncs on the copy-out
        stream).
        """
        b, d, L, n = self.batch, self.dim, self.length, self.dstate
        io = self.dtype
        for k in _PER_SEQ_IN:
            if k == "z" and not self.with_z:
                continue
            self._check_host(k, inputs[k], (b, d, L), io)
        for k in _PER_SEQ_BC:
            self._check_host(k, inputs[k], (b, n, L), io)
        for k in ("out", "du", "ddelta") + (("dz",) if self.with_z else ()):
            self._check_host(k, outputs[k], (b, d, L), io)
        for k in _PER_SEQ_DBC:
            self._check_host(k, outputs[k], (b, n, L), io)
        self._check_host("A", inputs["A"], (d, n), torch.float32)
        self._check_host("dA", outputs["dA"], (d, n), torch.float32)
        for k in ("D", "delta_bias"):
            self._check_host(k, inputs[k], (d,), torch.float32)
        for k in ("dD", "ddelta_bias"):
            self._check_host(k, outputs[k], (d,), torch.float32)
        seq = inputs.get("seq_lens")
        if seq is not None:
            self._check_host("seq_lens", seq, (b,), torch.int32)

        cur = torch.cuda.current_stream(self.device)
        # the previous run's copy-out has finished reading the accumulators
        # (the host synchronised on it); parameters go in on the copy-in stream
        with torch.cuda.stream(self.s_in):
            self.s_in.wait_stream(cur)
            for k in ("A", "D", "delta_bias"):
                self.params[k].copy_(inputs[k], non_blocking=True)
        params_in = torch.cuda.Event()
        params_in.record(self.s_in)
        with torch.cuda.stream(self.s_run):
            self.s_run.wait_stream(cur)
            for v in self.acc.values():
                v.zero_()
        A, Dp, bias = self.params["A"], self.params["D"], self.params["delta_bias"]

        chunks = [(b0, min(b, b0 + self.chunk)) for b0 in range(0, b, self.chunk)]
        for i, (b0, b1) in enumerate(chunks):
            s = self.slots[i % self.depth]
            m = b1 - b0
            v = {k: s[k][:m] for k in _PER_SEQ_IN + _PER_SEQ_OUT + _PER_SEQ_BC + _PER_SEQ_DBC
                 + ("pre", "seq", "last")}
            # ---- copy in (after the slot's previous copy-out)
            with torch.cuda.stream(self.s_in):
                if i >= self.depth:
                    self.s_in.wait_event(s["free"])
                for k in _PER_SEQ_IN + _PER_SEQ_BC:
                    if k == "z" and not self.with_z:
                        continue
                    v[k].copy_(inputs[k][b0:b1], non_blocking=True)
                if seq is not None:
                    v["seq"].copy_(seq[b0:b1], non_blocking=True)
                s["in_ready"].record(self.s_in)
            # ---- forward + backward
            with torch.cuda.stream(self.s_run):
                self.s_run.wait_event(s["in_ready"])
                if i == 0:
                    self.s_run.wait_event(params_in)
                z = v["z"] if self.with_z else None
                sl = v["seq"] if seq is not None else None
                cs = s["cs"][:chunk_states_elems(m, L, d, n)]
                fused_forward_into(v["u"], v["delta"], A, v["B"], v["C"], Dp, z, bias,
                                   delta_softplus, None, sl, v["out"], v["last"], cs, zoh,
                                   v["pre"] if z is not None else None)
                ws = s["ws"]  # sized for a full chunk: enough for a shorter last one
                fused_backward_into(v["u"], v["delta"], A, v["B"], v["C"], Dp, z, bias,
                                    delta_softplus, None, sl, cs, v["dout"], None,
                                    v["du"], v["ddelta"], s["dA"], v["dB"], v["dC"], s["dD"],
                                    v["dz"] if z is not None else None, s["dbias"], None, ws,
                                    zoh, v["pre"] if z is not None else None)
                self.acc["dA"].add_(s["dA"])
                self.acc["dD"].add_(s["dD"])
                self.acc["dbias"].add_(s["dbias"])
                s["out_ready"].record(self.s_run)
            # ---- copy out
            with torch.cuda.stream(self.s_out):
                self.s_out.wait_event(s["out_ready"])
                for k in ("out", "du", "ddelta", "dz") + _PER_SEQ_DBC:
                    if k == "dz" and not self.with_z:
                        continue
                    outputs[k][b0:b1].copy_(v[k], non_blocking=True)
                s["free"].record(self.s_out)
        with torch.cuda.stream(self.s_run):
            if reduce_params is not None:
                flat = torch.cat([self.acc["dA"].flatten(), self.acc["dD"], self.acc["dbias"]])
                reduce_params(flat)
                self.acc["dA"].copy_(flat[:d * n].view(d, n))
                self.acc["dD"].copy_(flat[d * n:d * n + d])
                self.acc["dbias"].copy_(flat[d * n + d:])
            done = torch.cuda.Event()
            done.record(self.s_run)
        with torch.cuda.stream(self.s_out):
            self.s_out.wait_event(done)
            outputs["dA"].copy_(self.acc["dA"], non_blocking=True)
            outputs["dD"].copy_(self.acc["dD"], non_blocking=True)
            outputs["ddelta_bias"].copy_(self.acc["dbias"], non_blocking=True)
        cur.wait_stream(self.s_out)
        self.s_out.synchronize()
        return outputs


def alloc_host_outputs(batch, dim, length, dstate, dtype=torch.float32, with_z=True):
    """Pinned host output tensors for ``HostScanPipeline.run``."""
    pin = dict(dtype=dtype, pin_memory=True)
    o = {k: torch.empty((batch, dim, length), **pin) for k in ("out", "du", "ddelta")}
    if with_z:
        o["dz"] = torch.empty((batch, dim, length), **pin)
    o.update({k: torch.empty((batch, dstate, length), **pin) for k in ("dB", "dC")})
    f32 = dict(dtype=torch.float32, pin_memory=True)
    o["dA"] = torch.empty((dim, dstate), **f32)
    o["dD"] = torch.empty((dim,), **f32)
    o["ddelta_bias"] = torch.empty((dim,), **f32)
    return o

