"""The host-buffer pipeline (mamba.host_pipeline) against the float64 oracle:
batch chunks copied in, scanned and copied out on three streams give the
results of one whole-batch call (fp32 1e-5 forward / 1e-4 backward; bf16
2e-2), including a last chunk shorter than the others, slot reuse (more
chunks than slots), right padding and runs repeated on the same buffers."""
import numpy as np
import pytest
import torch

from _helpers import (assert_bf16_close, BF16_TOL, BWD_TOL, FWD_TOL, assert_close, bf16_round, oracle_fused,
                      rel_err)
from oracle import selective_scan_oracle as orc

pytestmark = pytest.mark.gpu


def _host(a, dtype):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dtype).pin_memory()


def _run(x, io, chunk, depth, with_z=True, repeats=1):
    from mamba.host_pipeline import HostScanPipeline, alloc_host_outputs

    b, d, L = x["u"].shape
    n = x["A"].shape[1]
    inp = {k: _host(x[k], io) for k in ("u", "delta", "dout", "B", "C")}
    if with_z:
        inp["z"] = _host(x["z"], io)
    for k in ("A", "D", "delta_bias"):
        inp[k] = _host(x[k], torch.float32)
    if x["seq_lens"] is not None:
        inp["seq_lens"] = torch.from_numpy(x["seq_lens"]).pin_memory()
    outs = alloc_host_outputs(b, d, L, n, io, with_z=with_z)
    pipe = HostScanPipeline(b, d, L, n, io, with_z=with_z, chunk=chunk, depth=depth)
    for _ in range(repeats):
        for v in outs.values():
            v.fill_(float("nan"))
        pipe.run(inp, outs, delta_softplus=x["delta_softplus"])
    return {k: v.float().numpy() for k, v in outs.items()}


_KEYS = {"du": "du", "ddelta": "ddelta", "dz": "dz", "dB": "dB", "dC": "dC", "dA": "dA",
         "dD": "dD", "ddelta_bias": "ddelta_bias"}


@pytest.mark.parametrize("batch,chunk,depth", [(1, None, 3), (5, 2, 2), (8, 1, 3), (7, 3, 2)])
def test_pipeline_fp32(batch, chunk, depth):
    x = orc.make_inputs(batch, 40, 300, 16, seed=50 + batch)
    ref = oracle_fused(x)
    res = _run(x, torch.float32, chunk, depth, repeats=2)
    assert_close(res["out"], ref["out"], FWD_TOL, "out")
    for k, r in _KEYS.items():
        assert_close(res[k], ref[r], BWD_TOL, k)


def test_pipeline_bf16_padded_no_z():
    x = orc.make_inputs(6, 24, 512, 16, seed=61, with_z=False, valid_lengths=(100, 512))
    ref = oracle_fused(x, io_round=bf16_round)
    res = _run(x, torch.bfloat16, 2, 2, with_z=False)
    assert_bf16_close(res["out"], ref["out"])
    for k, r in _KEYS.items():
        if k != "dz":
            assert_bf16_close(res[k], ref[r], k)
    # padding positions are exact zeros
    for b, n in enumerate(x["seq_lens"]):
        assert not res["out"][b, :, n:].any()
        assert not res["du"][b, :, n:].any()


def test_pipeline_rejects_device_or_misshapen_inputs():
    from mamba.host_pipeline import HostScanPipeline, alloc_host_outputs

    x = orc.make_inputs(2, 8, 64, 4, seed=3)
    pipe = HostScanPipeline(2, 8, 64, 4)
    outs = alloc_host_outputs(2, 8, 64, 4)
    inp = {k: _host(x[k], torch.float32) for k in ("u", "delta", "z", "dout", "B", "C",
                                                   "A", "D", "delta_bias")}
    bad = dict(inp, u=inp["u"].cuda())
    with pytest.raises(ValueError, match="host tensor"):
        pipe.run(bad, outs)
    bad = dict(inp, B=inp["B"][:, :2])
    with pytest.raises(ValueError, match="shape"):
        pipe.run(bad, outs)
