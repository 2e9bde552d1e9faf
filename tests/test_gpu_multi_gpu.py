"""Multi-GPU parity on hardware: tests/_multi_gpu_check.py under
torch.distributed.run with one rank per visible GPU (NCCL), comparing the
batch-sharded parameter gradients and the channel-sharded dB/dC, summed over
the ranks, with a whole-problem run. Skipped with fewer than 2 GPUs."""
import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs 2 or more GPUs")
def test_sharded_gradients_match_one_gpu():
    world = min(torch.cuda.device_count(), 8)
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={world}", "--master-addr=127.0.0.1", "--master-port=29533",
           str(ROOT / "tests" / "_multi_gpu_check.py")]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=600, env=env)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert f"MULTI_GPU_OK {world}" in r.stdout
