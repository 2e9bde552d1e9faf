"""bench.py's host-side pieces: the seeded valid lengths of the right-padded
config are one global draw dealt to the ranks token-balanced (every rank sees
the same draw; the shards partition the batch), the line's config block
reports that draw's valid fraction, and the CPU sample is a real slice of the
config."""
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

import bench  # noqa: E402


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_seq_lens_partition_the_global_draw(world):
    cfg = bench.CONFIGS["c2"]
    shards = [bench._seq_lens(cfg, r, world) for r in range(world)]
    draws = [all_lens.tolist() for _, all_lens in shards]
    assert all(d == draws[0] for d in draws)  # one draw, seen identically by every rank
    mine = sorted(v for lens, _ in shards for v in lens.tolist())
    assert mine == sorted(draws[0])
    assert all(len(lens) == cfg["batch"] for lens, _ in shards)
    assert all(512 <= v <= cfg["length"] for v in draws[0])
    sums = [int(lens.sum()) for lens, _ in shards]
    assert max(sums) - min(sums) <= cfg["length"]


def test_config_block_and_cpu_sample():
    cfg = bench.CONFIGS["c2"]
    block = bench._config_block(cfg, 1)
    _, all_lens = bench._seq_lens(cfg, 0, 1)
    assert block["valid_fraction"] == round(float(all_lens.sum()) / (16 * 4096), 4)
    assert block["global_batch"] == 16 and block["io_dtype"] == "bf16"
    b, d, L, n = bench._cpu_sample_shape(cfg, 15.0)
    assert b == 1 and d <= cfg["dim"] and L == cfg["length"] and n == cfg["dstate"]
    c4 = bench._config_block(bench.CONFIGS["c4"], 8)
    assert c4["dim_per_gpu"] == 640 and c4["global_batch"] == 1
