"""The C-ABI library loads and exports every symbol include/*.h declares;
argument validation answers without touching a GPU."""
import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def _declared_symbols():
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        text = h.read_text()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names.update(re.findall(r"\b(mamba_ss_\w+)\s*\(", text))
    return sorted(names)


@pytest.fixture(scope="module")
def lib():
    from mamba import _native

    return _native.load()


def test_exports_every_declared_symbol(lib):
    names = _declared_symbols()
    assert len(names) >= 9
    for n in names:
        assert hasattr(lib, n), n


def test_bindings_cover_the_header():
    from mamba import _native

    assert set(_declared_symbols()) <= set(_native.SIGNATURES)


def test_sizes(lib):
    # one carry per 4 steps; small problems add the time-segment scratch
    assert lib.mamba_ss_chunk_states_elems(8, 2048, 1536, 16) == 8 * 1536 * 512 * 16
    assert lib.mamba_ss_chunk_states_elems(2, 512, 128, 16) >= 2 * 128 * 128 * 16
    assert lib.mamba_ss_chunk_states_elems(2, 513, 128, 16) >= 2 * 128 * 129 * 16
    assert lib.mamba_ss_chunk_states_elems(0, 257, 128, 16) == 0
    f32 = lib.mamba_ss_bwd_workspace_bytes(8, 2048, 1536, 16, 0)
    bf16 = lib.mamba_ss_bwd_workspace_bytes(8, 2048, 1536, 16, 1)
    assert f32 >= 8 * 1536 * 16 * 4 + 2 * 8 * 1536 * 4
    assert bf16 >= f32 + 2 * 8 * 16 * 2048 * 4
    assert lib.mamba_ss_version().startswith(b"mamba-ss-b200")


@pytest.mark.parametrize("case,msg", [
    (dict(dstate=3), b"N must be one of"),
    (dict(batch=0), b"must be positive"),
    (dict(length=-1), b"must be positive"),
    (dict(disc=2), b"discretization"),
    (dict(io=7), b"io_dtype"),
])
def test_invalid_arguments(lib, case, msg):
    a = dict(batch=1, length=8, dim=4, dstate=16, disc=0, io=0)
    a.update(case)
    p = ctypes.c_void_p(16)  # never dereferenced: validation fails first
    st = lib.mamba_ss_fused_fwd(None, a["io"], a["disc"], a["batch"], a["length"], a["dim"],
                                a["dstate"], p, p, p, p, p, None, None, None, 0, None, None,
                                p, None, None, p)
    assert st == 1
    assert msg in lib.mamba_ss_last_error()


def test_null_required_pointer(lib):
    st = lib.mamba_ss_fused_fwd(None, 0, 0, 1, 8, 4, 16, None, None, None, None, None, None,
                                None, None, 0, None, None, None, None, None, None)
    assert st == 1
    assert b"non-null" in lib.mamba_ss_last_error()


def test_backward_rejects_small_workspace(lib):
    p = ctypes.c_void_p(256)
    st = lib.mamba_ss_fused_bwd(None, 0, 0, 1, 8, 4, 16, p, p, p, p, p, None, None, None, 0,
                                None, None, p, None, p, None, p, p, p, p, p, None, None, None,
                                None, p, 16)
    assert st == 1
    assert b"workspace needs" in lib.mamba_ss_last_error()


def test_bench_rejects_nonpositive_repeats(lib):
    p = ctypes.c_void_p(256)
    st = lib.mamba_ss_fwd_bench(None, 0, 0, 1, 8, 4, 16, p, p, p, p, p, p, p, p, p)
    assert st == 1
    assert b"repeats" in lib.mamba_ss_last_error()
