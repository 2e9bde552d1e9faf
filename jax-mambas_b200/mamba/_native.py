"""ctypes binding of libmamba_ss_b200.so (the C ABI in include/mamba_selective_scan.h).

The library is looked up next to the package (``jax-mambas_b200/lib``), the
in-tree location ``build.py`` writes to. There is no fallback: if the library
is missing, loading raises ``FileNotFoundError`` naming the searched paths,
like the reference's ``register_cuda_kernel``
(mamba/selective_scan_cuda.py:26-40).
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

_PKG_ROOT = Path(__file__).resolve().parents[1]
LIB_NAME = "libmamba_ss_b200.so"

MSS_OK = 0
MSS_INVALID_ARGUMENT = 1
MSS_INTERNAL = 2
MSS_F32 = 0
MSS_BF16 = 1
MSS_EULER = 0
MSS_ZOH = 1
CHUNK = 4

_c_void_p = ctypes.c_void_p
_i32 = ctypes.c_int32
_f32p = ctypes.c_void_p  # device pointers are passed as integers

# name -> (restype, argtypes)
SIGNATURES = {
    "mamba_ss_last_error": (ctypes.c_char_p, []),
    "mamba_ss_version": (ctypes.c_char_p, []),
    "mamba_ss_take_device_error": (ctypes.c_uint32, []),
    "mamba_ss_chunk_states_elems": (ctypes.c_int64, [_i32, _i32, _i32, _i32]),
    "mamba_ss_bwd_workspace_bytes": (ctypes.c_size_t, [_i32, _i32, _i32, _i32, _i32]),
    "mamba_ss_fwd": (ctypes.c_int, [_c_void_p, _i32, _i32, _i32, _i32, _i32] + [_f32p] * 9),
    "mamba_ss_fwd_bench": (ctypes.c_int, [_c_void_p, _i32, _i32, _i32, _i32, _i32, _i32] + [_f32p] * 9),
    "mamba_ss_bwd": (
        ctypes.c_int,
        [_c_void_p, _i32, _i32, _i32, _i32, _i32] + [_f32p] * 15 + [_c_void_p, ctypes.c_size_t],
    ),
    "mamba_ss_fused_fwd": (
        ctypes.c_int,
        [_c_void_p, _i32, _i32, _i32, _i32, _i32, _i32]
        + [_c_void_p] * 8  # u delta A B C D z delta_bias
        + [_i32]  # delta_softplus
        + [_c_void_p] * 6,  # initial_state seq_lens out out_pre last_state chunk_states
    ),
    "mamba_ss_fused_bwd": (
        ctypes.c_int,
        [_c_void_p, _i32, _i32, _i32, _i32, _i32, _i32]
        + [_c_void_p] * 8  # u delta A B C D z delta_bias
        + [_i32]  # delta_softplus
        + [_c_void_p] * 16  # initial_state seq_lens chunk_states out_pre dout dlast du ddelta dA dB dC dD dz dbias dinit workspace
        + [ctypes.c_size_t],
    ),
    "mamba_ss_fused_step": (
        ctypes.c_int,
        [_c_void_p, _i32, _i32, _i32, _i32, _i32]
        + [_c_void_p] * 8  # state u delta A B C D z
        + [_c_void_p, _i32, _c_void_p],  # delta_bias delta_softplus out
    ),
    "mamba_ss_conv1d_bwd_workspace_bytes": (ctypes.c_size_t, [_i32, _i32, _i32, _i32]),
    "mamba_ss_conv1d_fwd": (
        ctypes.c_int,
        [_c_void_p, _i32, _i32, _i32, _i32, _i32]
        + [_c_void_p] * 7,  # x weight bias seq_lens conv_state u final_state
    ),
    "mamba_ss_conv1d_bwd": (
        ctypes.c_int,
        [_c_void_p, _i32, _i32, _i32, _i32, _i32]
        + [_c_void_p] * 11  # x weight bias seq_lens conv_state du dx dweight dbias dconv_state workspace
        + [ctypes.c_size_t],
    ),
    "mamba_ss_conv1d_step": (
        ctypes.c_int,
        [_c_void_p, _i32, _i32, _i32, _i32] + [_c_void_p] * 5,  # x weight bias conv_state u
    ),
    "mamba_ss_complex_chunk_states_elems": (ctypes.c_int64, [_i32, _i32, _i32, _i32]),
    "mamba_ss_complex_bwd_workspace_bytes": (ctypes.c_size_t, [_i32, _i32, _i32, _i32]),
    "mamba_ss_complex_fwd": (
        ctypes.c_int,
        [_c_void_p, _i32, _i32, _i32, _i32, _i32]
        + [_c_void_p] * 8  # u delta A B C D z delta_bias
        + [_i32]  # delta_softplus
        + [_c_void_p] * 6,  # initial_state seq_lens out out_pre last_state chunk_states
    ),
    "mamba_ss_complex_bwd": (
        ctypes.c_int,
        [_c_void_p, _i32, _i32, _i32, _i32, _i32]
        + [_c_void_p] * 8  # u delta A B C D z delta_bias
        + [_i32]  # delta_softplus
        + [_c_void_p] * 16  # initial_state seq_lens chunk_states out_pre dout dlast du ddelta dA dB dC dD dz dbias dinit workspace
        + [ctypes.c_size_t],
    ),
    "mamba_ss_segments": (_i32, [_i32, _i32, _i32, _i32]),
    "mamba_ss_debug_set_wait_polls": (None, [ctypes.c_int64]),
    "mamba_ss_set_deterministic": (None, [_i32]),
    "mamba_ss_deterministic": (_i32, []),
    "mamba_ss_bounds_checked": (_i32, []),
    "mamba_ss_take_bounds_violations": (ctypes.c_uint64, [ctypes.POINTER(ctypes.c_int64)]),
    "mamba_ss_bounds_selftest": (ctypes.c_int, []),
    "mamba_ss_noalloc_scratch_bytes": (ctypes.c_size_t, []),
    "mamba_ss_fused_bwd_noalloc": (
        ctypes.c_int,
        [_c_void_p, _i32, _i32, _i32, _i32, _i32, _i32]
        + [_c_void_p] * 8  # u delta A B C D z delta_bias
        + [_i32]  # delta_softplus
        + [_c_void_p] * 15,  # initial_state seq_lens chunk_states out_pre dout dlast du ddelta dA dB dC dD dz dbias dinit
    ),
}

_LIB = None


def library_candidates(library_path=None):
    if library_path is not None:
        return [Path(library_path)]
    env = os.environ.get("MAMBA_SS_B200_LIB")
    cands = [Path(env)] if env else []
    cands.append(_PKG_ROOT / "lib" / LIB_NAME)
    return cands


def load(library_path=None):
    """Load (once) and return the ctypes handle of the selective-scan library."""
    global _LIB
    if _LIB is not None and library_path is None:
        return _LIB
    cands = library_candidates(library_path)
    path = next((c for c in cands if c.is_file()), None)
    if path is None:
        searched = ", ".join(str(c) for c in cands)
        raise FileNotFoundError(
            f"The selective-scan CUDA library is not built; searched: {searched}"
        )
    lib = ctypes.CDLL(str(path))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if library_path is None:
        _LIB = lib
    return lib


class SelectiveScanError(RuntimeError):
    """A failed call into the C ABI (status + message from mamba_ss_last_error)."""

    def __init__(self, status, message):
        super().__init__(message)
        self.status = status


def check(lib, status):
    if status != MSS_OK:
        msg = lib.mamba_ss_last_error().decode()
        if status == MSS_INVALID_ARGUMENT:
            raise ValueError(msg)
        raise SelectiveScanError(status, msg)
