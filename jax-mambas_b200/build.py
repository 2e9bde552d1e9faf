"""Builds libmamba_ss_b200.so (the sm_100a selective-scan kernels + C ABI).

Each ``csrc/*.cu`` file is compiled by nvcc for sm_100a only and linked into
one shared library next to this file (``lib/``), so the library travels with
the source tree. Run ``python jax-mambas_b200/build.py`` or call
``build_library()``.

``build_library(bounds=True)`` (``build.py --bounds``) builds the debug bounds
library ``libmamba_ss_b200_bounds.so`` from the same sources with
``-DMSS_BOUNDS_CHECK``: its scan kernels check every computed global index
against its array's extent and report violations through
``mamba_ss_take_bounds_violations()`` instead of faulting. Load it in place of
the normal library with ``MAMBA_SS_B200_LIB``.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_ROOT = Path(__file__).resolve().parent
CSRC = PKG_ROOT / "csrc"
LIB_DIR = PKG_ROOT / "lib"
LIB_NAME = "libmamba_ss_b200.so"
BOUNDS_LIB_NAME = "libmamba_ss_b200_bounds.so"
BUILD_DIR = PKG_ROOT / "_build"
BOUNDS_BUILD_DIR = PKG_ROOT / "_build_bounds"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xcompiler",
    "-fPIC",
    "-Xptxas",
    "-v",
]


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found; the selective-scan library needs CUDA 12.8+")
    return cand


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted(
        (PKG_ROOT.parent / "include").glob("*.h")
    )


def library_path(bounds: bool = False) -> Path:
    return LIB_DIR / (BOUNDS_LIB_NAME if bounds else LIB_NAME)


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build_library(force: bool = False, verbose: bool = False, bounds: bool = False) -> Path:
    nvcc = _nvcc()
    build_dir = BOUNDS_BUILD_DIR if bounds else BUILD_DIR
    build_dir.mkdir(exist_ok=True)
    LIB_DIR.mkdir(exist_ok=True)
    headers = _headers()
    extra = ["-DMSS_BOUNDS_CHECK"] if bounds else []
    objs = []
    jobs = []
    for src in _sources():
        obj = build_dir / (src.stem + ".o")
        objs.append(obj)
        if force or _stale(obj, [src] + headers):
            cmd = [nvcc, *ARCH_FLAGS, *NVCC_FLAGS, *extra, "-c", str(src), "-o", str(obj)]
            jobs.append((src, cmd))

    def run(job):
        src, cmd = job
        r = subprocess.run(cmd, capture_output=True, text=True)
        return src, cmd, r

    with cf.ThreadPoolExecutor(max_workers=max(1, min(len(jobs), os.cpu_count() or 1))) as ex:
        for src, cmd, r in ex.map(run, jobs):
            if r.returncode != 0:
                raise RuntimeError(
                    f"nvcc failed for {src.name}:\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}"
                )
            log = build_dir / (src.stem + ".ptxas.txt")
            log.write_text(r.stdout + r.stderr)
            if verbose:
                sys.stdout.write(r.stderr)

    lib = library_path(bounds)
    if force or jobs or _stale(lib, objs):
        cmd = [nvcc, *ARCH_FLAGS, "-shared", "-o", str(lib), *map(str, objs), "-lcuda"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return lib


if __name__ == "__main__":
    print(build_library(force="--force" in sys.argv, verbose="-v" in sys.argv,
                        bounds="--bounds" in sys.argv))
