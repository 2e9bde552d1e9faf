"""The CMake recipe (jax-mambas_b200/CMakeLists.txt) builds the same library as
build.py: configured and built for sm_100a into a temporary directory, it
exports exactly the mamba_ss_* symbols of the build.py library, and those are
every entry point include/*.h declares. nvcc cross-compiles, so no GPU is
needed (about a minute and a half of compiling)."""
import os
import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / "jax-mambas_b200"


def _exported(lib):
    out = subprocess.run(["nm", "-D", "--defined-only", str(lib)], capture_output=True,
                         text=True, check=True).stdout
    return {line.split()[-1] for line in out.splitlines()
            if line.split() and line.split()[-1].startswith("mamba_ss_")}


@pytest.mark.skipif(shutil.which("cmake") is None or shutil.which("nvcc") is None,
                    reason="cmake and nvcc are needed")
@pytest.mark.timeout(900)
def test_cmake_builds_the_same_library(tmp_path):
    import importlib.util

    spec = importlib.util.spec_from_file_location("mamba_ss_build", PKG / "build.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    ref_lib = mod.build_library()

    env = dict(os.environ)
    subprocess.run(["cmake", "-S", str(PKG), "-B", str(tmp_path), "-DCMAKE_BUILD_TYPE=Release"],
                   check=True, capture_output=True, env=env)
    subprocess.run(["cmake", "--build", str(tmp_path), "-j", str(os.cpu_count() or 4)],
                   check=True, capture_output=True, env=env)
    lib = tmp_path / "libmamba_ss_b200.so"
    assert lib.is_file()
    assert _exported(lib) == _exported(ref_lib)

    from test_capi import _declared_symbols

    assert set(_declared_symbols()) <= _exported(lib)
