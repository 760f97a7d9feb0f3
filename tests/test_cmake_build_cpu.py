"""The CMake / scikit-build-core project at the repository root (the build
the reference's own packaging uses: CMakeLists.txt:25-45 of
gongyisheng/inference-kernel, with CMAKE_CUDA_ARCHITECTURES=100a here):
configured and built into a temporary directory without a GPU, it yields
libaotk.so exporting every entry point of include/aotk.h, compiled for
sm_100a, and a ``_C`` module that registers the ``aot_kernel`` operators."""

from __future__ import annotations

import ctypes
import os
import shutil
import subprocess
import sys
from pathlib import Path

import pytest

from tests.test_capi_cpu import declared_symbols

REPO = Path(__file__).resolve().parents[1]

pytestmark = pytest.mark.skipif(shutil.which("cmake") is None or shutil.which("ninja") is None,
                                reason="cmake / ninja not installed")


@pytest.fixture(scope="module")
def cmake_build(tmp_path_factory):
    out = tmp_path_factory.mktemp("cmake_build")
    cfg = subprocess.run(["cmake", "-S", str(REPO), "-B", str(out), "-G", "Ninja",
                          "-DCMAKE_BUILD_TYPE=Release", f"-DPython_EXECUTABLE={sys.executable}"],
                         capture_output=True, text=True, timeout=600)
    assert cfg.returncode == 0, cfg.stdout[-2000:] + cfg.stderr[-2000:]
    bld = subprocess.run(["cmake", "--build", str(out), "-j", str(os.cpu_count() or 4)],
                         capture_output=True, text=True, timeout=1200)
    assert bld.returncode == 0, bld.stdout[-3000:] + bld.stderr[-3000:]
    return out


def test_cmake_compiles_for_sm100a_only(cmake_build):
    flags = (cmake_build / "build.ninja").read_text()
    assert "arch=compute_100a" in flags and "sm_100a" in flags
    for other in ("sm_90", "sm_120", "sm_80"):
        assert other not in flags


def test_cmake_library_exports_every_declared_symbol(cmake_build):
    lib = ctypes.CDLL(str(cmake_build / "libaotk.so"))
    missing = [s for s in declared_symbols() if not hasattr(lib, s)]
    assert not missing, f"CMake-built libaotk.so lacks {missing}"


def test_cmake_torch_module_registers_operators(cmake_build):
    mods = list(cmake_build.glob("_C*.so"))
    assert len(mods) == 1, mods
    # a fresh interpreter: the in-tree _C may already hold the library name here
    code = (
        "import importlib.util, torch, sys\n"
        f"spec = importlib.util.spec_from_file_location('_C', r'{mods[0]}')\n"
        "m = importlib.util.module_from_spec(spec); spec.loader.exec_module(m)\n"
        "names = ['gemm', 'gemm_opt', 'rmsnorm_forward', 'silu_forward', 'relu_forward',\n"
        "         'silu_mul_forward', 'gemm_silu_mul', 'scaled_gemm']\n"
        "missing = [n for n in names if not hasattr(torch.ops.aot_kernel, n)]\n"
        "print('missing', missing); sys.exit(1 if missing else 0)\n")
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
