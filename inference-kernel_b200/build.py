"""Builds the two native libraries of this package in place.

* ``aot_kernel/libaotk.so`` - every CUDA kernel plus the C ABI declared in
  ``include/aotk.h``; compiled by nvcc for sm_100a only, static cudart, no
  torch dependency (loadable through ctypes by any host program).
* ``aot_kernel/_C.<abi>.so`` - the torch operator library ``aot_kernel``
  (``csrc/registration.cc``), linked against libaotk.so (rpath ``$ORIGIN``).

Usage: ``python inference-kernel_b200/build.py [--clean] [--verbose]``.
Objects are rebuilt only when a source or header is newer than them.  The
CMake/scikit-build project at the repository root builds the same sources.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
import sysconfig
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
REPO = PKG_DIR.parent
CSRC = PKG_DIR / "csrc"
INCLUDE = REPO / "include"
OUT_DIR = PKG_DIR / "aot_kernel"
OBJ_DIR = PKG_DIR / "_build" / "obj"
CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
NVCC = str(CUDA_HOME / "bin" / "nvcc")

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    *ARCH_FLAGS,
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    f"-I{INCLUDE}",
    f"-I{CSRC}",
]


def _headers() -> list[Path]:
    return sorted(list(CSRC.glob("*.h")) + list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h")))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _run(cmd: list[str], verbose: bool) -> None:
    if verbose:
        print(" ".join(cmd), flush=True)
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        sys.stderr.write(proc.stdout + proc.stderr)
        raise RuntimeError(f"build step failed: {' '.join(cmd[:3])} ... (exit {proc.returncode})")
    if verbose and (proc.stdout or proc.stderr):
        sys.stderr.write(proc.stdout + proc.stderr)


def _compile_cu(src: Path, verbose: bool, extra: list[str]) -> Path:
    obj = OBJ_DIR / (src.stem + ".o")
    if _stale(obj, [src, *_headers()]):
        _run([NVCC, *NVCC_FLAGS, *extra, "-c", str(src), "-o", str(obj)], verbose)
    return obj


def build_libaotk(verbose: bool = False, jobs: int | None = None, extra: list[str] | None = None) -> Path:
    """Compiles csrc/*.cu and links aot_kernel/libaotk.so."""
    OBJ_DIR.mkdir(parents=True, exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    with cf.ThreadPoolExecutor(max_workers=jobs or os.cpu_count() or 4) as ex:
        objs = list(ex.map(lambda s: _compile_cu(s, verbose, extra or []), sources))
    lib = OUT_DIR / "libaotk.so"
    if _stale(lib, objs):
        _run(
            [NVCC, *ARCH_FLAGS, "-shared", "--cudart", "static", "-o", str(lib), *map(str, objs)],
            verbose,
        )
    return lib


def build_torch_ext(verbose: bool = False) -> Path:
    """Compiles csrc/registration.cc into the aot_kernel._C extension module."""
    import torch
    from torch.utils import cpp_extension

    suffix = sysconfig.get_config_var("EXT_SUFFIX") or ".so"
    target = OUT_DIR / f"_C{suffix}"
    lib = OUT_DIR / "libaotk.so"
    src = CSRC / "registration.cc"
    if not _stale(target, [src, lib, *_headers()]):
        return target
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    includes = [*cpp_extension.include_paths(device_type="cuda"), sysconfig.get_paths()["include"]]
    torch_lib = Path(torch.__file__).resolve().parent / "lib"
    cmd = [
        "g++",
        "-O2",
        "-std=c++17",
        "-fPIC",
        "-shared",
        f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
        "-DTORCH_EXTENSION_NAME=_C",
        *[f"-I{p}" for p in includes],
        f"-I{INCLUDE}",
        str(src),
        "-o",
        str(target),
        f"-L{OUT_DIR}",
        "-laotk",
        f"-L{torch_lib}",
        "-lc10",
        "-lc10_cuda",
        "-ltorch_cpu",
        "-ltorch",
        "-Wl,-rpath,$ORIGIN",
        f"-Wl,-rpath,{torch_lib}",
    ]
    _run(cmd, verbose)
    return target


def build(verbose: bool = False, torch_ext: bool = True) -> None:
    build_libaotk(verbose)
    if torch_ext:
        build_torch_ext(verbose)


def clean() -> None:
    shutil.rmtree(PKG_DIR / "_build", ignore_errors=True)
    for p in OUT_DIR.glob("*.so"):
        p.unlink()


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--clean", action="store_true")
    ap.add_argument("--verbose", "-v", action="store_true")
    ap.add_argument("--no-torch", action="store_true", help="build libaotk.so only")
    args = ap.parse_args()
    if args.clean:
        clean()
    build(verbose=args.verbose, torch_ext=not args.no_torch)
    print(f"built {OUT_DIR / 'libaotk.so'}")


if __name__ == "__main__":
    main()
