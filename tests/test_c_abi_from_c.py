"""The C ABI from a plain C program: tests/c/abi_from_c.c is compiled with gcc
against include/aotk.h, linked with libaotk.so and run.  Only entry points
that finish before device work are called, so this runs without a GPU; it
shows that a non-Python, non-torch host binds the library with nothing but
the header and the shared object."""

from __future__ import annotations

import shutil
import subprocess
from pathlib import Path

import pytest

from aot_kernel import capi

REPO = Path(__file__).resolve().parents[1]


@pytest.mark.skipif(shutil.which("gcc") is None, reason="gcc not available")
def test_c_program_binds_the_abi(tmp_path):
    exe = tmp_path / "abi_from_c"
    lib_dir = capi.LIB_PATH.parent
    subprocess.run(
        ["gcc", "-std=c11", "-Wall", "-Werror", str(REPO / "tests" / "c" / "abi_from_c.c"),
         f"-I{REPO / 'include'}", f"-L{lib_dir}", "-laotk", f"-Wl,-rpath,{lib_dir}", "-o",
         str(exe)],
        check=True, capture_output=True, text=True)
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert run.returncode == 0, run.stdout + run.stderr
    assert run.stdout.count("ok ") == 7
