"""The reference's own CUDA tests of the hot-path ops, run unchanged against
this package.

The reference's ``tests/gemm/test_cuda.py``, ``tests/norm/test_cuda.py`` and
``tests/activation/test_cuda.py`` import ``aot_kernel`` (the package under
test) and ``ref`` (the torch oracle, ref/gemm.py:4-5, ref/norm.py:11-12,
ref/activation.py:11-16), and their helpers from the reference's
``tests/conftest.py``.  This test runs those files in a child pytest with
this repository's ``aot_kernel`` first on the import path and the installed
reference's ``ref`` after it, and requires every collected case to pass:
that is the drop-in claim for ``from aot_kernel import gemm, rmsnorm, silu``.

The files are staged by ``tests/stage_reference_suite.py`` into
``baseline/_ref/_suite`` (beside the reference's installed packages); the
test is skipped where they are not staged.
"""

from __future__ import annotations

import os
import re
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

REPO = Path(__file__).resolve().parents[1]
REF_INSTALL = REPO / "baseline" / "_ref"
SUITE = REF_INSTALL / "_suite"
FILES = ["tests/gemm/test_cuda.py", "tests/norm/test_cuda.py", "tests/activation/test_cuda.py"]


def _staged() -> bool:
    return (REF_INSTALL / "ref" / "__init__.py").is_file() and all(
        (SUITE / f).is_file() for f in FILES)


def _env() -> dict:
    env = dict(os.environ)
    # this package's aot_kernel shadows the reference's own (also installed
    # under baseline/_ref); ``ref`` comes from the reference install
    env["PYTHONPATH"] = os.pathsep.join([str(REPO / "inference-kernel_b200"), str(REF_INSTALL)])
    return env


@pytest.mark.skipif(not _staged(), reason="reference test files not staged under baseline/_ref/_suite")
def test_reference_cuda_tests_pass_unchanged(tmp_path):
    env = _env()
    which = subprocess.run(
        [sys.executable, "-c", "import aot_kernel, ref; print(aot_kernel.__file__); print(ref.__file__)"],
        cwd=SUITE, env=env, capture_output=True, text=True, timeout=300)
    assert which.returncode == 0, which.stderr[-2000:]
    ak_file, ref_file = which.stdout.split()
    assert Path(ak_file).resolve().is_relative_to(REPO / "inference-kernel_b200"), ak_file
    assert Path(ref_file).resolve().is_relative_to(REF_INSTALL), ref_file

    ini = tmp_path / "pytest.ini"  # the reference's markers (its pyproject.toml stays behind)
    ini.write_text("[pytest]\nmarkers =\n    cuda: requires a CUDA device\n"
                   "    triton: requires triton\n    slow: long-running\n")
    r = subprocess.run(
        [sys.executable, "-m", "pytest", "-q", "-p", "no:cacheprovider", "-c", str(ini),
         "--rootdir", str(SUITE), "--strict-markers", *FILES],
        cwd=SUITE, env=env, capture_output=True, text=True, timeout=900)
    tail = r.stdout[-3000:] + r.stderr[-2000:]
    assert r.returncode == 0, tail
    summary = r.stdout.strip().splitlines()[-1]
    passed = re.search(r"(\d+) passed", summary)
    assert passed and int(passed.group(1)) > 0, summary
    for bad in ("failed", "error", "skipped"):
        assert bad not in summary, summary
