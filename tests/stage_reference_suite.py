"""Stages the reference's own hot-path test files for
``tests/test_reference_suite_cuda.py``.

Run in the build container, where the reference tree is mounted, after the
reference has been installed into ``baseline/_ref`` (its ``ref`` package is
the oracle those tests import):

    python tests/stage_reference_suite.py --reference <reference checkout>

It copies, unmodified, the reference's ``tests/__init__.py``,
``tests/conftest.py`` and the CUDA test modules of the three hot-path ops
(``tests/gemm/test_cuda.py``, ``tests/norm/test_cuda.py``,
``tests/activation/test_cuda.py``, with their package ``__init__.py``) into
``baseline/_ref/_suite/tests/``.  ``baseline/_ref`` is kept out of version
control; it travels with the working tree to the machine that runs the GPU
tests, where the reference checkout itself is absent.
"""

from __future__ import annotations

import argparse
import shutil
from pathlib import Path

REPO = Path(__file__).resolve().parents[1]
SUITE = REPO / "baseline" / "_ref" / "_suite"
FILES = ("tests/__init__.py", "tests/conftest.py",
         "tests/gemm/__init__.py", "tests/gemm/test_cuda.py",
         "tests/norm/__init__.py", "tests/norm/test_cuda.py",
         "tests/activation/__init__.py", "tests/activation/test_cuda.py")


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--reference", required=True, type=Path,
                    help="root of the reference checkout (holds tests/ and ref/)")
    args = ap.parse_args()
    for rel in FILES:
        src = args.reference / rel
        if not src.is_file():
            raise SystemExit(f"missing {src}")
        dst = SUITE / rel
        dst.parent.mkdir(parents=True, exist_ok=True)
        shutil.copyfile(src, dst)
    print(f"staged {len(FILES)} files under {SUITE}")


if __name__ == "__main__":
    main()
