"""Generates the golden vectors in this folder from the reference's own oracle.

Run in the build container, where the reference tree is mounted:

    python tests/golden/make_golden.py --reference /root/reference

It imports the reference's ``ref`` package (torch on CPU), feeds it the seeded
inputs of every case in ``cases.py`` and stores the outputs as bit patterns
(``golden.npz``) plus a manifest with input/output SHA-256 digests
(``manifest.json``).  Nothing at test time reads the reference tree: the
tests regenerate the inputs from the seeds and compare the oracle in
``oracle/`` (and, through it, the kernels) with these files.
"""

from __future__ import annotations

import argparse
import hashlib
import json
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]


def bits(x: np.ndarray, dtype: str) -> np.ndarray:
    from oracle.ops import bf16_bits

    x = np.ascontiguousarray(x, dtype=np.float32)
    if dtype == "bfloat16":
        return bf16_bits(x)
    if dtype == "float16":
        return x.astype(np.float16).view(np.uint16)
    return x.view(np.uint32)


def digest(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def run_reference(ref, case, inputs):
    import torch

    if case.op == "scaled_gemm":
        return run_reference_scaled(case, inputs)
    tdt = {"float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16}[case.dtype]
    t = [torch.from_numpy(np.ascontiguousarray(x)).to(tdt) for x in inputs]
    if case.op == "gemm":
        y = ref.gemm(*t)
    elif case.op == "rmsnorm":
        y = ref.rmsnorm(t[0], t[1], eps=case.eps)
    elif case.op == "add_rmsnorm":
        y = ref.rmsnorm(t[0] + t[1], t[2], eps=case.eps)  # the reference composition
    elif case.op == "silu":
        y = ref.silu(t[0])
    elif case.op == "relu":
        y = ref.relu(t[0])
    elif case.op == "silu_mul":
        y = ref.silu(t[0]) * t[1]
    else:
        raise ValueError(case.op)
    return y.float().numpy()


def run_reference_scaled(case, inputs):
    """The reference's scaled-GEMM oracle, ``_scaled_reference`` of
    tests/gemm/test_triton.py:104-107, on CPU tensors of the case's inputs."""
    import importlib

    import torch

    mod = importlib.import_module("tests.gemm.test_triton")  # the reference's test module
    qt = {"e4m3": torch.float8_e4m3fn, "e5m2": torch.float8_e5m2, "int8": torch.int8}[case.qdtype]
    a_q, b_q, sa, sb = inputs
    a = torch.from_numpy(np.ascontiguousarray(a_q)).view(qt)
    b = torch.from_numpy(np.ascontiguousarray(b_q)).view(qt)
    out_dt = {"float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16}[case.dtype]
    y = mod._scaled_reference(a, b, torch.from_numpy(sa), torch.from_numpy(sb), out_dt)
    return y.float().numpy()


def input_digest(x: np.ndarray, case) -> str:
    if x.dtype in (np.uint8, np.int8) or case.op == "scaled_gemm":
        return digest(x)
    return digest(bits(x, case.dtype))


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("AOTK_REFERENCE_DIR"),
                    required="AOTK_REFERENCE_DIR" not in os.environ,
                    help="reference checkout, read only (default: $AOTK_REFERENCE_DIR)")
    args = ap.parse_args()
    sys.path.insert(0, str(REPO))
    sys.path.insert(0, str(HERE))
    sys.path.insert(0, args.reference)
    import torch

    import ref  # the reference's oracle package
    from cases import all_cases, make_inputs, sampled

    torch.set_num_threads(max(1, torch.get_num_threads()))
    arrays: dict[str, np.ndarray] = {}
    manifest = {"torch": torch.__version__, "numpy": np.__version__, "cases": {}}
    for case in all_cases():
        inputs = make_inputs(case)
        out = run_reference(ref, case, inputs)
        b = bits(out, case.dtype)
        arrays[case.id] = bits(sampled(case, out), case.dtype)
        manifest["cases"][case.id] = {
            "op": case.op,
            "shape": list(case.shape),
            "dtype": case.dtype,
            "eps": case.eps,
            "sample_rows": case.sample_rows,
            "input_sha256": [input_digest(x, case) for x in inputs],
            "output_sha256": digest(b),
        }
        print(f"{case.id}: {out.shape}")
    np.savez_compressed(HERE / "golden.npz", **arrays)
    (HERE / "manifest.json").write_text(json.dumps(manifest, indent=1, sort_keys=True) + "\n")
    print(f"wrote {len(arrays)} cases")


if __name__ == "__main__":
    main()
