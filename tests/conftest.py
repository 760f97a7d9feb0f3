"""Shared pytest configuration.

* ``gpu`` marks tests that need a B200; they are skipped when CUDA is absent.
* Tolerances are the reference's (tests/conftest.py:47-100 of
  gongyisheng/inference-kernel) plus the GEMM bound
  max|err| <= 2e-2 * max|ref| for 16-bit outputs.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parents[1]
for p in (REPO, REPO / "inference-kernel_b200", REPO / "tests" / "golden"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config: pytest.Config) -> None:
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU")
    config.addinivalue_line("markers", "slow: long-running")


def pytest_collection_modifyitems(config, items):
    try:
        import torch

        has_gpu = torch.cuda.is_available()
    except ImportError:
        has_gpu = False
    if has_gpu:
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


# tolerances: dtype name -> (rtol, atol)
TOL_COMMON = {"float32": (1e-5, 1e-6), "float16": (1e-3, 1e-3), "bfloat16": (1e-2, 1e-2)}
TOL_GEMM = {"float32": (1e-4, 1e-4), "float16": (1e-2, 1e-2), "bfloat16": (2e-2, 2e-2)}
GEMM_MAX_ERR_FRAC = 2e-2  # max|err| <= 2e-2 * max|ref| (16-bit GEMM outputs)
ELEM_MAX_ERR_FRAC = 1e-2  # rms_norm / silu: relative 1e-2


def _as_np(x) -> np.ndarray:
    if isinstance(x, np.ndarray):
        return x.astype(np.float32)
    return x.detach().float().cpu().numpy()


def assert_close_np(actual, expected, rtol: float, atol: float) -> None:
    a, e = _as_np(actual), _as_np(expected)
    assert a.shape == e.shape, f"shape {a.shape} != {e.shape}"
    nan_a, nan_e = np.isnan(a), np.isnan(e)
    assert np.array_equal(nan_a, nan_e), "NaN positions differ"
    ok = np.isclose(a, e, rtol=rtol, atol=atol) | nan_a
    if not ok.all():
        idx = np.argwhere(~ok)[:5]
        bad = [(tuple(i), float(a[tuple(i)]), float(e[tuple(i)])) for i in idx]
        raise AssertionError(f"{(~ok).sum()} / {ok.size} mismatches (rtol={rtol}, atol={atol}): {bad}")


def assert_close_common(actual, expected, dtype: str) -> None:
    assert_close_np(actual, expected, *TOL_COMMON[dtype])


def assert_close_for_gemm(actual, expected, dtype: str) -> None:
    assert_close_np(actual, expected, *TOL_GEMM[dtype])
    if dtype != "float32":
        assert_max_err_frac(actual, expected, GEMM_MAX_ERR_FRAC)


def assert_max_err_frac(actual, expected, frac: float) -> None:
    a, e = _as_np(actual), _as_np(expected)
    scale = float(np.nanmax(np.abs(e))) if e.size else 0.0
    err = float(np.nanmax(np.abs(a - e))) if e.size else 0.0
    assert err <= frac * scale + 1e-30, f"max|err| {err:.3e} > {frac} * max|ref| {scale:.3e}"


TORCH_DTYPES = {}


def torch_dtype(name: str):
    import torch

    return {"float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16}[name]


def to_device(x: np.ndarray, dtype: str, device="cuda"):
    """Exact transfer of oracle inputs (float32 values representable in dtype) to a torch tensor."""
    import torch

    return torch.from_numpy(np.ascontiguousarray(x)).to(device=device, dtype=torch_dtype(dtype))


@pytest.fixture(params=["float32", "float16", "bfloat16"], ids=["fp32", "fp16", "bf16"])
def dtype(request) -> str:
    return request.param


@pytest.fixture(scope="session")
def device():
    import torch

    return torch.device("cuda")
