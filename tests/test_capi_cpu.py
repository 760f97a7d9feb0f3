"""The C ABI without a GPU: libaotk.so loads, exports every entry point that
include/aotk.h declares, and rejects bad arguments with status codes before
touching the device.  The torch extension loads and registers the reference's
operator schemas."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from aot_kernel import capi

HEADER = Path(__file__).resolve().parents[1] / "include" / "aotk.h"


def declared_symbols() -> list[str]:
    text = HEADER.read_text()
    return sorted(set(re.findall(r"AOTK_API\s+[\w\s\*]*?\b(aotk_\w+)\s*\(", text)))


def test_header_declares_entry_points():
    syms = declared_symbols()
    assert "aotk_gemm_opt" in syms and "aotk_rmsnorm_forward" in syms and len(syms) >= 11


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(str(capi.LIB_PATH))
    missing = [s for s in declared_symbols() if not hasattr(lib, s)]
    assert not missing, f"libaotk.so lacks {missing}"


def test_binding_covers_header():
    assert set(capi.SIGNATURES) | {"aotk_last_error"} == set(declared_symbols())


def test_version():
    assert capi.load().aotk_version() >= 100


@pytest.mark.parametrize(
    "call,status",
    [
        (lambda: capi.gemm_opt(256, 256, 256, 4, 4, 4, 0), capi.ERR_UNSUPPORTED),  # fp32 on the tensor-core path (rejected before any device access)
        (lambda: capi.gemm_opt(0, 0, 0, -1, 4, 4, 2), capi.ERR_INVALID_ARGUMENT),  # negative M
        (lambda: capi.gemm(0, 0, 0, 4, 4, 4, 7), capi.ERR_UNSUPPORTED),           # unknown dtype
        (lambda: capi.gemm_opt(None, None, None, 4, 4, 4, 2), capi.ERR_INVALID_ARGUMENT),
        (lambda: capi.silu_forward(0, 0, -5, 2), capi.ERR_INVALID_ARGUMENT),
        (lambda: capi.relu_forward(None, None, 8, 2), capi.ERR_INVALID_ARGUMENT),
        (lambda: capi.rmsnorm_forward(0, 0, 0, -1, 8, 1e-6, 2), capi.ERR_INVALID_ARGUMENT),
        (lambda: capi.silu_mul_forward(8, 4, 8, 4, 8, 4, 2, 8, 2), capi.ERR_INVALID_ARGUMENT),  # stride < cols
        # scaled GEMM: 16-bit input, bad output dtype, bad scale mode, null scale, negative size
        (lambda: capi.scaled_gemm(16, 16, 16, 16, 16, 4, 4, 4, capi.BFLOAT16, capi.BFLOAT16,
                                  capi.SCALE_TENSOR), capi.ERR_UNSUPPORTED),
        (lambda: capi.scaled_gemm(16, 16, 16, 16, 16, 4, 4, 4, capi.INT8, capi.INT8,
                                  capi.SCALE_TENSOR), capi.ERR_UNSUPPORTED),
        (lambda: capi.scaled_gemm(16, 16, 16, 16, 16, 4, 4, 4, capi.FLOAT8_E4M3, capi.BFLOAT16,
                                  7), capi.ERR_INVALID_ARGUMENT),
        (lambda: capi.scaled_gemm(16, 16, 16, None, 16, 4, 4, 4, capi.FLOAT8_E4M3, capi.BFLOAT16,
                                  capi.SCALE_ROW), capi.ERR_INVALID_ARGUMENT),
        (lambda: capi.scaled_gemm_simt(16, 16, 16, 16, 16, 4, -4, 4, capi.INT8, capi.FLOAT32,
                                       capi.SCALE_ROW), capi.ERR_INVALID_ARGUMENT),
        (lambda: capi.scaled_gemm_tc(16, 16, 16, 16, 16, 4, 4, 0, capi.FLOAT8_E5M2, capi.FLOAT16,
                                     capi.SCALE_ROW), capi.ERR_INVALID_ARGUMENT),  # empty K
        # host-buffer GEMM: fp32, null device buffer, negative size
        (lambda: capi.gemm_host(16, 16, 16, 4, 4, 4, capi.FLOAT32, 16, 16, 16),
         capi.ERR_UNSUPPORTED),
        (lambda: capi.gemm_host(16, 16, 16, 4, 4, 4, capi.BFLOAT16, None, 16, 16),
         capi.ERR_INVALID_ARGUMENT),
        (lambda: capi.gemm_host(16, 16, 16, -4, 4, 4, capi.BFLOAT16, 16, 16, 16),
         capi.ERR_INVALID_ARGUMENT),
    ],
)
def test_argument_errors_without_device(call, status):
    with pytest.raises(capi.AotkError) as exc:
        call()
    assert exc.value.status == status
    assert capi.load().aotk_last_error()


def test_empty_problems_are_no_ops():
    capi.gemm_opt(0, 0, 0, 0, 16, 16, capi.BFLOAT16)
    capi.silu_forward(0, 0, 0, capi.BFLOAT16)
    capi.rmsnorm_forward(0, 0, 0, 0, 4096, 1e-6, capi.BFLOAT16)
    capi.silu_mul_forward(0, 0, 0, 0, 0, 0, 0, 16, capi.BFLOAT16)
    capi.scaled_gemm(0, 0, 0, 0, 0, 0, 16, 16, capi.INT8, capi.BFLOAT16, capi.SCALE_TENSOR)
    capi.gemm_host(0, 0, 0, 0, 16, 16, capi.BFLOAT16, 0, 0, 0)
    assert capi.scaled_gemm_workspace_size(256, 250, 256, capi.FLOAT8_E4M3) == 0  # N % 16 != 0


def test_torch_extension_registers_reference_schemas():
    import torch

    import aot_kernel  # noqa: F401

    ops = torch.ops.aot_kernel
    for name in ("gemm", "gemm_opt", "rmsnorm_forward", "silu_forward", "relu_forward",
                 "silu_mul_forward", "add_rmsnorm_forward", "gemm_silu_mul", "scaled_gemm"):
        assert hasattr(ops, name)
    schema = ops.scaled_gemm.default._schema
    assert [a.name for a in schema.arguments] == ["out", "a", "b", "scale_a", "scale_b", "optimized"]
    schema = ops.rmsnorm_forward.default._schema
    assert [a.name for a in schema.arguments] == ["out", "x", "weight", "eps"]
    assert schema.arguments[0].alias_info.is_write and str(schema.arguments[3].type) == "float"
    assert len(schema.returns) == 0
