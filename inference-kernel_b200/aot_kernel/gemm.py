"""GEMM wrappers: ``gemm`` (tensor-core path) and ``gemm_naive`` (SIMT path).

Mirrors aot_kernel/gemm.py:22-51 of the reference: validate, allocate ``out``,
call the registered op.  ``gemm`` sends fp16/bf16 to ``gemm_opt``, which picks
the persistent tcgen05 kernel (M > 128), the skinny split-K tcgen05 kernel
(M <= 128) or, for shapes TMA cannot address, the SIMT kernel; fp32 goes to
the SIMT ``gemm`` op, as in the reference.
"""

import torch

from . import _C  # noqa: F401  (registers torch.ops.aot_kernel.*)
from .utils import assert_contiguous, assert_is_cuda, assert_same_device, assert_same_dtype

_TENSOR_CORE_DTYPES = (torch.float16, torch.bfloat16)


def _validate(a: torch.Tensor, b: torch.Tensor):
    assert_is_cuda(a, b)
    assert_contiguous(a, b)
    device = assert_same_device(a, b)
    dtype = assert_same_dtype(a, b)
    if a.dim() != 2 or b.dim() != 2:
        raise ValueError(f"gemm expects 2D tensors, got a.dim={a.dim()} b.dim={b.dim()}")
    if a.size(1) != b.size(0):
        raise ValueError(f"inner dims mismatch: {a.size(1)} vs {b.size(0)}")
    return device, dtype


def gemm(a: torch.Tensor, b: torch.Tensor, *, out: torch.Tensor | None = None) -> torch.Tensor:
    """C = A @ B with fp32 accumulation and one rounding to the input dtype.

    ``out`` (keyword-only, not in the reference signature) may name a
    contiguous [M, N] tensor to write into, e.g. a row slice of a larger buffer.
    """
    device, dtype = _validate(a, b)
    if out is None:
        out = torch.empty((a.size(0), b.size(1)), device=device, dtype=dtype)
    if dtype in _TENSOR_CORE_DTYPES:
        torch.ops.aot_kernel.gemm_opt(out, a, b)
    else:
        torch.ops.aot_kernel.gemm(out, a, b)
    return out


def gemm_naive(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """C = A @ B on the SIMT kernel (any dtype, any shape)."""
    device, dtype = _validate(a, b)
    out = torch.empty((a.size(0), b.size(1)), device=device, dtype=dtype)
    torch.ops.aot_kernel.gemm(out, a, b)
    return out
