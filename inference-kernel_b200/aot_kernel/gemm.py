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


GATE_UP_BLOCK = 128  # column block of the interleaved gate/up layout


def interleave_gate_up(w_gate: torch.Tensor, w_up: torch.Tensor) -> torch.Tensor:
    """[K, I] gate and up weights -> the [K, 2I] layout ``gemm_silu_mul`` reads:
    columns [256j, 256j+128) are gate block j, [256j+128, 256j+256) up block j."""
    if w_gate.shape != w_up.shape or w_gate.dim() != 2:
        raise ValueError("gate and up weights must be 2-D and of the same shape")
    K, inter = w_gate.shape
    if inter % GATE_UP_BLOCK:
        raise ValueError(f"intermediate size {inter} is not a multiple of {GATE_UP_BLOCK}")
    g = w_gate.reshape(K, inter // GATE_UP_BLOCK, 1, GATE_UP_BLOCK)
    u = w_up.reshape(K, inter // GATE_UP_BLOCK, 1, GATE_UP_BLOCK)
    return torch.cat([g, u], dim=2).reshape(K, 2 * inter).contiguous()


def gemm_silu_mul(a: torch.Tensor, w_gate_up: torch.Tensor) -> torch.Tensor:
    """silu(a @ W_gate) * (a @ W_up) in one kernel; ``w_gate_up`` from
    ``interleave_gate_up``.  The gate/up product stays in TMEM: silu and the
    product use the fp32 accumulators and the result is rounded once."""
    device, dtype = _validate(a, w_gate_up)
    if dtype not in _TENSOR_CORE_DTYPES:
        raise ValueError(f"gemm_silu_mul supports fp16/bf16, got {dtype}")
    out = torch.empty((a.size(0), w_gate_up.size(1) // 2), device=device, dtype=dtype)
    torch.ops.aot_kernel.gemm_silu_mul(out, a, w_gate_up)
    return out
