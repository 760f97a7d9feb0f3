"""RMSNorm wrapper (reference: aot_kernel/norm.py:9-18)."""

import torch

from . import _C  # noqa: F401  (registers torch.ops.aot_kernel.*)
from .utils import assert_contiguous, assert_same_device, assert_same_dtype


def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """y = x * rsqrt(mean(x**2, -1) + eps) * weight over the last dim, fp32 math."""
    if not x.is_cuda:
        raise ValueError("cuda rmsnorm requires a CUDA tensor")
    assert_contiguous(x, weight)
    assert_same_device(x, weight)
    assert_same_dtype(x, weight)
    out = torch.empty_like(x)
    torch.ops.aot_kernel.rmsnorm_forward(out, x, weight, eps)
    return out


rms_norm = rmsnorm


def add_rmsnorm(x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor,
                eps: float = 1e-6) -> tuple[torch.Tensor, torch.Tensor]:
    """(rmsnorm(h, weight, eps), h) with h = x + residual rounded to the dtype.

    The pre-norm step of a transformer block in one pass: equal to
    ``rmsnorm(x + residual, weight, eps)`` and ``x + residual``.
    """
    if not x.is_cuda:
        raise ValueError("cuda add_rmsnorm requires a CUDA tensor")
    assert_contiguous(x, residual, weight)
    assert_same_device(x, residual, weight)
    assert_same_dtype(x, residual, weight)
    if x.shape != residual.shape:
        raise ValueError(f"shape mismatch: x {tuple(x.shape)} vs residual {tuple(residual.shape)}")
    out = torch.empty_like(x)
    h = torch.empty_like(x)
    torch.ops.aot_kernel.add_rmsnorm_forward(out, h, x, residual, weight, eps)
    return out, h


def rms_rstd(x: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """fp32 rsqrt(mean(x**2, -1) + eps), one value per row: rms_norm's row
    statistic, for folding the normalisation into the next GEMM
    (``gemm_silu_mul(x, fold_norm_weight(w_gate_up, w), row_scale=rstd)``)."""
    if not x.is_cuda:
        raise ValueError("cuda rms_rstd requires a CUDA tensor")
    assert_contiguous(x)
    rstd = torch.empty(x.shape[:-1], dtype=torch.float32, device=x.device)
    torch.ops.aot_kernel.rmsnorm_rstd(rstd, x, eps)
    return rstd
