"""Activation wrappers (reference: aot_kernel/activation.py:10-23) plus the
fused ``silu_mul`` = silu(gate) * up used between the gate/up and down
projections of a gated MLP."""

import torch

from . import _C  # noqa: F401  (registers torch.ops.aot_kernel.*)
from .utils import assert_contiguous, assert_is_cuda, assert_same_device, assert_same_dtype


def relu(x: torch.Tensor) -> torch.Tensor:
    assert_is_cuda(x)
    assert_contiguous(x)
    out = torch.empty_like(x)
    torch.ops.aot_kernel.relu_forward(out, x)
    return out


def silu(x: torch.Tensor) -> torch.Tensor:
    assert_is_cuda(x)
    assert_contiguous(x)
    out = torch.empty_like(x)
    torch.ops.aot_kernel.silu_forward(out, x)
    return out


def silu_mul(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """silu(gate) * up in fp32 with one rounding.

    ``gate`` and ``up`` may be contiguous tensors or 2-D views with contiguous
    rows (e.g. ``gu[:, :I]`` and ``gu[:, I:]`` of a fused gate/up projection).
    """
    assert_is_cuda(gate, up)
    assert_same_device(gate, up)
    assert_same_dtype(gate, up)
    if gate.shape != up.shape:
        raise ValueError(f"shape mismatch: gate {tuple(gate.shape)} vs up {tuple(up.shape)}")
    for t in (gate, up):
        if not t.is_contiguous() and not (t.dim() == 2 and t.stride(1) == 1):
            raise ValueError("silu_mul inputs must be contiguous or 2-D views with contiguous rows")
    out = torch.empty(gate.shape, dtype=gate.dtype, device=gate.device)
    torch.ops.aot_kernel.silu_mul_forward(out, gate, up)
    return out
