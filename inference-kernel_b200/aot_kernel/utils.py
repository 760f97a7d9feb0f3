"""Tensor checks shared by the op wrappers.

Error types follow the reference's wrappers (aot_kernel/utils.py:6-36):
ValueError for device / dtype mismatches and non-contiguous inputs,
RuntimeError for tensors that are not on a CUDA device.
"""

import torch


def assert_same_device(*tensors: torch.Tensor) -> torch.device:
    """Returns the common device of `tensors`; ValueError if they differ."""
    if not tensors:
        raise ValueError("assert_same_device needs at least one tensor")
    device = tensors[0].device
    for t in tensors[1:]:
        if t.device != device:
            raise ValueError(f"device mismatch: {device} vs {t.device}")
    return device


def assert_same_dtype(*tensors: torch.Tensor) -> torch.dtype:
    """Returns the common dtype of `tensors`; ValueError if they differ."""
    if not tensors:
        raise ValueError("assert_same_dtype needs at least one tensor")
    dtype = tensors[0].dtype
    for t in tensors[1:]:
        if t.dtype != dtype:
            raise ValueError(f"dtype mismatch: {dtype} vs {t.dtype}")
    return dtype


def assert_contiguous(*tensors: torch.Tensor) -> None:
    for t in tensors:
        if not t.is_contiguous():
            raise ValueError("tensor must be contiguous")


def assert_is_cuda(*tensors: torch.Tensor) -> None:
    for t in tensors:
        if not t.is_cuda:
            raise RuntimeError("tensor must be a CUDA tensor")
