"""Input validation of the Python wrappers, which runs before any device
work: the reference's rejection tests (tests/gemm/test_cuda.py:55-83,
tests/norm/test_cuda.py:49-67, tests/activation/test_cuda.py:25-41)."""

import pytest
import torch

import aot_kernel
from aot_kernel.activation import relu, silu, silu_mul
from aot_kernel.gemm import gemm, gemm_naive
from aot_kernel.norm import rmsnorm


def test_public_names():
    assert set(aot_kernel.__all__) >= {"gemm", "gemm_naive", "relu", "rmsnorm", "rms_norm", "silu",
                                       "silu_mul"}
    assert aot_kernel.rms_norm is aot_kernel.rmsnorm


@pytest.mark.parametrize("fn", [gemm, gemm_naive])
def test_gemm_rejects_cpu_tensor(fn):
    with pytest.raises((ValueError, RuntimeError)):
        fn(torch.randn(8, 16), torch.randn(16, 8))


def test_rmsnorm_rejects_cpu_tensor():
    with pytest.raises((ValueError, RuntimeError)):
        rmsnorm(torch.randn(8, 16), torch.randn(16))


@pytest.mark.parametrize("fn", [silu, relu])
def test_activation_rejects_cpu_tensor(fn):
    with pytest.raises((ValueError, RuntimeError)):
        fn(torch.randn(8))


def test_silu_mul_rejects_cpu_tensor():
    with pytest.raises((ValueError, RuntimeError)):
        silu_mul(torch.randn(8), torch.randn(8))


def test_scaled_gemm_checks_before_device_work():
    """The reference's scaled_gemm checks (jit_kernel/gemm.py:207-226): 2-D
    inputs (AssertionError), CUDA tensors (RuntimeError), matching K."""
    from aot_kernel.gemm import scaled_gemm

    a = torch.zeros(8, 16, dtype=torch.int8)
    b = torch.zeros(16, 8, dtype=torch.int8)
    s = torch.ones(1)
    with pytest.raises(AssertionError):
        scaled_gemm(torch.zeros(8, dtype=torch.int8), b, s, s)
    with pytest.raises(RuntimeError):
        scaled_gemm(a, b, s, s)
    assert "scaled_gemm" in aot_kernel.__all__
