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


def test_interleave_and_fold_weights_on_cpu():
    """The weight-layout helpers are plain torch and run on any device: the
    interleaved [K, 2I] layout puts gate block j at columns [256j, 256j+128)
    and up block j right after it; folding scales row k by norm_weight[k]
    in fp32 and rounds once."""
    from aot_kernel.gemm import fold_norm_weight, interleave_gate_up

    K, inter = 8, 256
    g = torch.arange(K * inter, dtype=torch.float32).reshape(K, inter).to(torch.bfloat16)
    u = -g
    w = interleave_gate_up(g, u)
    assert w.shape == (K, 2 * inter)
    assert torch.equal(w[:, 0:128], g[:, 0:128]) and torch.equal(w[:, 128:256], u[:, 0:128])
    assert torch.equal(w[:, 256:384], g[:, 128:256]) and torch.equal(w[:, 384:512], u[:, 128:256])
    nw = torch.linspace(0.5, 1.5, K).to(torch.bfloat16)
    f = fold_norm_weight(w, nw)
    assert f.dtype == w.dtype and f.shape == w.shape
    assert torch.equal(f, (w.float() * nw.float().reshape(-1, 1)).to(torch.bfloat16))
    with pytest.raises(ValueError):
        interleave_gate_up(g[:, :100], u[:, :100])  # not a multiple of 128 columns
    with pytest.raises(ValueError):
        fold_norm_weight(w, nw[:-1])


def test_gemm_host_checks_before_device_work():
    from aot_kernel.gemm import gemm_host

    a = torch.zeros(4, 8, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        gemm_host(a, torch.zeros(8, 4, dtype=torch.float32))  # dtype mismatch
    with pytest.raises(ValueError):
        gemm_host(a.float(), torch.zeros(8, 4))  # fp32: tensor-core dtypes only
    with pytest.raises(ValueError):
        gemm_host(a, torch.zeros(7, 4, dtype=torch.bfloat16))  # inner dims
    with pytest.raises(ValueError):
        gemm_host(a.t(), torch.zeros(4, 4, dtype=torch.bfloat16))  # not contiguous
