"""Seeded synthetic inputs shared by the oracle, the tests, smoke() and bench.py.

TEST INFRASTRUCTURE.  Values are drawn as float32 from numpy's PCG64 generator
(bit-reproducible across machines), scaled, then rounded to the target dtype,
so the oracle and the GPU kernels see identical bits.
"""

from __future__ import annotations

import numpy as np

from .ops import fp8_encode, round_to


def randn(shape, seed: int, dtype: str = "bfloat16", mean: float = 0.0, std: float = 1.0) -> np.ndarray:
    """float32 array of N(mean, std) samples rounded to `dtype` ("float32"/"float16"/"bfloat16")."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal(size=tuple(shape), dtype=np.float32)
    if std != 1.0:
        x = x * np.float32(std)
    if mean != 0.0:
        x = x + np.float32(mean)
    return round_to(x, dtype)


def quantized(shape, seed: int, qdtype: str) -> np.ndarray:
    """8-bit GEMM inputs as the reference's tests draw them
    (tests/gemm/test_triton.py:85-93): fp8 = N(0, 1) float32 samples converted
    to the format (uint8 codes); int8 = integers uniform in [-8, 8)."""
    rng = np.random.default_rng(seed)
    if qdtype == "int8":
        return rng.integers(-8, 8, size=tuple(shape), dtype=np.int8)
    x = rng.standard_normal(size=tuple(shape), dtype=np.float32)
    return fp8_encode(x, qdtype)


def scales(M: int, N: int, mode: str, seed: int):
    """Dequantisation scales as the reference's tests draw them
    (tests/gemm/test_triton.py:96-101): tensorwise 0.05 and 0.03; rowwise
    U(0, 1) * 0.1 + 0.01 of length M and N (float32)."""
    if mode == "tensor":
        return np.array([0.05], np.float32), np.array([0.03], np.float32)
    rng = np.random.default_rng(seed)
    sa = rng.random(M, dtype=np.float32) * np.float32(0.1) + np.float32(0.01)
    sb = rng.random(N, dtype=np.float32) * np.float32(0.1) + np.float32(0.01)
    return sa.astype(np.float32), sb.astype(np.float32)
