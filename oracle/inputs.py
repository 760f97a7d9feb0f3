"""Seeded synthetic inputs shared by the oracle, the tests, smoke() and bench.py.

TEST INFRASTRUCTURE.  Values are drawn as float32 from numpy's PCG64 generator
(bit-reproducible across machines), scaled, then rounded to the target dtype,
so the oracle and the GPU kernels see identical bits.
"""

from __future__ import annotations

import numpy as np

from .ops import round_to


def randn(shape, seed: int, dtype: str = "bfloat16", mean: float = 0.0, std: float = 1.0) -> np.ndarray:
    """float32 array of N(mean, std) samples rounded to `dtype` ("float32"/"float16"/"bfloat16")."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal(size=tuple(shape), dtype=np.float32)
    if std != 1.0:
        x = x * np.float32(std)
    if mean != 0.0:
        x = x + np.float32(mean)
    return round_to(x, dtype)
