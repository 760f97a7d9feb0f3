"""numpy restatement of the reference oracle's arithmetic.  TEST INFRASTRUCTURE.

All inputs are float32 arrays whose values are exactly representable in the
op's dtype ("float32", "float16" or "bfloat16"); outputs are float32 arrays
holding values of that dtype.  Each function cites the reference call site it
restates and the PyTorch 2.11.0 behaviour of that call on CPU tensors.
"""

from __future__ import annotations

import numpy as np

DTYPES = ("float32", "float16", "bfloat16")


# ---- rounding ---------------------------------------------------------------

def bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bfloat16 bit patterns (uint16), round to nearest even; NaN stays NaN."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    rounded = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    nan = np.isnan(x)
    if nan.any():
        rounded = rounded.copy()
        rounded[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return rounded


def bf16_from_bits(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def round_to(x: np.ndarray, dtype: str) -> np.ndarray:
    """Rounds float32 values to `dtype` (RNE) and returns them as float32."""
    x = np.asarray(x, dtype=np.float32)
    if dtype == "float32":
        return x
    if dtype == "float16":
        with np.errstate(over="ignore"):
            return x.astype(np.float16).astype(np.float32)
    if dtype == "bfloat16":
        return bf16_from_bits(bf16_bits(x))
    raise ValueError(f"unsupported dtype {dtype!r}")


# ---- ops --------------------------------------------------------------------

def gemm(a: np.ndarray, b: np.ndarray, dtype: str) -> np.ndarray:
    """ref.gemm = ``a @ b`` (ref/gemm.py:4-5).

    torch CPU matmul of fp16/bf16 tensors multiplies exactly in fp32,
    accumulates in fp32 and rounds each output once to the input dtype; fp32
    inputs accumulate in fp32.  Restated as a float32 matmul (BLAS sgemm)
    followed by one rounding.  Summation order differs from torch's, which is
    why the golden comparison allows a few output ulps.
    """
    a = np.ascontiguousarray(a, dtype=np.float32)
    b = np.ascontiguousarray(b, dtype=np.float32)
    return round_to(a @ b, dtype)


def rmsnorm(x: np.ndarray, weight: np.ndarray, eps: float, dtype: str) -> np.ndarray:
    """ref.rmsnorm = ``F.rms_norm(x, weight.shape, weight, eps)`` (ref/norm.py:11-12).

    torch 2.11 upcasts 16-bit inputs to fp32, forms mean(x^2) over the last
    dim, multiplies x by rsqrt(mean + eps) and then by the weight, all in fp32,
    and rounds once to the input dtype (checked bit-for-bit against the
    reference in tests/golden).
    """
    x = np.asarray(x, dtype=np.float32)
    w = np.asarray(weight, dtype=np.float32)
    ms = np.mean(x * x, axis=-1, keepdims=True, dtype=np.float32)
    rstd = (np.float32(1.0) / np.sqrt(ms + np.float32(eps))).astype(np.float32)
    return round_to((x * rstd) * w, dtype)


def add_rmsnorm(x: np.ndarray, residual: np.ndarray, weight: np.ndarray, eps: float, dtype: str):
    """(``ref.rmsnorm(x + r, w, eps)``, ``x + r``): the 16-bit addition rounds
    (torch's elementwise add of two 16-bit tensors computes in fp32 and rounds
    once), then rmsnorm of the rounded sum."""
    h = round_to(np.asarray(x, dtype=np.float32) + np.asarray(residual, dtype=np.float32), dtype)
    return rmsnorm(h, weight, eps, dtype), h


def _silu_f32(x: np.ndarray) -> np.ndarray:
    x = np.asarray(x, dtype=np.float32)
    with np.errstate(over="ignore"):
        return (x / (np.float32(1.0) + np.exp(-x))).astype(np.float32)


def silu(x: np.ndarray, dtype: str) -> np.ndarray:
    """ref.silu = ``F.silu(x)`` (ref/activation.py:15-16): x / (1 + e^-x) in fp32, one rounding."""
    return round_to(_silu_f32(x), dtype)


def relu(x: np.ndarray, dtype: str) -> np.ndarray:
    """ref.relu = ``F.relu(x)`` (ref/activation.py:11-12): max(x, 0), NaN propagates."""
    x = np.asarray(x, dtype=np.float32)
    return round_to(np.where(np.isnan(x) | (x > 0), x, np.float32(0.0)), dtype)


def silu_mul(gate: np.ndarray, up: np.ndarray, dtype: str) -> np.ndarray:
    """Fused silu(gate) * up: fp32 throughout, one rounding (the kernel's contract)."""
    return round_to(_silu_f32(gate) * np.asarray(up, dtype=np.float32), dtype)


def silu_mul_composed(gate: np.ndarray, up: np.ndarray, dtype: str) -> np.ndarray:
    """``ref.silu(gate) * up``: the reference's composition, rounding after silu and after the product."""
    return round_to(silu(gate, dtype) * np.asarray(up, dtype=np.float32), dtype)


def gemm_silu_mul(a: np.ndarray, w_gate: np.ndarray, w_up: np.ndarray, dtype: str) -> np.ndarray:
    """silu(a @ W_gate) * (a @ W_up) with both products and the activation in
    fp32 and one rounding (the fused gate/up kernel's contract; the reference
    composes ref.silu(ref.gemm(a, W_gate)) * ref.gemm(a, W_up), rounding each
    step)."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    g = a @ np.ascontiguousarray(w_gate, dtype=np.float32)
    u = a @ np.ascontiguousarray(w_up, dtype=np.float32)
    return round_to(_silu_f32(g) * u, dtype)


def mlp_block(x, norm_w, w_gate_up, w_down, eps: float, dtype: str) -> np.ndarray:
    """Unsharded Llama MLP block as a composition of the ops above:
    rms_norm -> x @ [W_gate | W_up] -> silu(gate) * up -> @ W_down.

    The tensor-parallel block (column-split gate/up, row-split down, one
    all-reduce) must reproduce this within the GEMM tolerance.
    """
    h = rmsnorm(x, norm_w, eps, dtype)
    gu = gemm(h, w_gate_up, dtype)
    inter = w_gate_up.shape[1] // 2
    act = silu_mul(gu[:, :inter], gu[:, inter:], dtype)
    return gemm(act, w_down, dtype)


def mlp_block_sharded(x, norm_w, w_gate_up, w_down, eps: float, dtype: str, world: int) -> np.ndarray:
    """The tensor-parallel block restated on one CPU: rank r owns gate/up
    columns and down rows [r*I/W, (r+1)*I/W); each rank's down output is
    rounded to `dtype`, and the partials are summed in rank order in fp32 and
    rounded once (the all-reduce)."""
    inter = w_gate_up.shape[1] // 2
    if inter % world:
        raise ValueError("intermediate size must divide by the world size")
    shard = inter // world
    h = rmsnorm(x, norm_w, eps, dtype)
    total = None
    for r in range(world):
        cols = slice(r * shard, (r + 1) * shard)
        wg = w_gate_up[:, :inter][:, cols]
        wu = w_gate_up[:, inter:][:, cols]
        gu = gemm(h, np.concatenate([wg, wu], axis=1), dtype)
        act = silu_mul(gu[:, :shard], gu[:, shard:], dtype)
        part = gemm(act, w_down[cols, :], dtype)
        total = part if total is None else total + part
    return round_to(total, dtype)
