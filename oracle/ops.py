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


def rms_rstd(x: np.ndarray, eps: float) -> np.ndarray:
    """rms_norm's row statistic rsqrt(mean(x^2) + eps) in fp32 (the factor
    ``rmsnorm`` applies before the weight)."""
    x = np.asarray(x, dtype=np.float32)
    ms = np.mean(x * x, axis=-1, dtype=np.float32)
    return (np.float32(1.0) / np.sqrt(ms + np.float32(eps))).astype(np.float32)


def gemm_silu_mul_folded(x: np.ndarray, norm_w: np.ndarray, w_gate: np.ndarray,
                         w_up: np.ndarray, eps: float, dtype: str) -> np.ndarray:
    """rms_norm folded into the fused gate/up kernel: the norm weight scales
    the weight rows once (W' = diag(w) W rounded to `dtype`), the GEMM runs
    on x, and each row's fp32 accumulators are multiplied by rstd before
    silu(gate) * up and the single rounding.  Equal to
    ``gemm_silu_mul(rmsnorm(x, w), W_gate, W_up)`` up to where the roundings
    fall."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.asarray(norm_w, dtype=np.float32).reshape(-1, 1)
    wg = round_to(np.asarray(w_gate, dtype=np.float32) * w, dtype)
    wu = round_to(np.asarray(w_up, dtype=np.float32) * w, dtype)
    rstd = rms_rstd(x, eps).reshape(-1, 1)
    g = (x @ wg) * rstd
    u = (x @ wu) * rstd
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


# ---- 8-bit formats and the scaled GEMM ----------------------------------------

QDTYPES = ("e4m3", "e5m2", "int8")

# (exponent bits, mantissa bits, bias) of the OCP 8-bit float formats torch
# names float8_e4m3fn and float8_e5m2.
_FP8_FORMATS = {"e4m3": (4, 3, 7), "e5m2": (5, 2, 15)}


def _fp8_positive_values(kind: str) -> np.ndarray:
    """Values of the codes 0..127 (sign bit clear) as float64; NaN / inf where
    the format has them (e4m3fn: 0x7F is NaN, no infinities; e5m2: exponent
    all ones is inf (mantissa 0) or NaN)."""
    e_bits, m_bits, bias = _FP8_FORMATS[kind]
    codes = np.arange(128)
    e = codes >> m_bits
    m = codes & ((1 << m_bits) - 1)
    frac = m / float(1 << m_bits)
    v = np.where(e == 0, frac * 2.0 ** (1 - bias), (1.0 + frac) * 2.0 ** (e - bias))
    if kind == "e4m3":
        v[127] = np.nan
    else:
        top = (1 << e_bits) - 1
        v[(e == top) & (m == 0)] = np.inf
        v[(e == top) & (m != 0)] = np.nan
    return v


def fp8_decode(codes: np.ndarray, kind: str) -> np.ndarray:
    """uint8 codes -> float32 values (exact: every fp8 value is a float32)."""
    c = np.asarray(codes, dtype=np.uint8)
    pos = _fp8_positive_values(kind)[c & 0x7F]
    return np.where(c & 0x80, -pos, pos).astype(np.float32)


def fp8_encode(x: np.ndarray, kind: str) -> np.ndarray:
    """float32 -> uint8 codes, round to nearest, ties to the even code, the
    sign kept for zeros.  Magnitudes that round past the largest finite value
    become NaN (e4m3fn, which has no infinity) or inf (e5m2); NaN stays NaN.
    Restates torch's ``Tensor.to(torch.float8_e4m3fn / float8_e5m2)`` on CPU,
    the conversion the reference's tests quantise with
    (tests/gemm/test_triton.py:85-93)."""
    x = np.asarray(x, dtype=np.float32)
    vals = _fp8_positive_values(kind)
    n_finite = 127 if kind == "e4m3" else 124  # codes 0 .. n_finite-1 are finite
    over_code = 127 if kind == "e4m3" else 124  # NaN resp. +inf
    # Finite values plus the value the format would have next, so that
    # rounding just past the maximum behaves as in an unbounded format.
    top = vals[n_finite - 1]
    step = top - vals[n_finite - 2]
    table = np.append(vals[:n_finite], top + step)
    mag = np.abs(x.astype(np.float64))
    hi = np.clip(np.searchsorted(table, mag, side="left"), 1, len(table) - 1)
    lo = hi - 1
    d_lo = mag - table[lo]
    d_hi = table[hi] - mag
    pick_hi = (d_hi < d_lo) | ((d_hi == d_lo) & (hi % 2 == 0))
    code = np.where(pick_hi, hi, lo)
    code = np.where(mag > table[-1], n_finite, code)   # beyond the virtual value
    code = np.where(code >= n_finite, over_code, code)
    code = np.where(np.isnan(x), 127, code)
    sign = np.signbit(x) & ~np.isnan(x)
    return (code | np.where(sign, 0x80, 0)).astype(np.uint8)


def dequant(q: np.ndarray, qdtype: str) -> np.ndarray:
    """8-bit inputs -> float64 values: fp8 codes decoded, int8 as integers."""
    if qdtype == "int8":
        return np.asarray(q).view(np.int8).astype(np.float64)
    return fp8_decode(q, qdtype).astype(np.float64)


def scaled_gemm(a_q: np.ndarray, b_q: np.ndarray, scale_a: np.ndarray, scale_b: np.ndarray,
                qdtype: str, out_dtype: str) -> np.ndarray:
    """The reference's ``scaled_gemm`` (jit_kernel/gemm.py:199-248; kernels
    jit_kernel/gemm.py:86-123 and 144-196): acc = A @ B accumulated in fp32
    (restated in float64, which is exact for int8 and holds the fp8 sum to
    far below fp32 rounding), then ``acc * scale_a[m] * scale_b[n]`` in fp32,
    left to right, and one rounding to the output dtype.  scale_a / scale_b
    hold one value each (tensorwise) or M / N values (rowwise)."""
    a = dequant(a_q, qdtype)
    b = dequant(b_q, qdtype)
    acc = (a @ b).astype(np.float32)
    sa = np.asarray(scale_a, dtype=np.float32).reshape(-1)
    sb = np.asarray(scale_b, dtype=np.float32).reshape(-1)
    sa = sa.reshape(-1, 1) if sa.size == acc.shape[0] and sa.size != 1 else sa.reshape(1, 1)
    sb = sb.reshape(1, -1) if sb.size == acc.shape[1] and sb.size != 1 else sb.reshape(1, 1)
    y = (acc * sa) * sb
    return round_to(y.astype(np.float32), out_dtype)


def scaled_gemm_dequant_first(a_q, b_q, scale_a, scale_b, qdtype: str, out_dtype: str):
    """The reference tests' formulation (tests/gemm/test_triton.py:104-107):
    ``(a.float() * scale_a[:, None]) @ (b.float() * scale_b[None, :])`` in
    fp32, rounded once.  Differs from ``scaled_gemm`` only by fp32 rounding
    before the final rounding."""
    a = dequant(a_q, qdtype).astype(np.float32) * np.asarray(scale_a, np.float32).reshape(-1, 1)
    b = dequant(b_q, qdtype).astype(np.float32) * np.asarray(scale_b, np.float32).reshape(1, -1)
    return round_to((a.astype(np.float64) @ b.astype(np.float64)).astype(np.float32), out_dtype)
