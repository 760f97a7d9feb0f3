"""GEMM wrappers: ``gemm`` (tensor-core path), ``gemm_naive`` (SIMT path),
the fused ``gemm_silu_mul`` and the 8-bit ``scaled_gemm``.

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


def gemm_host(a: torch.Tensor, b: torch.Tensor, *, out: torch.Tensor | None = None,
              device: torch.device | int | None = None) -> torch.Tensor:
    """C = A @ B for fp16/bf16 matrices in HOST memory, on the current (or
    given) CUDA device, through the C ABI entry ``aotk_gemm_host``: B and row
    blocks of A are copied in while earlier blocks compute and finished blocks
    of C are copied out, so the PCIe link runs both directions during the
    GEMM.  ``a`` / ``b`` / ``out`` should be pinned (``pin_memory()``) for the
    copies to overlap; ``out`` defaults to a new pinned [M, N] tensor.  The
    result is complete when this returns (the call synchronises its stream).
    Not in the reference, whose callers copy with torch and call ``gemm``."""
    from . import capi

    if a.is_cuda or b.is_cuda:
        raise ValueError("gemm_host takes host tensors; use gemm for device tensors")
    assert_contiguous(a, b)
    dtype = assert_same_dtype(a, b)
    if dtype not in _TENSOR_CORE_DTYPES:
        raise ValueError(f"gemm_host supports fp16/bf16, got {dtype}")
    if a.dim() != 2 or b.dim() != 2 or a.size(1) != b.size(0):
        raise ValueError(f"gemm_host expects a [M, K] and b [K, N], got {tuple(a.shape)} {tuple(b.shape)}")
    M, K = a.shape
    N = b.size(1)
    dev = torch.device("cuda", torch.cuda.current_device() if device is None else
                       torch.device("cuda", device).index)
    if out is None:
        out = torch.empty((M, N), dtype=dtype, pin_memory=True)
    elif out.is_cuda or tuple(out.shape) != (M, N) or out.dtype != dtype or not out.is_contiguous():
        raise ValueError("out must be a contiguous host tensor of shape [M, N] and the inputs' dtype")
    code = capi.dtype_code(dtype)
    with torch.cuda.device(dev):
        a_d = torch.empty((M, K), dtype=dtype, device=dev)
        b_d = torch.empty((K, N), dtype=dtype, device=dev)
        c_d = torch.empty((M, N), dtype=dtype, device=dev)
        nbytes = capi.gemm_host_workspace_size(M, N, K, code)
        ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=dev)
        stream = torch.cuda.current_stream(dev)
        capi.gemm_host(out, a, b, M, N, K, code, a_d, b_d, c_d, ws if nbytes else None, nbytes,
                       stream.cuda_stream)
        stream.synchronize()
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


def gemm_silu_mul(a: torch.Tensor, w_gate_up: torch.Tensor,
                  row_scale: torch.Tensor | None = None) -> torch.Tensor:
    """silu(a @ W_gate) * (a @ W_up) in one kernel; ``w_gate_up`` from
    ``interleave_gate_up``.  The gate/up product stays in TMEM: silu and the
    product use the fp32 accumulators and the result is rounded once.

    With ``row_scale`` (fp32 [M]) both products of row m are scaled by
    row_scale[m] before silu: with a = x, row_scale = ``rms_rstd(x)`` and
    ``fold_norm_weight(w_gate_up, norm_w)``, this is the gate/up projection
    of ``rms_norm(x, norm_w)`` with the normalisation folded into the GEMM."""
    device, dtype = _validate(a, w_gate_up)
    if dtype not in _TENSOR_CORE_DTYPES:
        raise ValueError(f"gemm_silu_mul supports fp16/bf16, got {dtype}")
    out = torch.empty((a.size(0), w_gate_up.size(1) // 2), device=device, dtype=dtype)
    if row_scale is None:
        torch.ops.aot_kernel.gemm_silu_mul(out, a, w_gate_up)
    else:
        torch.ops.aot_kernel.gemm_silu_mul_rowscale(out, a, w_gate_up,
                                                    row_scale.reshape(-1).contiguous())
    return out


def fold_norm_weight(w: torch.Tensor, norm_weight: torch.Tensor) -> torch.Tensor:
    """diag(norm_weight) @ w rounded once to w's dtype (computed in fp32): the
    weight that takes rms_norm's elementwise scale, so that
    ``rms_norm(x, g) @ w == diag(rstd(x)) (x @ fold_norm_weight(w, g))`` up to
    rounding.  Row k of ``w`` (any column layout, e.g. interleaved gate/up) is
    multiplied by norm_weight[k]."""
    if w.dim() != 2 or norm_weight.dim() != 1 or norm_weight.numel() != w.size(0):
        raise ValueError("fold_norm_weight expects w [K, N] and norm_weight [K]")
    return (w.float() * norm_weight.float().reshape(-1, 1)).to(w.dtype).contiguous()


_SCALED_INPUT_DTYPES = (torch.float8_e4m3fn, torch.float8_e5m2, torch.int8)


def scaled_gemm(
    a: torch.Tensor,
    b: torch.Tensor,
    scale_a: torch.Tensor,
    scale_b: torch.Tensor,
    out_dtype: torch.dtype = torch.bfloat16,
    optimized: bool = True,
) -> torch.Tensor:
    """C = (A @ B) * scale_a * scale_b for quantised 8-bit A [M, K] and B [K, N].

    Same signature, checks and error types as the reference's
    ``jit_kernel.gemm.scaled_gemm`` (jit_kernel/gemm.py:199-248): A and B are
    both float8_e4m3fn, both float8_e5m2 or both int8; the scales are float32
    and either tensorwise (one value each) or rowwise (``scale_a.numel() == M``,
    ``scale_b.numel() == N``), anything else is a ValueError.  The product is
    accumulated in fp32 (int8: exactly, in int32), scaled as
    ``(acc * scale_a[m]) * scale_b[n]`` and rounded once to ``out_dtype``
    (bfloat16, float16 or float32).  ``optimized=True`` runs the tcgen05
    kernel (kind::f8f6f4 / kind::i8) where K and N are multiples of 16, the
    SIMT kernel otherwise; ``optimized=False`` always runs the SIMT kernel.
    """
    if a.dim() != 2 or b.dim() != 2:
        raise AssertionError("gemm expects 2D inputs")
    assert_is_cuda(a, b)
    assert_contiguous(a, b)
    device = assert_same_device(a, b)
    dtype = assert_same_dtype(a, b)
    M, K1 = a.shape
    K2, N = b.shape
    if K1 != K2:
        raise AssertionError("gemm shape mismatch")
    assert_is_cuda(scale_a, scale_b)
    if scale_a.dtype != torch.float32 or scale_b.dtype != torch.float32:
        raise AssertionError("scales must be float32")
    if dtype not in _SCALED_INPUT_DTYPES:
        raise ValueError(
            f"scaled_gemm expects float8_e4m3fn, float8_e5m2 or int8 inputs, got {dtype}"
        )
    sa_n, sb_n = scale_a.numel(), scale_b.numel()
    if not ((sa_n == 1 and sb_n == 1) or (sa_n == M and sb_n == N)):
        raise ValueError(
            "expect tensorwise (scalar scale_a and scale_b) "
            "or rowwise (scale_a.numel()==M, scale_b.numel()==N)"
        )
    if scale_a.device != device or scale_b.device != device:
        raise ValueError(
            f"device mismatch: scales on {scale_a.device} / {scale_b.device}, inputs on {device}"
        )
    out = torch.empty((M, N), device=device, dtype=out_dtype)
    sa = scale_a.reshape(-1).contiguous()
    sb = scale_b.reshape(-1).contiguous()
    torch.ops.aot_kernel.scaled_gemm(out, a, b, sa, sb, bool(optimized))
    return out
