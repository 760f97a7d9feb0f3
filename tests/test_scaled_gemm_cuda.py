"""Scaled (dequantising) 8-bit GEMM parity on a B200.

The reference's tests (tests/gemm/test_triton.py:60-157) compare
``scaled_gemm`` with ``(a.float() * sa) @ (b.float() * sb)`` at rtol = atol =
2e-2; here every path is held to that against the golden outputs of the
reference's own formula, and tighter against the oracle:

* int8: the integer accumulation is exact on every path (tcgen05 s32, SIMT
  int32, fp32 K-split partials of integers), so the output equals the
  oracle's ``(float(acc) * sa) * sb`` rounded once - bit for bit;
* fp8: fp32 accumulation in another order, so |got - oracle| is bounded by
  K * 2^-24 * (|A| @ |B|) * |sa| * |sb| plus one output ulp.
"""

from __future__ import annotations

import numpy as np
import pytest

from cases import all_cases, make_inputs
from oracle import ops
from oracle.inputs import quantized, scales
from tests.conftest import assert_close_np

pytestmark = pytest.mark.gpu

SCALED_CASES = [c for c in all_cases() if c.op == "scaled_gemm"]


def _qtorch(qdtype: str):
    import torch

    return {"e4m3": torch.float8_e4m3fn, "e5m2": torch.float8_e5m2, "int8": torch.int8}[qdtype]


def _otorch(out: str):
    import torch

    return {"float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16}[out]


def _dev(q: np.ndarray, qdtype: str):
    import torch

    return torch.from_numpy(np.ascontiguousarray(q)).cuda().view(_qtorch(qdtype))


def _fdev(x: np.ndarray):
    import torch

    return torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).cuda()


def _ulp(x: np.ndarray, out: str) -> np.ndarray:
    mant = {"bfloat16": 7, "float16": 10, "float32": 23}[out]
    e = np.floor(np.log2(np.maximum(np.abs(x), 1e-30)))
    return 2.0 ** (e - mant)


def _check_against_oracle(got, a_q, b_q, sa, sb, qdtype: str, out: str) -> None:
    got = got.float().cpu().numpy()
    want = ops.scaled_gemm(a_q, b_q, sa, sb, qdtype, out)
    assert got.shape == want.shape
    if qdtype == "int8":
        bad = np.argwhere(got != want)[:5]
        assert bad.size == 0, [(tuple(i), got[tuple(i)], want[tuple(i)]) for i in bad]
        return
    K = a_q.shape[1]
    mag = (np.abs(ops.dequant(a_q, qdtype)) @ np.abs(ops.dequant(b_q, qdtype))).astype(np.float64)
    mag *= np.abs(sa.astype(np.float64)).reshape(-1, 1) if sa.size > 1 else abs(float(sa[0]))
    mag *= np.abs(sb.astype(np.float64)).reshape(1, -1) if sb.size > 1 else abs(float(sb[0]))
    bound = K * 2.0**-24 * mag + _ulp(want, out) * 1.0001
    diff = np.abs(got.astype(np.float64) - want.astype(np.float64))
    worst = np.unravel_index(np.argmax(diff - bound), diff.shape)
    assert np.all(diff <= bound), (worst, got[worst], want[worst], bound[worst])


# ---- the reference's cases through the Python API --------------------------------

@pytest.mark.parametrize("optimized", [False, True], ids=["naive", "optimized"])
@pytest.mark.parametrize("case", SCALED_CASES, ids=lambda c: c.id)
def test_scaled_gemm_matches_reference_and_oracle(case, optimized):
    import aot_kernel

    a_q, b_q, sa, sb = make_inputs(case)
    got = aot_kernel.scaled_gemm(_dev(a_q, case.qdtype), _dev(b_q, case.qdtype), _fdev(sa),
                                 _fdev(sb), out_dtype=_otorch(case.dtype), optimized=optimized)
    M, K, N = case.shape
    assert tuple(got.shape) == (M, N) and got.dtype == _otorch(case.dtype)
    golden = np.load(_golden_path())[case.id]
    ref = {"bfloat16": ops.bf16_from_bits,
           "float16": lambda b: b.view(np.float16).astype(np.float32),
           "float32": lambda b: b.view(np.float32)}[case.dtype](golden).reshape(M, N)
    assert_close_np(got, ref, 2e-2, 2e-2)  # the reference test's own tolerance
    _check_against_oracle(got, a_q, b_q, sa, sb, case.qdtype, case.dtype)


def _golden_path():
    from pathlib import Path

    return Path(__file__).resolve().parent / "golden" / "golden.npz"


def test_scaled_gemm_preserves_shape_and_dtype():
    import torch

    import aot_kernel

    for qdtype in ("e4m3", "int8"):
        a = _dev(quantized((64, 128), 1, qdtype), qdtype)
        b = _dev(quantized((128, 96), 2, qdtype), qdtype)
        c = aot_kernel.scaled_gemm(a, b, torch.tensor([0.05], device="cuda"),
                                   torch.tensor([0.03], device="cuda"), out_dtype=torch.bfloat16)
        assert c.shape == (64, 96) and c.dtype == torch.bfloat16


def test_scaled_gemm_rejects_bad_scale_shape():
    import torch

    import aot_kernel

    a = _dev(quantized((64, 128), 1, "int8"), "int8")
    b = _dev(quantized((128, 96), 2, "int8"), "int8")
    with pytest.raises((ValueError, AssertionError)):
        aot_kernel.scaled_gemm(a, b, torch.rand(63, device="cuda"), torch.rand(96, device="cuda"))
    with pytest.raises((ValueError, AssertionError)):
        aot_kernel.scaled_gemm(a, b, torch.rand(64, device="cuda"), torch.rand(1, device="cuda"))
    with pytest.raises(AssertionError):
        aot_kernel.scaled_gemm(a, b, torch.rand(64, device="cuda", dtype=torch.float64),
                               torch.rand(96, device="cuda"))


def test_scaled_gemm_rejects_16bit_inputs():
    import torch

    import aot_kernel

    a = torch.randn(16, 16, device="cuda", dtype=torch.bfloat16)
    s = torch.ones(1, device="cuda")
    with pytest.raises(ValueError):
        aot_kernel.scaled_gemm(a, a, s, s)


def test_scaled_gemm_accepts_2d_and_strided_scales():
    """Scales shaped [M, 1] / [1, N] (as torch._scaled_mm takes them) and a
    non-contiguous view are flattened like the reference's stride(0) reads."""
    import torch

    import aot_kernel

    M, K, N = 96, 128, 80
    a_q, b_q = quantized((M, K), 3, "int8"), quantized((K, N), 4, "int8")
    sa, sb = scales(M, N, "row", 5)
    wide = torch.zeros(2 * N, device="cuda")
    wide[::2] = _fdev(sb)
    got = aot_kernel.scaled_gemm(_dev(a_q, "int8"), _dev(b_q, "int8"), _fdev(sa).reshape(M, 1),
                                 wide[::2], out_dtype=torch.float32)
    _check_against_oracle(got, a_q, b_q, sa, sb, "int8", "float32")


def test_scaled_gemm_empty_k_gives_zeros():
    import torch

    import aot_kernel

    a = torch.empty(4, 0, device="cuda", dtype=torch.int8)
    b = torch.empty(0, 8, device="cuda", dtype=torch.int8)
    s = torch.ones(1, device="cuda")
    assert torch.count_nonzero(aot_kernel.scaled_gemm(a, b, s, s)) == 0


@pytest.mark.parametrize("optimized", [False, True], ids=["naive", "optimized"])
def test_scaled_gemm_nan_input_propagates(optimized):
    """An fp8 NaN code in A row 0 makes row 0 of C NaN and nothing else."""
    import torch

    import aot_kernel

    M, K, N = 128, 256, 256
    a_q, b_q = quantized((M, K), 6, "e4m3"), quantized((K, N), 7, "e4m3")
    a_q[0, 5] = 0x7F
    s = torch.ones(1, device="cuda")
    got = aot_kernel.scaled_gemm(_dev(a_q, "e4m3"), _dev(b_q, "e4m3"), s, s,
                                 optimized=optimized).float().cpu().numpy()
    assert np.isnan(got[0]).all() and not np.isnan(got[1:]).any()


# ---- through the C ABI, one kernel at a time ---------------------------------------

def _capi_run(fn, M, K, N, qdtype, out, mode, seed, workspace=False):
    import torch

    from aot_kernel import capi

    a_q, b_q = quantized((M, K), seed, qdtype), quantized((K, N), seed + 1, qdtype)
    sa, sb = scales(M, N, mode, seed + 2)
    a, b, dsa, dsb = _dev(a_q, qdtype), _dev(b_q, qdtype), _fdev(sa), _fdev(sb)
    c = torch.empty(M, N, device="cuda", dtype=_otorch(out))
    args = (c, a, b, dsa, dsb, M, N, K, capi.dtype_code(_qtorch(qdtype)),
            capi.dtype_code(_otorch(out)),
            capi.SCALE_ROW if mode == "row" else capi.SCALE_TENSOR)
    if fn == "simt":
        capi.scaled_gemm_simt(*args)
    else:
        ws = None
        nbytes = 0
        if workspace:
            nbytes = capi.scaled_gemm_workspace_size(M, N, K, capi.dtype_code(_qtorch(qdtype)))
            ws = torch.empty(max(nbytes, 1), device="cuda", dtype=torch.uint8)
        getattr(capi, "scaled_gemm_tc" if fn == "tc" else "scaled_gemm")(*args, ws, nbytes)
    torch.cuda.synchronize()
    return c, a_q, b_q, sa, sb


TC_SHAPES = [
    (128, 128, 256),      # one tile
    (200, 384, 272),      # ragged M and N inside the tiles (N % 16 == 0)
    (1, 512, 1024),       # decode row
    (1024, 1024, 1024),
    (64, 16, 32),         # one K step of 16 bytes, N narrower than a box
    (2304, 256, 4096),    # 288 tiles: one wave and 140 left, run whole
]


@pytest.mark.parametrize("qdtype", ["e4m3", "e5m2", "int8"])
@pytest.mark.parametrize("shape", TC_SHAPES, ids=str)
def test_scaled_gemm_tc_matches_oracle(shape, qdtype):
    M, K, N = shape
    for mode in ("tensor", "row"):
        got, a_q, b_q, sa, sb = _capi_run("tc", M, K, N, qdtype, "bfloat16", mode, seed=M + K + N)
        _check_against_oracle(got, a_q, b_q, sa, sb, qdtype, "bfloat16")


@pytest.mark.parametrize("out", ["float16", "float32"])
@pytest.mark.parametrize("qdtype", ["e4m3", "int8"])
def test_scaled_gemm_tc_output_dtypes(qdtype, out):
    got, a_q, b_q, sa, sb = _capi_run("tc", 300, 256, 528, qdtype, out, "row", seed=11)
    _check_against_oracle(got, a_q, b_q, sa, sb, qdtype, out)


@pytest.mark.parametrize("qdtype", ["e4m3", "int8"])
def test_scaled_gemm_tc_k_split_tail(qdtype):
    """8 tiles of 128 x 256 on 148 SMs with K = 16384 (128 K blocks of 128):
    each tile is cut along K into 4 units whose partials the last unit sums
    from the workspace (deterministic: two runs agree bit for bit)."""
    import torch

    from aot_kernel import capi

    props = torch.cuda.get_device_properties(0)
    if props.multi_processor_count != 148:
        pytest.skip("tile arithmetic assumes 148 SMs")
    M, K, N = 256, 16384, 1024
    assert capi.scaled_gemm_workspace_size(M, N, K, capi.dtype_code(_qtorch(qdtype))) > 0
    got, a_q, b_q, sa, sb = _capi_run("tc", M, K, N, qdtype, "bfloat16", "row", seed=21,
                                      workspace=True)
    _check_against_oracle(got, a_q, b_q, sa, sb, qdtype, "bfloat16")
    again, *_ = _capi_run("tc", M, K, N, qdtype, "bfloat16", "row", seed=21, workspace=True)
    assert torch.equal(got, again)


@pytest.mark.parametrize("qdtype", ["e4m3", "int8"])
@pytest.mark.parametrize("shape", [(130, 64, 130), (129, 257, 193), (1, 7, 3), (70, 48, 64)],
                         ids=str)
def test_scaled_gemm_simt_and_dispatch_match_oracle(shape, qdtype):
    M, K, N = shape
    for fn in ("simt", "dispatch"):
        for mode in ("tensor", "row"):
            got, a_q, b_q, sa, sb = _capi_run(fn, M, K, N, qdtype, "bfloat16", mode, seed=M * 3 + N)
            _check_against_oracle(got, a_q, b_q, sa, sb, qdtype, "bfloat16")


def test_scaled_gemm_tc_rejects_unaligned_shapes():
    import torch

    from aot_kernel import capi

    a = torch.zeros(64, 72, device="cuda", dtype=torch.int8)
    b = torch.zeros(72, 64, device="cuda", dtype=torch.int8)
    c = torch.empty(64, 64, device="cuda", dtype=torch.bfloat16)
    s = torch.ones(1, device="cuda")
    with pytest.raises(capi.AotkError) as e:
        capi.scaled_gemm_tc(c, a, b, s, s, 64, 64, 72, capi.INT8, capi.BFLOAT16, capi.SCALE_TENSOR)
    assert e.value.status == capi.ERR_UNSUPPORTED


def test_scaled_gemm_large_int8_matches_integer_matmul():
    """A 4096 x 4096 x 4096 int8 product against torch's exact integer matmul
    on the GPU (int64 accumulation): bit-exact after the fp32 scaling."""
    import torch

    from aot_kernel import capi

    M = K = N = 4096
    g = torch.Generator(device="cuda").manual_seed(0)
    a = torch.randint(-8, 8, (M, K), device="cuda", dtype=torch.int8, generator=g)
    b = torch.randint(-8, 8, (K, N), device="cuda", dtype=torch.int8, generator=g)
    sa = torch.rand(M, device="cuda", generator=g) * 0.1 + 0.01
    sb = torch.rand(N, device="cuda", generator=g) * 0.1 + 0.01
    c = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    nbytes = capi.scaled_gemm_workspace_size(M, N, K, capi.INT8)
    ws = torch.empty(max(nbytes, 1), device="cuda", dtype=torch.uint8)
    capi.scaled_gemm(c, a, b, sa, sb, M, N, K, capi.INT8, capi.BFLOAT16, capi.SCALE_ROW, ws, nbytes)
    acc = (a.double() @ b.double()).float()  # |acc| <= 64 * 4096 < 2^24: exact
    want = ((acc * sa[:, None]) * sb[None, :]).to(torch.bfloat16)
    assert torch.equal(c, want)
