"""rms_norm / silu / relu / silu_mul parity on a B200 against the oracle and
against the reference's golden outputs."""

from __future__ import annotations

import numpy as np
import pytest

from cases import ACT_SHAPES, RMSNORM_SHAPES, all_cases, make_inputs, sampled
from tests.conftest import assert_close_common, assert_close_np, assert_max_err_frac, to_device, torch_dtype
from oracle import ops
from oracle.inputs import randn

pytestmark = pytest.mark.gpu


# ---- operator API, the reference's tests/norm/test_cuda.py and tests/activation/test_cuda.py ----

@pytest.mark.parametrize("shape", RMSNORM_SHAPES, ids=str)
def test_rmsnorm_matches_oracle(shape, dtype):
    from aot_kernel.norm import rmsnorm

    x = randn(shape, 1, dtype)
    w = randn((shape[-1],), 2, dtype)
    got = rmsnorm(to_device(x, dtype), to_device(w, dtype))
    assert got.shape == tuple(shape) and got.dtype == torch_dtype(dtype)
    assert_close_common(got, ops.rmsnorm(x, w, 1e-6, dtype), dtype)


def test_rmsnorm_custom_eps():
    from aot_kernel.norm import rmsnorm

    x = randn((4, 32), 3, "float32")
    w = randn((32,), 4, "float32")
    got = rmsnorm(to_device(x, "float32"), to_device(w, "float32"), eps=1e-3)
    assert_close_np(got, ops.rmsnorm(x, w, 1e-3, "float32"), rtol=1.3e-6, atol=1e-5)


@pytest.mark.parametrize("cols", [8, 24, 256, 2048, 4096, 8192, 16384, 32768, 65536, 70000, 1023, 1])
def test_rmsnorm_row_lengths(cols):
    from aot_kernel.norm import rmsnorm

    x = randn((5, cols), cols, "bfloat16")
    w = randn((cols,), cols + 1, "bfloat16", mean=1.0, std=0.1)
    got = rmsnorm(to_device(x, "bfloat16"), to_device(w, "bfloat16"))
    assert_close_common(got, ops.rmsnorm(x, w, 1e-6, "bfloat16"), "bfloat16")


def test_rmsnorm_rejects_non_contiguous():
    import torch

    from aot_kernel.norm import rmsnorm

    x = torch.randn(8, 8, device="cuda").t()
    with pytest.raises((ValueError, RuntimeError, AssertionError)):
        rmsnorm(x, torch.randn(8, device="cuda"))


@pytest.mark.parametrize("shape", ACT_SHAPES + [(7,), (3, 5, 9), (0,)], ids=str)
@pytest.mark.parametrize("op", ["silu", "relu"])
def test_activation_matches_oracle(op, shape, dtype):
    import aot_kernel

    x = randn(shape, 5, dtype, std=2.0)
    got = getattr(aot_kernel, op)(to_device(x, dtype))
    assert got.shape == tuple(shape)
    assert_close_common(got, getattr(ops, op)(x, dtype), dtype)


def test_activation_special_values(dtype):
    import aot_kernel

    x = np.array([0.0, -0.0, np.inf, np.nan, 30.0, -30.0, 1e-3, -1e-3, 3.0, -100.0], dtype=np.float32)
    x = ops.round_to(x, dtype)
    for op in ("silu", "relu"):
        got = getattr(aot_kernel, op)(to_device(x, dtype))
        assert_close_common(got, getattr(ops, op)(x, dtype), dtype)


@pytest.mark.parametrize("op", ["silu", "relu"])
def test_activation_rejects_non_contiguous(op):
    import torch

    import aot_kernel

    x = torch.randn(8, 8, device="cuda").t()
    with pytest.raises((ValueError, RuntimeError)):
        getattr(aot_kernel, op)(x)


@pytest.mark.parametrize("shape", [(4, 1024), (3, 1000), (17, 14336), (1, 8)], ids=str)
def test_silu_mul_matches_oracle(shape, dtype):
    from aot_kernel import silu_mul

    g = randn(shape, 6, dtype, std=2.0)
    u = randn(shape, 7, dtype, std=2.0)
    got = silu_mul(to_device(g, dtype), to_device(u, dtype))
    assert_close_common(got, ops.silu_mul(g, u, dtype), dtype)


def test_silu_mul_strided_halves(dtype):
    """gate and up as the two column halves of one [rows, 2*I] tensor."""
    from aot_kernel import silu_mul

    rows, inter = 33, 1032
    gu = randn((rows, 2 * inter), 8, dtype, std=2.0)
    t = to_device(gu, dtype)
    got = silu_mul(t[:, :inter], t[:, inter:])
    assert_close_common(got, ops.silu_mul(gu[:, :inter], gu[:, inter:], dtype), dtype)


# ---- C ABI against the reference's golden outputs ----

GOLDEN_CASES = [c for c in all_cases()
                if c.op in ("rmsnorm", "add_rmsnorm", "silu", "relu", "silu_mul")]


@pytest.mark.parametrize("case", GOLDEN_CASES, ids=lambda c: c.id)
def test_capi_against_reference_golden(case):
    import torch

    from aot_kernel import capi
    from tests.test_oracle_golden import _from_bits

    golden = np.load(__import__("pathlib").Path(__file__).parent / "golden" / "golden.npz")
    dt = case.dtype
    code = capi.dtype_code(torch_dtype(dt))
    ins = [to_device(x, dt) for x in make_inputs(case)]
    out = torch.empty_like(ins[0])
    if case.op == "rmsnorm":
        cols = case.shape[-1]
        capi.rmsnorm_forward(out, ins[0], ins[1], ins[0].numel() // cols, cols, case.eps, code)
    elif case.op == "add_rmsnorm":
        cols = case.shape[-1]
        h = torch.empty_like(ins[0])
        capi.add_rmsnorm_forward(out, h, ins[0], ins[1], ins[2], ins[0].numel() // cols, cols,
                                 case.eps, code)
    elif case.op in ("silu", "relu"):
        getattr(capi, f"{case.op}_forward")(out, ins[0], ins[0].numel(), code)
    else:
        rows, cols = case.shape
        capi.silu_mul_forward(out, cols, ins[0], cols, ins[1], cols, rows, cols, code)
    torch.cuda.synchronize()
    got = sampled(case, out.float().cpu().numpy())
    ref = _from_bits(golden[case.id], dt).reshape(got.shape)
    assert_close_common(got, ref, dt)
    if dt != "float32":
        assert_max_err_frac(got, ref, 1e-2)


@pytest.mark.parametrize("shape", [(8, 16), (4, 16, 128), (2, 3, 1023), (33, 4096), (5, 8192),
                                   (3, 16384), (2, 40000)], ids=str)
def test_add_rmsnorm_matches_oracle(shape, dtype):
    from aot_kernel import add_rmsnorm

    x = randn(shape, 31, dtype)
    r = randn(shape, 32, dtype)
    w = randn((shape[-1],), 33, dtype, mean=1.0, std=0.1)
    y, h = add_rmsnorm(to_device(x, dtype), to_device(r, dtype), to_device(w, dtype))
    ey, eh = ops.add_rmsnorm(x, r, w, 1e-6, dtype)
    assert_close_np(h, eh, rtol=0, atol=0) if dtype != "float32" else assert_close_common(h, eh, dtype)
    assert_close_common(y, ey, dtype)


def test_add_rmsnorm_in_place_residual():
    """residual_out may alias residual (the usual in-place update)."""
    import torch

    from aot_kernel import capi

    x = randn((64, 4096), 34, "bfloat16")
    r = randn((64, 4096), 35, "bfloat16")
    w = randn((4096,), 36, "bfloat16", mean=1.0, std=0.1)
    tx, tr, tw = to_device(x, "bfloat16"), to_device(r, "bfloat16"), to_device(w, "bfloat16")
    y = torch.empty_like(tx)
    capi.add_rmsnorm_forward(y, tr, tx, tr, tw, 64, 4096, 1e-6, capi.BFLOAT16)
    torch.cuda.synchronize()
    ey, eh = ops.add_rmsnorm(x, r, w, 1e-6, "bfloat16")
    assert_close_np(tr, eh, rtol=0, atol=0)
    assert_close_common(y, ey, "bfloat16")


# ---- full-size configurations ----

def test_rmsnorm_config_size():
    import torch

    from aot_kernel import rms_norm

    x = randn((8192, 4096), 10, "bfloat16")
    w = randn((4096,), 11, "bfloat16", mean=1.0, std=0.1)
    got = rms_norm(to_device(x, "bfloat16"), to_device(w, "bfloat16"))
    torch.cuda.synchronize()
    assert_close_common(got, ops.rmsnorm(x, w, 1e-6, "bfloat16"), "bfloat16")


def test_silu_and_silu_mul_config_size():
    import torch

    from aot_kernel import silu, silu_mul

    g = randn((8192, 14336), 12, "bfloat16", std=2.0)
    u = randn((8192, 14336), 13, "bfloat16", std=2.0)
    tg, tu = to_device(g, "bfloat16"), to_device(u, "bfloat16")
    s = silu(tg)
    sm = silu_mul(tg, tu)
    torch.cuda.synchronize()
    rows = slice(0, 8192, 97)
    assert_close_common(s[rows], ops.silu(g[rows], "bfloat16"), "bfloat16")
    assert_close_common(sm[rows], ops.silu_mul(g[rows], u[rows], "bfloat16"), "bfloat16")


# ---- rms_norm's row statistic and rms_norm folded into the gate/up GEMM ----

@pytest.mark.parametrize("shape", [(4096, 8192), (7, 1000), (3, 4096), (1, 70000)], ids=str)
def test_rms_rstd_matches_oracle(shape):
    import aot_kernel

    x = randn(shape, sum(shape), "bfloat16")
    got = aot_kernel.rms_rstd(to_device(x, "bfloat16"), 1e-6).cpu().numpy()
    want = ops.rms_rstd(x, 1e-6)
    np.testing.assert_allclose(got, want, rtol=1e-5, atol=0)  # fp32 sums in another order


@pytest.mark.parametrize("shape", [(256, 512, 256), (300, 1024, 384), (2048, 4096, 1792),
                                   (4096, 8192, 3584), (1000, 4096, 9344)], ids=str)
def test_gemm_silu_mul_folded_norm_matches_oracle(shape):
    """(M, H, I): rms_rstd(x) + gemm_silu_mul(x, fold_norm_weight(W), row_scale)
    against the folded oracle, and against the unfused rms_norm -> gate/up ->
    silu_mul composition within the GEMM tolerance.  (4096, 8192, 3584) is
    the 8-way tensor-parallel gate/up of the Llama-70B block (896 tiles: 8
    left over, cut along K through the workspace, then row-scaled); the last
    runs on the CTA-pair kernel (256 x 512 tiles, the last one half past 2I)."""
    import torch

    import aot_kernel
    from tests.conftest import assert_close_for_gemm

    M, H, inter = shape
    if shape == (1000, 4096, 9344):
        from aot_kernel import capi

        assert capi.gemm_path(M, 2 * inter, H, 148) == "tc2_wide"
    x = randn((M, H), M + 11, "bfloat16")
    nw = randn((H,), H + 12, "bfloat16", mean=1.0, std=0.1)
    wg = randn((H, inter), H + 13, "bfloat16", std=H ** -0.5)
    wu = randn((H, inter), H + 14, "bfloat16", std=H ** -0.5)
    tx = to_device(x, "bfloat16")
    w = aot_kernel.interleave_gate_up(to_device(wg, "bfloat16"), to_device(wu, "bfloat16"))
    wf = aot_kernel.fold_norm_weight(w, to_device(nw, "bfloat16"))
    act = aot_kernel.gemm_silu_mul(tx, wf, aot_kernel.rms_rstd(tx, 1e-6))
    torch.cuda.synchronize()
    rows = np.unique(np.concatenate([np.random.default_rng(4).integers(0, M, size=40),
                                     np.arange(max(0, M - 128), M, 7)]))
    got = act[torch.as_tensor(rows, device="cuda")]
    assert_close_for_gemm(got, ops.gemm_silu_mul_folded(x[rows], nw, wg, wu, 1e-6, "bfloat16"),
                          "bfloat16")
    unfused = ops.gemm_silu_mul(ops.rmsnorm(x[rows], nw, 1e-6, "bfloat16"), wg, wu, "bfloat16")
    assert_close_for_gemm(got, unfused, "bfloat16")
