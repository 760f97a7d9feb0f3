"""GEMM parity on a B200: every path against the oracle (and, through the
golden file, against the reference's own outputs)."""

from __future__ import annotations

import numpy as np
import pytest

from cases import GEMM_SHAPES
from tests.conftest import assert_close_for_gemm, to_device, torch_dtype
from oracle import ops
from oracle.inputs import randn

pytestmark = pytest.mark.gpu


def _inputs(M, K, N, dtype, seed=0, a_std=1.0, b_std=1.0):
    return randn((M, K), seed, dtype, std=a_std), randn((K, N), seed + 1, dtype, std=b_std)


# ---- through the operator API (the reference's tests/gemm/test_cuda.py:14-41) ----

@pytest.mark.parametrize("impl", ["gemm", "gemm_naive"])
@pytest.mark.parametrize("shape", GEMM_SHAPES + [(1, 64, 256), (300, 520, 328)], ids=str)
def test_gemm_matches_oracle(impl, shape, dtype):
    import aot_kernel

    M, K, N = shape
    a, b = _inputs(M, K, N, dtype, seed=M * 7 + K)
    got = getattr(aot_kernel, impl)(to_device(a, dtype), to_device(b, dtype))
    assert got.dtype == torch_dtype(dtype) and tuple(got.shape) == (M, N)
    assert_close_for_gemm(got, ops.gemm(a, b, dtype), dtype)


def test_gemm_preserves_shape_and_dtype(dtype):
    import torch

    from aot_kernel.gemm import gemm

    a = torch.randn(3, 5, dtype=torch_dtype(dtype), device="cuda")
    b = torch.randn(5, 7, dtype=torch_dtype(dtype), device="cuda")
    c = gemm(a, b)
    assert c.shape == (3, 7) and c.dtype == a.dtype


def test_gemm_rejects_non_contiguous():
    import torch

    from aot_kernel.gemm import gemm

    a = torch.randn(8, 8, device="cuda").t()
    with pytest.raises((ValueError, RuntimeError, AssertionError)):
        gemm(a, torch.randn(8, 8, device="cuda"))


def test_gemm_rejects_mismatched_dtype():
    import torch

    from aot_kernel.gemm import gemm

    a = torch.randn(8, 8, device="cuda", dtype=torch.float32)
    b = torch.randn(8, 8, device="cuda", dtype=torch.float16)
    with pytest.raises((ValueError, RuntimeError)):
        gemm(a, b)


def test_gemm_empty_k_gives_zeros():
    import torch

    from aot_kernel.gemm import gemm

    a = torch.empty(4, 0, device="cuda", dtype=torch.bfloat16)
    b = torch.empty(0, 8, device="cuda", dtype=torch.bfloat16)
    assert torch.count_nonzero(gemm(a, b)) == 0


# ---- through the C ABI, one kernel at a time ----

def _run_capi(fn, a, b, dtype):
    import torch

    from aot_kernel import capi

    M, K = a.shape
    N = b.shape[1]
    ta, tb = to_device(a, dtype), to_device(b, dtype)
    tc = torch.full((M, N), float("nan"), device="cuda", dtype=torch_dtype(dtype))
    fn(tc, ta, tb, M, N, K, capi.dtype_code(torch_dtype(dtype)))
    torch.cuda.synchronize()
    return tc


TC_SHAPES = [(128, 64, 256), (256, 128, 512), (129, 72, 264), (300, 328, 520), (1000, 4096, 264),
             (640, 1024, 2048), (1024, 1024, 1024)]


@pytest.mark.parametrize("shape", TC_SHAPES, ids=str)
@pytest.mark.parametrize("dt", ["bfloat16", "float16"])
def test_capi_gemm_tc(shape, dt):
    from aot_kernel import capi

    M, K, N = shape
    a, b = _inputs(M, K, N, dt, seed=M + N)
    got = _run_capi(capi.gemm_tc, a, b, dt)
    assert_close_for_gemm(got, ops.gemm(a, b, dt), dt)
    assert capi.watchdog_status() == 0


# Most of these leave a last round of at most 37 pair tiles (or are a single
# such round), which the kernel cuts into N halves.
@pytest.mark.parametrize("shape", TC_SHAPES + [(256, 64, 256), (8192, 1024, 2048),
                                               (1024, 512, 4864), (1000, 512, 4856)], ids=str)
@pytest.mark.parametrize("dt", ["bfloat16", "float16"])
def test_capi_gemm_tc2(shape, dt):
    from aot_kernel import capi

    M, K, N = shape
    a, b = _inputs(M, K, N, dt, seed=2 * M + N)
    got = _run_capi(capi.gemm_tc2, a, b, dt)
    assert_close_for_gemm(got, ops.gemm(a, b, dt), dt)
    assert capi.watchdog_status() == 0


# The 256 x 512 pair tile: partial tiles in M (rows of the second CTA past M)
# and N (the second MMA's columns past N), a single tile, several waves; a
# last round of at most 37 tiles runs as N halves of 256 columns ((256, 64,
# 512), (520, 4096, 1544), (2304, 512, 5120), (1000, 512, 4600) with a
# ragged last half, (4096, 512, 10240) after four whole rounds).
TC2W_SHAPES = TC_SHAPES + [(256, 64, 512), (520, 4096, 1544), (8192, 1024, 2048),
                           (2304, 512, 5120), (1000, 512, 4600), (4096, 512, 10240)]


@pytest.mark.parametrize("shape", TC2W_SHAPES, ids=str)
@pytest.mark.parametrize("dt", ["bfloat16", "float16"])
def test_capi_gemm_tc2w(shape, dt):
    from aot_kernel import capi

    M, K, N = shape
    a, b = _inputs(M, K, N, dt, seed=5 * M + N)
    got = _run_capi(capi.gemm_tc2w, a, b, dt)
    assert_close_for_gemm(got, ops.gemm(a, b, dt), dt)
    assert capi.watchdog_status() == 0


SKINNY = [(1, 64, 256), (1, 4096, 1024), (3, 328, 520), (16, 1024, 2048), (17, 512, 264),
          (64, 2048, 768), (100, 1000, 1032), (128, 4096, 512)]


@pytest.mark.parametrize("shape", SKINNY, ids=str)
@pytest.mark.parametrize("dt", ["bfloat16", "float16"])
def test_capi_gemm_skinny(shape, dt):
    from aot_kernel import capi

    M, K, N = shape
    a, b = _inputs(M, K, N, dt, seed=3 * M + N)
    got = _run_capi(capi.gemm_skinny, a, b, dt)
    assert_close_for_gemm(got, ops.gemm(a, b, dt), dt)
    assert capi.watchdog_status() == 0


def test_capi_tc_rejects_unaligned():
    import torch

    from aot_kernel import capi

    a = torch.zeros(16, 33, device="cuda", dtype=torch.bfloat16)
    b = torch.zeros(33, 16, device="cuda", dtype=torch.bfloat16)
    c = torch.zeros(16, 16, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(capi.AotkError) as e:
        capi.gemm_tc(c, a, b, 16, 16, 33, capi.BFLOAT16)
    assert e.value.status == capi.ERR_UNSUPPORTED


def test_output_canaries_untouched():
    """Writes stay inside C: the rows/columns around a sub-block view keep their sentinel."""
    import torch

    from aot_kernel import capi

    M, K, N = 200, 256, 264
    a, b = _inputs(M, K, N, "bfloat16", seed=11)
    big = torch.full((M + 16, N + 8), 7.0, device="cuda", dtype=torch.bfloat16)
    # C occupies rows 8..8+M of a [M+16, N] dense buffer region: use a separate dense buffer
    # with guard rows before and after.
    buf = torch.full(((M + 16) * N,), 7.0, device="cuda", dtype=torch.bfloat16)
    c = buf[8 * N: 8 * N + M * N].view(M, N)
    for fn in (capi.gemm_tc, capi.gemm_skinny if M <= 128 else None):
        if fn is None:
            continue
        fn(c, to_device(a, "bfloat16"), to_device(b, "bfloat16"), M, N, K, capi.BFLOAT16)
    torch.cuda.synchronize()
    assert torch.all(buf[: 8 * N] == 7.0) and torch.all(buf[8 * N + M * N:] == 7.0)
    del big


# ---- full-size configurations, checked on sampled rows ----

FULL = [
    (8192, 8192, 8192),       # square sweep, the headline size
    (2048, 2048, 2048),
    (4096, 4096, 4096),
    (1, 4096, 28672),         # Llama-3-8B fused gate+up, decode
    (16, 4096, 6144),
    (128, 14336, 4096),
    (128, 4096, 28672),       # M <= 128 on the 1-CTA kernel: 112 whole tiles, one wave
    (2048, 4096, 28672),
    (8192, 14336, 4096),
    (8192, 4096, 28672),      # the pair kernel on 256 x 512 tiles (aotk_gemm_path)
    (2048, 14336, 4096),
    # the TP block's down GEMM per rank at W = 1 / 2 / 4: 256 x 512 pair
    # tiles, 3 rounds on 74 pairs and 34 tiles run as 256-column halves
    (4096, 28672, 8192),
    (4096, 14336, 8192),
    (4096, 7168, 8192),
]


@pytest.mark.parametrize("shape", FULL, ids=str)
def test_full_size_sampled_rows(shape):
    import torch

    import aot_kernel

    M, K, N = shape
    a, b = _inputs(M, K, N, "bfloat16", seed=5, b_std=(1.0 / np.sqrt(K)) if M == K == N else 0.02)
    got = aot_kernel.gemm(to_device(a, "bfloat16"), to_device(b, "bfloat16"))
    torch.cuda.synchronize()
    rows = np.unique(np.random.default_rng(0).integers(0, M, size=min(M, 48)))
    expect = ops.gemm(a[rows], b, "bfloat16")
    assert_close_for_gemm(got[torch.as_tensor(rows, device="cuda")], expect, "bfloat16")


# ---- K-split last wave (aotk_gemm_opt_ws) ----

# (M, K, N) whose tail is cut along K on a 148-SM B200: 8, 22, 8 tiles left
# after whole waves (K = 8192), a single partial wave of 16 tiles, and a
# ragged single wave of 32 tiles.
SPLIT_SHAPES = [(2048, 8192, 14336), (1280, 8192, 4352), (4096, 8192, 7168), (256, 8192, 2048),
                (1000, 8192, 1000)]
# (M, K, N) whose tail runs as N halves: 68, 16 and 12 tiles left (K too short
# to split), and single partial waves of 9 and 64 tiles.
HALF_SHAPES = [(4096, 4096, 4096), (2048, 4096, 28672), (2560, 1024, 2048), (300, 328, 768),
               (1024, 2048, 2048)]


@pytest.mark.parametrize("shape", SPLIT_SHAPES, ids=str)
def test_split_last_wave_matches_oracle(shape):
    """Shapes whose tile count leaves a small partial last wave: the leftover
    tiles are computed in K splits through a workspace and must match the
    oracle, be bit-identical across calls, and not depend on the workspace
    contents."""
    import torch

    from aot_kernel import capi

    M, K, N = shape
    a, b = _inputs(M, K, N, "bfloat16", seed=M + 3 * N, b_std=K ** -0.5)
    ta, tb = to_device(a, "bfloat16"), to_device(b, "bfloat16")
    ws_bytes = capi.gemm_opt_workspace_size(M, N, K, capi.BFLOAT16)
    assert ws_bytes > 0, "shape expected to use the split schedule"
    ws = torch.full((ws_bytes,), 0xAB, dtype=torch.uint8, device="cuda")  # garbage on purpose
    outs = []
    for _ in range(2):
        c = torch.empty((M, N), device="cuda", dtype=torch.bfloat16)
        capi.gemm_opt_ws(c, ta, tb, M, N, K, capi.BFLOAT16, ws, ws_bytes)
        outs.append(c)
    torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[1])
    rows = np.unique(np.random.default_rng(1).integers(0, M, size=64))
    # the split tiles are the last ones in raster order: check the last 128-row block too
    rows = np.unique(np.concatenate([rows, np.arange(M - 128, M, 7)]))
    expect = ops.gemm(a[rows], b, "bfloat16")
    assert_close_for_gemm(outs[0][torch.as_tensor(rows, device="cuda")], expect, "bfloat16")
    assert capi.watchdog_status() == 0


@pytest.mark.parametrize("shape", HALF_SHAPES, ids=str)
def test_half_tile_tail_matches_oracle(shape):
    """Tails run as two N halves per tile need no workspace: compared with the
    oracle on sampled rows and the last row block, and with an fp32 torch
    matmul of the same inputs on every element."""
    import torch

    from aot_kernel import capi

    M, K, N = shape
    a, b = _inputs(M, K, N, "bfloat16", seed=M + 5 * N, b_std=K ** -0.5)
    ta, tb = to_device(a, "bfloat16"), to_device(b, "bfloat16")
    assert capi.gemm_opt_workspace_size(M, N, K, capi.BFLOAT16) == 0
    c = torch.empty((M, N), device="cuda", dtype=torch.bfloat16)
    capi.gemm_tc(c, ta, tb, M, N, K, capi.BFLOAT16)
    rows = np.unique(np.concatenate([np.random.default_rng(3).integers(0, M, size=48),
                                     np.arange(max(0, M - 128), M, 5)]))
    expect = ops.gemm(a[rows], b, "bfloat16")
    assert_close_for_gemm(c[torch.as_tensor(rows, device="cuda")], expect, "bfloat16")
    torch.backends.cuda.matmul.allow_tf32 = False
    full = (ta.float() @ tb.float()).to(torch.bfloat16)
    torch.cuda.synchronize()
    assert_close_for_gemm(c, full, "bfloat16")
    assert capi.watchdog_status() == 0


def test_half_tiles_equal_whole_tiles():
    """A tail tile run as two N halves (MMA N = 128) gives the same bits as the
    same tile run whole (N = 256): 4096^3 leaves 68 tail tiles (halves);
    the same rows computed as two 2048-row GEMMs (256 tiles: one wave and
    108 whole tiles) must agree exactly."""
    import torch

    from aot_kernel import capi

    M, K, N = 4096, 4096, 4096
    a, b = _inputs(M, K, N, "bfloat16", seed=31, b_std=K ** -0.5)
    ta, tb = to_device(a, "bfloat16"), to_device(b, "bfloat16")
    halves = torch.empty((M, N), device="cuda", dtype=torch.bfloat16)
    capi.gemm_tc(halves, ta, tb, M, N, K, capi.BFLOAT16)
    whole = torch.empty_like(halves)
    for r0 in (0, M // 2):
        capi.gemm_tc(whole[r0:r0 + M // 2], ta[r0:r0 + M // 2], tb, M // 2, N, K, capi.BFLOAT16)
    torch.cuda.synchronize()
    assert torch.equal(halves, whole)


def test_split_and_whole_schedules_agree():
    import torch

    import aot_kernel
    from aot_kernel import capi

    M, K, N = 1280, 8192, 4352
    a, b = _inputs(M, K, N, "bfloat16", seed=77, b_std=K ** -0.5)
    ta, tb = to_device(a, "bfloat16"), to_device(b, "bfloat16")
    whole = torch.empty((M, N), device="cuda", dtype=torch.bfloat16)
    capi.gemm_tc(whole, ta, tb, M, N, K, capi.BFLOAT16)
    split = aot_kernel.gemm(ta, tb)  # the op allocates the workspace
    torch.cuda.synchronize()
    diff = (whole.float() - split.float()).abs().max().item()
    assert diff <= 2e-2 * whole.float().abs().max().item()


# ---- gate/up GEMM fused with silu(gate) * up ----

@pytest.mark.parametrize("shape", [(256, 512, 256), (300, 328, 384), (2560, 1024, 1024),
                                   (4096, 8192, 3584), (2048, 4096, 3072), (1024, 4096, 9472),
                                   (1000, 4096, 9344), (1000, 4096, 1280), (1000, 4096, 1024),
                                   (1000, 4096, 15488), (4096, 8192, 14336)],
                         ids=str)
def test_gemm_silu_mul_matches_oracle(shape):
    """(M, K, I): interleaved [K, 2I] weight, act [M, I]; the tails of the
    first three run as N halves (each half keeps matching gate and up
    columns), (4096, 8192, 3584) leaves 8 tiles cut along K (fused finalize);
    (1024, 4096, 9472) and (1000, 4096, 9344) run on the CTA-pair kernel on
    256 x 512 tiles (two gate/up block pairs; ragged M, and a last tile whose
    second pair is past 2I), (1000, 4096, 1280) on 256 x 256 pair tiles, and
    (1000, 4096, 1024) on 256 x 256 pair tiles cut into N halves (32 tiles
    on 64 pairs: gate and up quarters stay together), and (1000, 4096,
    15488) on 256 x 512 tiles whose last 22 run as halves of one [gate | up]
    block each (the last tile's second block is past 2I), as do the last 8
    tiles of (4096, 8192, 14336), the TP block's gate/up per rank at W = 2."""
    import torch

    import aot_kernel
    from aot_kernel import capi

    M, K, inter = shape
    expect_path = {(1024, 4096, 9472): "tc2_wide", (1000, 4096, 9344): "tc2_wide",
                   (1000, 4096, 1280): "tc2", (1000, 4096, 1024): "tc2",
                   (1000, 4096, 15488): "tc2_wide", (4096, 8192, 14336): "tc2_wide"}.get(shape)
    if expect_path:
        assert capi.gemm_path(M, 2 * inter, K, 148) == expect_path
    a = randn((M, K), M + 1, "bfloat16")
    wg = randn((K, inter), K + 2, "bfloat16", std=K ** -0.5)
    wu = randn((K, inter), K + 3, "bfloat16", std=K ** -0.5)
    ta = to_device(a, "bfloat16")
    w = aot_kernel.interleave_gate_up(to_device(wg, "bfloat16"), to_device(wu, "bfloat16"))
    act = aot_kernel.gemm_silu_mul(ta, w)
    torch.cuda.synchronize()
    rows = np.unique(np.concatenate([np.random.default_rng(2).integers(0, M, size=48),
                                     np.arange(max(0, M - 128), M, 9)]))
    expect = ops.gemm_silu_mul(a[rows], wg, wu, "bfloat16")
    got = act[torch.as_tensor(rows, device="cuda")]
    assert_close_for_gemm(got, expect, "bfloat16")
    # agrees with the unfused composition within the GEMM tolerance
    gate = aot_kernel.gemm(ta, to_device(wg, "bfloat16"))
    up = aot_kernel.gemm(ta, to_device(wu, "bfloat16"))
    ref2 = aot_kernel.silu_mul(gate, up)
    assert_close_for_gemm(act, ref2, "bfloat16")


# ---- host-resident operands (aot_kernel.gemm_host / aotk_gemm_host) ----

@pytest.mark.parametrize("shape", [(1000, 512, 776), (3000, 1024, 2048), (100, 256, 512),
                                   (2048, 4096, 4096)], ids=str)
@pytest.mark.parametrize("pinned", [True, False], ids=["pinned", "pageable"])
def test_gemm_host_matches_oracle(shape, pinned):
    """Row blocks of A (a remainder block, a single block, eight full blocks)
    streamed in while earlier blocks compute; pageable buffers stay correct."""
    import torch

    import aot_kernel

    M, K, N = shape
    a, b = _inputs(M, K, N, "bfloat16", seed=M + K + N, b_std=K ** -0.5)
    ta = torch.from_numpy(a).to(torch.bfloat16)
    tb = torch.from_numpy(b).to(torch.bfloat16)
    if pinned:
        ta, tb = ta.pin_memory(), tb.pin_memory()
    c = aot_kernel.gemm_host(ta, tb)
    assert not c.is_cuda and tuple(c.shape) == (M, N)
    rows = np.unique(np.concatenate([np.random.default_rng(5).integers(0, M, size=40),
                                     np.arange(max(0, M - 130), M, 3)]))
    assert_close_for_gemm(c[torch.as_tensor(rows)], ops.gemm(a[rows], b, "bfloat16"), "bfloat16")


def test_gemm_host_through_c_abi_on_a_side_stream():
    import torch

    from aot_kernel import capi

    M, K, N = 1536, 1024, 1024
    a, b = _inputs(M, K, N, "bfloat16", seed=9, b_std=K ** -0.5)
    ta = torch.from_numpy(a).to(torch.bfloat16).pin_memory()
    tb = torch.from_numpy(b).to(torch.bfloat16).pin_memory()
    c = torch.full((M, N), float("nan"), dtype=torch.bfloat16).pin_memory()
    a_d = torch.empty((M, K), dtype=torch.bfloat16, device="cuda")
    b_d = torch.empty((K, N), dtype=torch.bfloat16, device="cuda")
    c_d = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
    side = torch.cuda.Stream()
    for _ in range(2):  # the second call reuses the device buffers after the first
        capi.gemm_host(c, ta, tb, M, N, K, capi.BFLOAT16, a_d, b_d, c_d, stream=side.cuda_stream)
    side.synchronize()
    assert not torch.isnan(c).any()
    rows = np.arange(0, M, 37)
    assert_close_for_gemm(c[torch.as_tensor(rows)], ops.gemm(a[rows], b, "bfloat16"), "bfloat16")
