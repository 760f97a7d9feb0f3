"""aotk_gemm_opt_noalloc: the GEMM entry point for callers that cannot
allocate device memory (an FFI host with no CUDA allocator of its own, or a
serving loop that must not call cudaMalloc).  Its K-split scratch is a static
array inside libaotk.so.  Checked through the C ABI against aotk_gemm_opt_ws
with a caller-allocated workspace, on two calls in a row.  Kept in its own
file, named to be collected last."""

from __future__ import annotations

import pytest

from tests.conftest import to_device
from oracle.inputs import randn

pytestmark = pytest.mark.gpu

# (M, K, N): the first two leave a small partial last wave (8 and 22 tiles of
# 128 x 256 on a 148-SM B200) with K long enough to be split along K through
# the scratch; the third is a single partial wave (16 tiles) split the same
# way; the last needs none (whole tiles only).
SHAPES = [(2048, 8192, 14336), (1280, 8192, 4352), (256, 8192, 2048), (8192, 1024, 8192)]


@pytest.mark.parametrize("shape", SHAPES, ids=str)
def test_noalloc_matches_workspace_entry_point(shape):
    import torch

    from aot_kernel import capi

    M, K, N = shape
    a = to_device(randn((M, K), 900 + M, "bfloat16"), "bfloat16")
    b = to_device(randn((K, N), 901 + N, "bfloat16", std=K ** -0.5), "bfloat16")
    ws_bytes = capi.gemm_opt_workspace_size(M, N, K, capi.BFLOAT16)
    assert (ws_bytes > 0) == (shape != SHAPES[-1])
    ws = torch.empty((max(ws_bytes, 1),), dtype=torch.uint8, device="cuda")
    ref = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
    capi.gemm_opt_ws(ref, a, b, M, N, K, capi.BFLOAT16, ws, ws_bytes)
    outs = []
    for _ in range(2):  # two calls in a row share the static scratch
        c = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device="cuda")
        capi.gemm_opt_noalloc(c, a, b, M, N, K, capi.BFLOAT16)
        outs.append(c)
    torch.cuda.synchronize()
    for c in outs:
        assert not torch.isnan(c).any()
        assert torch.equal(c, ref)  # same schedule, deterministic split order
    assert capi.watchdog_status() == 0


def test_noalloc_takes_no_device_memory():
    """After a first call (which only looks up the static array's address),
    further calls leave the device's free memory exactly where it was."""
    import torch

    from aot_kernel import capi

    M, K, N = SHAPES[0]
    a = to_device(randn((M, K), 910, "bfloat16"), "bfloat16")
    b = to_device(randn((K, N), 911, "bfloat16", std=K ** -0.5), "bfloat16")
    c = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
    capi.gemm_opt_noalloc(c, a, b, M, N, K, capi.BFLOAT16)
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    for _ in range(3):
        capi.gemm_opt_noalloc(c, a, b, M, N, K, capi.BFLOAT16)
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0
    assert capi.watchdog_status() == 0

