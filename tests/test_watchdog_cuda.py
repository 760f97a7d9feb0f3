"""Failure detection on the GPU without a fault: the bounded waits of the
tensor-core kernels give up, report through the watchdog word, and leave the
context usable."""

import pytest

from oracle import ops
from oracle.inputs import randn
from tests.conftest import assert_close_for_gemm, to_device

pytestmark = pytest.mark.gpu


def test_bounded_waits_time_out_and_report():
    import time

    import torch

    from aot_kernel import capi

    capi.watchdog_status(clear=True)
    t0 = time.time()
    capi.watchdog_selftest()
    torch.cuda.synchronize()
    elapsed = time.time() - t0
    status = capi.watchdog_status(clear=True)
    assert status & 128, f"mbarrier wait did not report (status {status:#x})"
    assert status & 64, f"flag wait did not report (status {status:#x})"
    assert elapsed < 30.0
    assert capi.watchdog_status() == 0  # cleared

    # the context is still good: a GEMM on the tensor cores afterwards is correct
    M, K, N = 256, 512, 264
    a, b = randn((M, K), 1, "bfloat16"), randn((K, N), 2, "bfloat16")
    c = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
    capi.gemm_tc(c, to_device(a, "bfloat16"), to_device(b, "bfloat16"), M, N, K, capi.BFLOAT16)
    torch.cuda.synchronize()
    assert_close_for_gemm(c, ops.gemm(a, b, "bfloat16"), "bfloat16")
    assert capi.watchdog_status() == 0
