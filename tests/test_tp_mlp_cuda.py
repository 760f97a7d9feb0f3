"""Tensor-parallel MLP block on B200s: the aot_kernel ops plus one all-reduce
(NCCL, or fused into the down GEMM through NVSwitch multicast memory), against
the unsharded oracle composition of ref.rmsnorm (ref/norm.py:11-12), ref.gemm
(ref/gemm.py:4-5) and ref.silu (ref/activation.py:15-16).  World sizes beyond
the visible GPU count are skipped.  Ranks run under ``tests/_ranks.py``: the
parent never ends a rank; each rank bounds and releases itself."""

from __future__ import annotations

import os

import numpy as np
import pytest

from tests._ranks import run_ranks

pytestmark = pytest.mark.gpu

T, H, INTER = 256, 1024, 2048
# The Llama-3-70B block (hidden 8192, intermediate 28672) on 512 tokens.
T70, H70, I70 = 512, 8192, 28672
SAMPLE_ROWS = 48


def _weights():
    from oracle.inputs import randn

    return (randn((T, H), 201), randn((H,), 202, mean=1.0, std=0.1),
            randn((H, 2 * INTER), 203, std=0.03), randn((INTER, H), 204, std=0.03))


def _gpu_count() -> int:
    import torch

    return torch.cuda.device_count()


def _build_block(rank, world, dev, x, nw, wgu, wd, mode, chunks=1):
    from aot_kernel.tp_mlp import (MLPShard, TensorParallelMLP, shard_down, shard_gate_up,
                                   shard_gate_up_folded, shard_gate_up_interleaved)

    # "fused" runs also take the fused gate/up + silu kernel; "fused_fold"
    # additionally folds rms_norm into it.
    fused_silu = mode.startswith("fused")
    fold = mode == "fused_fold"
    if fold:
        wgu_r = shard_gate_up_folded(wgu, nw, rank, world)
    else:
        wgu_r = (shard_gate_up_interleaved if fused_silu else shard_gate_up)(wgu, rank, world)
    return TensorParallelMLP(MLPShard(nw, wgu_r, shard_down(wd, rank, world), fused_silu=fused_silu,
                                      fold_norm=fold),
                             chunks=chunks, allreduce="fused" if fused_silu else mode)


def _block_body(rank, world, dev, out_dir, guard, held, chunks, mode):
    import torch

    from aot_kernel import capi

    x, nw, wgu, wd = (torch.from_numpy(a).to(dev, torch.bfloat16) for a in _weights())
    held["block"] = block = _build_block(rank, world, dev, x, nw, wgu, wd, mode, chunks)
    for _ in range(2):  # the second call is epoch 2 of the fused path
        guard.check()
        y = block(x)
        torch.cuda.synchronize()
    assert capi.watchdog_status(rank) == 0
    np.save(os.path.join(out_dir, f"y{rank}.npy"), y.float().cpu().numpy())


def _check(y: np.ndarray, world: int) -> None:
    from oracle import ops

    x, nw, wgu, wd = _weights()
    full = ops.mlp_block(x, nw, wgu, wd, 1e-6, "bfloat16")
    err = np.abs(y - full).max()
    assert err <= 2e-2 * np.abs(full).max(), f"W={world}: max|err| {err} vs max|ref| {np.abs(full).max()}"


@pytest.mark.parametrize("mode", ["unfused", "fused_silu", "fold_norm"])
def test_block_single_gpu(mode):
    import torch

    from aot_kernel.tp_mlp import (MLPShard, TensorParallelMLP, shard_gate_up_folded,
                                   shard_gate_up_interleaved)

    x, nw, wgu, wd = (torch.from_numpy(a).to("cuda", torch.bfloat16) for a in _weights())
    if mode == "fused_silu":
        wgu = shard_gate_up_interleaved(wgu, 0, 1)
    elif mode == "fold_norm":
        wgu = shard_gate_up_folded(wgu, nw, 0, 1)
    y = TensorParallelMLP(MLPShard(nw, wgu, wd, fused_silu=mode != "unfused",
                                   fold_norm=mode == "fold_norm"))(x)
    torch.cuda.synchronize()
    _check(y.float().cpu().numpy(), 1)


@pytest.mark.parametrize("world,chunks,mode",
                         [(2, 1, "nccl"), (2, 4, "nccl"), (4, 1, "nccl"), (8, 2, "nccl"),
                          (2, 1, "fused"), (4, 1, "fused"), (8, 1, "fused"), (2, 1, "fused_fold"),
                          (4, 1, "fused_fold"), (8, 1, "fused_fold")])
def test_block_tensor_parallel(world, chunks, mode, tmp_path):
    if _gpu_count() < world:
        pytest.skip(f"needs {world} GPUs")
    codes = run_ranks(_block_body, world, tmp_path, (chunks, mode), nvls=mode != "nccl")
    assert codes == [0] * world, codes
    ys = [np.load(tmp_path / f"y{r}.npy") for r in range(world)]
    for r in range(1, world):
        np.testing.assert_array_equal(ys[r], ys[0])  # every rank holds the same reduced output
    _check(ys[0], world)


def _weights70(dev):
    """The 70B block's inputs drawn on the device (torch Philox, seeded), as
    the benchmark draws them."""
    import torch

    def rand(shape, seed, std=1.0, mean=0.0):
        g = torch.Generator(device=dev)
        g.manual_seed(seed)
        return (torch.randn(shape, generator=g, device=dev) * std + mean).to(torch.bfloat16)

    return (rand((T70, H70), 30), rand((H70,), 31, 0.1, 1.0), rand((H70, 2 * I70), 32, 0.02),
            rand((I70, H70), 33, 0.02))


def _rows70():
    return np.random.default_rng(7).choice(T70, SAMPLE_ROWS, replace=False)


def _block70_body(rank, world, dev, out_dir, guard, held, mode):
    import torch

    from aot_kernel import capi

    x, nw, wgu, wd = _weights70(dev)
    held["block"] = block = _build_block(rank, world, dev, x, nw, wgu, wd, mode)
    del wgu, wd
    torch.cuda.empty_cache()
    for _ in range(3):
        guard.check()
        y = block(x)
        torch.cuda.synchronize()
    assert capi.watchdog_status(rank) == 0
    rows = torch.from_numpy(_rows70()).to(dev)
    np.save(os.path.join(out_dir, f"y70_{rank}.npy"), y[rows].float().cpu().numpy())


@pytest.mark.parametrize("world,mode", [(1, "fused_fold"), (2, "fused_fold"), (8, "fused_fold"),
                                        (8, "nccl")])
def test_block_70b_shape(world, mode, tmp_path):
    """The Llama-3-70B block (H = 8192, I = 28672) on 512 tokens: sampled rows
    of every rank's output against the unsharded reference composition."""
    if _gpu_count() < world:
        pytest.skip(f"needs {world} GPUs")
    from oracle import ops

    codes = run_ranks(_block70_body, world, tmp_path, (mode,), nvls=mode != "nccl")
    assert codes == [0] * world, codes
    import torch

    # the same seeded draws, regenerated here once the ranks have ended
    x, nw, wgu, wd = (t.float().cpu().numpy() for t in _weights70(torch.device("cuda", 0)))
    torch.cuda.empty_cache()
    full = ops.mlp_block(x[_rows70()], nw, wgu, wd, 1e-6, "bfloat16")
    ys = [np.load(tmp_path / f"y70_{r}.npy") for r in range(world)]
    for r in range(1, world):
        np.testing.assert_array_equal(ys[r], ys[0])
    err = np.abs(ys[0] - full).max()
    assert err <= 2e-2 * np.abs(full).max(), f"W={world}: max|err| {err} vs {np.abs(full).max()}"


FUSED_SHAPE = (640, 384, 1032)  # M, K per rank, N: partial tiles in M and N


def _fused_body(rank, world, dev, out_dir, guard, held):
    import torch

    from aot_kernel import capi
    from aot_kernel.tp_mlp import FusedDownAllReduce
    from oracle.inputs import randn

    M, K, N = FUSED_SHAPE
    held["fused"] = fused = FusedDownAllReduce(M, N, torch.bfloat16, dev)
    for it in range(3):  # epochs 1..3 on fresh inputs
        a = torch.from_numpy(randn((M, K), 500 + 10 * it + rank)).to(dev, torch.bfloat16)
        b = torch.from_numpy(randn((K, N), 600 + 10 * it + rank, std=0.05)).to(dev, torch.bfloat16)
        guard.check()
        y = fused(a, b)
        torch.cuda.synchronize()
        np.save(os.path.join(out_dir, f"f{rank}_{it}.npy"), y.float().cpu().numpy())
    assert capi.watchdog_status(rank) == 0


@pytest.mark.parametrize("world", [2, 4, 8])
def test_fused_gemm_allreduce_matches_oracle(world, tmp_path):
    """aotk_gemm_allreduce: every rank holds round(sum_r round(A_r B_r)), over three epochs."""
    if _gpu_count() < world:
        pytest.skip(f"needs {world} GPUs")
    from oracle import ops
    from oracle.inputs import randn

    codes = run_ranks(_fused_body, world, tmp_path)
    assert codes == [0] * world, codes
    M, K, N = FUSED_SHAPE
    for it in range(3):
        parts = [ops.gemm(randn((M, K), 500 + 10 * it + r), randn((K, N), 600 + 10 * it + r, std=0.05),
                          "bfloat16") for r in range(world)]
        expect = ops.round_to(np.sum(parts, axis=0, dtype=np.float32), "bfloat16")
        ys = [np.load(tmp_path / f"f{r}_{it}.npy") for r in range(world)]
        for r in range(world):
            np.testing.assert_array_equal(ys[r], ys[0])
        err = np.abs(ys[0] - expect).max()
        assert err <= 2e-2 * np.abs(expect).max(), f"epoch {it + 1}: max|err| {err}"
