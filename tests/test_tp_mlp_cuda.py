"""Tensor-parallel MLP block on B200s: the aot_kernel ops plus one NCCL
all-reduce, against the unsharded oracle composition.  World sizes beyond the
visible GPU count are skipped."""

from __future__ import annotations

import multiprocessing as mp
import os
import socket
import sys
import time
from datetime import timedelta
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

REPO = Path(__file__).resolve().parents[1]
T, H, INTER = 256, 1024, 2048


def _weights():
    from oracle.inputs import randn

    return (randn((T, H), 201), randn((H,), 202, mean=1.0, std=0.1),
            randn((H, 2 * INTER), 203, std=0.03), randn((INTER, H), 204, std=0.03))


def _gpu_count() -> int:
    import torch

    return torch.cuda.device_count()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, chunks: int, out_dir: str,
               allreduce: str = "nccl") -> None:
    for p in (REPO, REPO / "inference-kernel_b200"):
        sys.path.insert(0, str(p))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch
    import torch.distributed as dist

    from aot_kernel.tp_mlp import (MLPShard, TensorParallelMLP, shard_down, shard_gate_up,
                                   shard_gate_up_folded, shard_gate_up_interleaved)

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=dev)
    x, nw, wgu, wd = (torch.from_numpy(a).to(dev, torch.bfloat16) for a in _weights())
    # The fused runs also take the fused gate/up + silu path; "fused_fold"
    # additionally folds rms_norm into it.
    fused_silu = allreduce.startswith("fused")
    fold = allreduce == "fused_fold"
    if fold:
        wgu_r = shard_gate_up_folded(wgu, nw, rank, world)
    else:
        wgu_r = (shard_gate_up_interleaved if fused_silu else shard_gate_up)(wgu, rank, world)
    block = TensorParallelMLP(MLPShard(nw, wgu_r, shard_down(wd, rank, world), fused_silu=fused_silu,
                                       fold_norm=fold),
                              chunks=chunks, allreduce="fused" if fused_silu else allreduce)
    y = block(x)
    y = block(x).clone()  # second call: epoch 2 of the fused path
    torch.cuda.synchronize()
    from aot_kernel import capi

    assert capi.watchdog_status(rank) == 0
    np.save(os.path.join(out_dir, f"y{rank}.npy"), y.float().cpu().numpy())
    dist.barrier()
    dist.destroy_process_group()


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


@pytest.mark.parametrize("world,chunks,allreduce",
                         [(2, 1, "nccl"), (2, 4, "nccl"), (4, 1, "nccl"), (8, 2, "nccl"),
                          (2, 1, "fused"), (4, 1, "fused"), (8, 1, "fused"), (2, 1, "fused_fold"),
                          (8, 1, "fused_fold")])
def test_block_tensor_parallel(world, chunks, allreduce, tmp_path):
    if _gpu_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, chunks, str(tmp_path), allreduce))
             for r in range(world)]
    for p in procs:
        p.start()
    deadline = time.time() + 240
    for p in procs:
        p.join(max(1.0, deadline - time.time()))
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    ys = [np.load(tmp_path / f"y{r}.npy") for r in range(world)]
    for r in range(1, world):
        np.testing.assert_array_equal(ys[r], ys[0])  # every rank holds the same reduced output
    _check(ys[0], world)


def _fused_rank_main(rank: int, world: int, port: int, out_dir: str) -> None:
    for p in (REPO, REPO / "inference-kernel_b200"):
        sys.path.insert(0, str(p))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch
    import torch.distributed as dist

    from aot_kernel import capi
    from aot_kernel.tp_mlp import FusedDownAllReduce
    from oracle.inputs import randn

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=dev)
    M, K, N = FUSED_SHAPE
    fused = FusedDownAllReduce(M, N, torch.bfloat16, dev)
    for it in range(3):  # epochs 1..3 on fresh inputs
        a = torch.from_numpy(randn((M, K), 500 + 10 * it + rank)).to(dev, torch.bfloat16)
        b = torch.from_numpy(randn((K, N), 600 + 10 * it + rank, std=0.05)).to(dev, torch.bfloat16)
        y = fused(a, b)
        torch.cuda.synchronize()
        np.save(os.path.join(out_dir, f"f{rank}_{it}.npy"), y.float().cpu().numpy())
    assert capi.watchdog_status(rank) == 0
    dist.barrier()
    dist.destroy_process_group()


FUSED_SHAPE = (640, 384, 1032)  # M, K per rank, N: partial tiles in M and N


@pytest.mark.parametrize("world", [2, 4, 8])
def test_fused_gemm_allreduce_matches_oracle(world, tmp_path):
    """aotk_gemm_allreduce: every rank holds round(sum_r round(A_r B_r)), over three epochs."""
    if _gpu_count() < world:
        pytest.skip(f"needs {world} GPUs")
    from oracle import ops
    from oracle.inputs import randn

    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_fused_rank_main, args=(r, world, port, str(tmp_path)))
             for r in range(world)]
    for p in procs:
        p.start()
    deadline = time.time() + 240
    for p in procs:
        p.join(max(1.0, deadline - time.time()))
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
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
