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


def _rank_main(rank: int, world: int, port: int, chunks: int, out_dir: str) -> None:
    for p in (REPO, REPO / "inference-kernel_b200"):
        sys.path.insert(0, str(p))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch
    import torch.distributed as dist

    from aot_kernel.tp_mlp import MLPShard, TensorParallelMLP, shard_down, shard_gate_up

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=dev)
    x, nw, wgu, wd = (torch.from_numpy(a).to(dev, torch.bfloat16) for a in _weights())
    block = TensorParallelMLP(MLPShard(nw, shard_gate_up(wgu, rank, world), shard_down(wd, rank, world)),
                              chunks=chunks)
    y = block(x)
    torch.cuda.synchronize()
    np.save(os.path.join(out_dir, f"y{rank}.npy"), y.float().cpu().numpy())
    dist.barrier()
    dist.destroy_process_group()


def _check(y: np.ndarray, world: int) -> None:
    from oracle import ops

    x, nw, wgu, wd = _weights()
    full = ops.mlp_block(x, nw, wgu, wd, 1e-6, "bfloat16")
    err = np.abs(y - full).max()
    assert err <= 2e-2 * np.abs(full).max(), f"W={world}: max|err| {err} vs max|ref| {np.abs(full).max()}"


def test_block_single_gpu():
    import torch

    from aot_kernel.tp_mlp import MLPShard, TensorParallelMLP

    x, nw, wgu, wd = (torch.from_numpy(a).to("cuda", torch.bfloat16) for a in _weights())
    y = TensorParallelMLP(MLPShard(nw, wgu, wd))(x)
    torch.cuda.synchronize()
    _check(y.float().cpu().numpy(), 1)


@pytest.mark.parametrize("world,chunks", [(2, 1), (2, 4), (4, 1), (8, 2)])
def test_block_tensor_parallel(world, chunks, tmp_path):
    if _gpu_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, chunks, str(tmp_path)))
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
