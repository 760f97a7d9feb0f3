"""Tensor-parallel MLP host logic on CPU ranks (gloo): sharding, the single
all-reduce, chunked overlap, and failure detection.  The block runs on
oracle-backed CPU ops injected through ``TensorParallelMLP(ops=...)``; the GPU
kernels are covered by the ``gpu`` tests."""

from __future__ import annotations

import multiprocessing as mp
import os
import socket
import sys
import time
from datetime import timedelta
from pathlib import Path
from types import SimpleNamespace

import numpy as np
import pytest

REPO = Path(__file__).resolve().parents[1]
T, H, INTER = 12, 64, 96
SEEDS = (101, 102, 103, 104)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _weights(mode: str = "plain"):
    """Block weights; the fused layouts need 128-column blocks per rank, so
    their intermediate size is 512 (4 ranks x 128)."""
    from oracle.inputs import randn

    inter = INTER if mode == "plain" else 512
    x = randn((T, H), SEEDS[0])
    nw = randn((H,), SEEDS[1], mean=1.0, std=0.1)
    wgu = randn((H, 2 * inter), SEEDS[2], std=0.15)
    wd = randn((inter, H), SEEDS[3], std=0.15 * (INTER / inter) ** 0.5)
    return x, nw, wgu, wd


def _cpu_ops() -> SimpleNamespace:
    import torch

    from oracle import ops

    def rms_norm(x, w, eps):
        return torch.from_numpy(ops.rmsnorm(x.numpy(), w.numpy(), eps, "bfloat16"))

    def gemm(a, b, out=None):
        r = torch.from_numpy(ops.gemm(a.contiguous().numpy(), b.numpy(), "bfloat16"))
        if out is None:
            return r
        out.copy_(r)
        return out

    def silu_mul(g, u):
        return torch.from_numpy(ops.silu_mul(g.contiguous().numpy(), u.contiguous().numpy(), "bfloat16"))

    def rms_rstd(x, eps):
        return torch.from_numpy(ops.rms_rstd(x.float().numpy(), eps))

    def gemm_silu_mul(a, w, row_scale=None):
        # w is [K, 2I] with gate and up interleaved in 128-column blocks
        K, n2 = w.shape
        blocks = w.float().reshape(K, n2 // 256, 2, 128)
        wg = blocks[:, :, 0, :].reshape(K, n2 // 2).numpy()
        wu = blocks[:, :, 1, :].reshape(K, n2 // 2).numpy()
        a32 = a.float().numpy()
        g, u = a32 @ wg, a32 @ wu
        if row_scale is not None:
            rs = row_scale.float().numpy().reshape(-1, 1)
            g, u = g * rs, u * rs
        return torch.from_numpy(ops.silu_mul(g, u, "bfloat16"))

    return SimpleNamespace(rms_norm=rms_norm, gemm=gemm, silu_mul=silu_mul, rms_rstd=rms_rstd,
                           gemm_silu_mul=gemm_silu_mul)


def _rank_main(rank: int, world: int, port: int, chunks: int, out_dir: str, fail_rank: int,
               mode: str = "plain") -> None:
    for p in (REPO, REPO / "inference-kernel_b200"):
        sys.path.insert(0, str(p))
    import torch
    import torch.distributed as dist

    from aot_kernel.tp_mlp import (MLPShard, TensorParallelMLP, shard_down, shard_gate_up,
                                   shard_gate_up_folded, shard_gate_up_interleaved)

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=8))
    x, nw, wgu, wd = (torch.from_numpy(a) for a in _weights(mode))
    if mode == "fold":
        wgu_r = shard_gate_up_folded(wgu, nw, rank, world)
    elif mode == "fused_silu":
        wgu_r = shard_gate_up_interleaved(wgu, rank, world)
    else:
        wgu_r = shard_gate_up(wgu, rank, world)
    shard = MLPShard(nw, wgu_r, shard_down(wd, rank, world), fused_silu=mode != "plain",
                     fold_norm=mode == "fold")
    block = TensorParallelMLP(shard, chunks=chunks, ops=_cpu_ops())
    if rank == fail_rank:
        os._exit(3)  # a rank that dies before the collective
    t0 = time.time()
    try:
        y = block(x)
        np.save(os.path.join(out_dir, f"y{rank}.npy"), y.numpy())
    except Exception as e:  # noqa: BLE001  (the failure the test expects)
        Path(out_dir, f"err{rank}.txt").write_text(f"{type(e).__name__} after {time.time() - t0:.1f}s")
    try:
        dist.destroy_process_group()
    except Exception:  # noqa: BLE001
        pass


def _launch(world: int, chunks: int, tmp_path, fail_rank: int = -1, timeout: float = 120.0,
            mode: str = "plain"):
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_rank_main,
                         args=(r, world, port, chunks, str(tmp_path), fail_rank, mode))
             for r in range(world)]
    for p in procs:
        p.start()
    deadline = time.time() + timeout
    for p in procs:
        p.join(max(1.0, deadline - time.time()))
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "ranks still running after the deadline (hang)"
    return procs


@pytest.mark.parametrize("world,chunks", [(1, 1), (2, 1), (4, 1), (2, 3), (4, 2)])
def test_tp_block_matches_oracle(world, chunks, tmp_path):
    from oracle import ops

    _launch(world, chunks, tmp_path)
    x, nw, wgu, wd = _weights()
    sharded = ops.mlp_block_sharded(x, nw, wgu, wd, 1e-6, "bfloat16", world)
    full = ops.mlp_block(x, nw, wgu, wd, 1e-6, "bfloat16")
    for r in range(world):
        y = ops.round_to(np.load(tmp_path / f"y{r}.npy"), "bfloat16")
        # every rank holds the same reduced output
        np.testing.assert_allclose(y, sharded, rtol=1e-2, atol=1e-2 * np.abs(sharded).max())
        assert np.abs(y - full).max() <= 2e-2 * np.abs(full).max()


@pytest.mark.parametrize("world", [1, 2, 4])
@pytest.mark.parametrize("mode", ["fused_silu", "fold"])
def test_tp_block_fused_layouts_match_oracle(world, mode, tmp_path):
    """The interleaved gate/up shard (fused silu) and the shard with the
    rms_norm weight folded into its rows: each rank's block, reduced over the
    group, matches the unsharded oracle block within the GEMM tolerance."""
    from oracle import ops

    procs = _launch(world, 1, tmp_path, mode=mode)
    assert all(p.exitcode == 0 for p in procs)
    x, nw, wgu, wd = _weights(mode)
    full = ops.mlp_block(x, nw, wgu, wd, 1e-6, "bfloat16")
    ys = [ops.round_to(np.load(tmp_path / f"y{r}.npy"), "bfloat16") for r in range(world)]
    for r in range(1, world):
        np.testing.assert_array_equal(ys[r], ys[0])
    assert np.abs(ys[0] - full).max() <= 2e-2 * np.abs(full).max()


def test_rank_failure_is_reported_not_hung(tmp_path):
    t0 = time.time()
    procs = _launch(2, 1, tmp_path, fail_rank=1, timeout=90.0)
    assert procs[1].exitcode == 3
    err = (tmp_path / "err0.txt")
    assert err.exists(), "surviving rank did not observe the failure"
    assert time.time() - t0 < 90.0
