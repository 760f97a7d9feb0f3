"""Multi-process GPU test harness: one spawned process per GPU rank.

The parent never ends a rank.  Ranks of the fused all-reduce hold buffers
bound to NVSwitch multicast objects, and a process that dies while a peer may
still read through them can fault the peer's GPU.  Each rank instead bounds
itself - every device wait in the kernels gives up after about a second, NCCL
raises on its process-group timeout (``rank_guard.nccl_env``), and the rank
leaves through ``RankGuard.finish`` (flag, wait, release, meet) - so the
parent only joins and reports.
"""

from __future__ import annotations

import gc
import multiprocessing as mp
import os
import socket
import sys
import time
import traceback
from datetime import timedelta
from pathlib import Path

REPO = Path(__file__).resolve().parents[1]


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_entry(body, rank: int, world: int, port: int, out_dir: str, args: tuple,
                nvls: bool) -> None:
    for p in (REPO, REPO / "inference-kernel_b200"):
        sys.path.insert(0, str(p))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    if not nvls:
        os.environ["NCCL_NVLS_ENABLE"] = "0"
    from aot_kernel.rank_guard import RankGuard, make_store, nccl_env

    nccl_env()
    import torch
    import torch.distributed as dist

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    store = make_store(rank, world, port)
    dist.init_process_group("nccl", store=store, rank=rank, world_size=world,
                            timeout=timedelta(seconds=60), device_id=dev)
    guard = RankGuard(store, rank, world)
    held: dict = {}
    ok = False
    try:
        body(rank, world, dev, out_dir, guard, held, *args)
        ok = True
    except BaseException:  # noqa: BLE001  (reported through the exit code and stderr)
        traceback.print_exc()

    def release():
        held.clear()
        gc.collect()
        torch.cuda.synchronize()

    clean = guard.finish(ok, release, sync=torch.cuda.synchronize)
    if clean:
        dist.destroy_process_group()
    sys.stdout.flush()
    sys.stderr.flush()
    os._exit(0 if clean else 1)


def run_ranks(body, world: int, out_dir, args: tuple = (), nvls: bool = True,
              deadline_s: float = 600.0) -> list[int | None]:
    """Runs ``body(rank, world, device, out_dir, guard, held, *args)`` on
    ``world`` spawned ranks and returns their exit codes (None for a rank
    still running at the deadline, which is left to end on its own)."""
    ctx = mp.get_context("spawn")
    port = free_port()
    procs = [ctx.Process(target=_rank_entry, args=(body, r, world, port, str(out_dir), args, nvls))
             for r in range(world)]
    for p in procs:
        p.start()
    end = time.time() + deadline_s
    for p in procs:
        p.join(max(1.0, end - time.time()))
    return [None if p.is_alive() else p.exitcode for p in procs]
