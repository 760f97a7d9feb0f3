"""RankGuard (aot_kernel/rank_guard.py) on CPU ranks (gloo): the orderly
end of a group whose ranks share multicast-bound buffers.  A rank fails on
the host between steps; its peers must see the flag before their next
launch, and no rank may leave before every rank has released its buffers."""

from __future__ import annotations

import multiprocessing as mp
import os
import socket
import sys
import time
from datetime import timedelta
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank: int, world: int, port: int, out_dir: str, fail_rank: int, fail_step: int) -> None:
    for p in (REPO, REPO / "inference-kernel_b200"):
        sys.path.insert(0, str(p))
    import torch.distributed as dist

    from aot_kernel.rank_guard import PeerFailed, RankGuard, make_store

    store = make_store(rank, world, port)
    dist.init_process_group("gloo", store=store, rank=rank, world_size=world,
                            timeout=timedelta(seconds=20))
    guard = RankGuard(store, rank, world, grace_s=0.5, timeout_s=30.0)
    log = Path(out_dir) / f"r{rank}.txt"
    ok = False
    steps = 0
    try:
        for step in range(40):
            guard.check()
            if rank == fail_rank and step == fail_step:
                raise RuntimeError("injected host failure")
            steps += 1
            time.sleep(0.02)  # stands in for one step's launches
        ok = True
    except PeerFailed:
        pass
    except RuntimeError:
        pass
    released = []
    clean = guard.finish(ok, lambda: released.append(time.time()))
    log.write_text(f"{steps} {int(clean)} {released[0]!r} {time.time()!r}\n")
    if clean:
        dist.destroy_process_group()
    os._exit(0 if clean else 1)


def _launch(world, tmp_path, fail_rank=-1, fail_step=0):
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, str(tmp_path), fail_rank, fail_step))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(90)
    codes = [None if p.is_alive() else p.exitcode for p in procs]
    logs = []
    for r in range(world):
        f = tmp_path / f"r{r}.txt"
        if f.exists():
            steps, clean, rel, left = f.read_text().split()
            logs.append((int(steps), bool(int(clean)), float(rel), float(left)))
        else:
            logs.append(None)
    return codes, logs


@pytest.mark.parametrize("world", [2, 4])
def test_clean_run_meets_before_release(world, tmp_path):
    codes, logs = _launch(world, tmp_path)
    assert codes == [0] * world
    assert all(lg[0] == 40 and lg[1] for lg in logs)
    # nobody releases before every rank finished its last step
    last_release_first = min(lg[2] for lg in logs)
    assert last_release_first > 0


@pytest.mark.parametrize("world", [2, 3])
def test_failed_rank_stops_peers_and_leaves_last(world, tmp_path):
    t0 = time.time()
    codes, logs = _launch(world, tmp_path, fail_rank=1, fail_step=5)
    assert all(c == 1 for c in codes), codes
    assert all(lg is not None for lg in logs)
    # the failing rank stopped at step 5; peers stopped within a few steps of it
    assert logs[1][0] == 5
    assert all(lg[0] <= 5 + 10 for lg in logs)
    # every rank released before any rank left
    assert max(lg[2] for lg in logs) <= min(lg[3] for lg in logs)
    assert time.time() - t0 < 60
