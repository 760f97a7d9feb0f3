"""Orderly shutdown for the ranks of a group that share NVSwitch multicast memory.

The fused down-GEMM + all-reduce (``aotk_gemm_allreduce``) binds every rank's
``part`` / ``out`` buffers to one NVLink multicast object.  A rank whose
process ends while a peer still reads through that object can fault the
peer's GPU, so no rank may die (or be killed) with its buffers bound while
peers might still be running kernels on them.  The device side already ends
on its own: every wait in the fused kernel gives up after about a second and
records a watchdog bit.  This module is the host side:

* every rank checks, between steps, whether a peer has flagged a failure
  (``check``), through the group's key-value store - never through a
  collective, which would itself wait for the failed peer;
* a rank that fails flags it, waits for its own kernels (bounded), gives its
  peers a grace period to finish theirs and to notice the flag, releases its
  symmetric buffers, and only then leaves;
* on success every rank meets the others at a store barrier (all launches of
  all ranks done) before it releases anything.

NCCL is told to raise instead of tearing the process down on a timeout
(``nccl_env``), so a rank blocked in a collective whose peer is gone also
comes back through this path.
"""

from __future__ import annotations

import os
import time
from datetime import timedelta
from typing import Callable


def nccl_env(blocking: bool = True) -> None:
    """Makes a timed-out NCCL collective come back as an error instead of
    tearing the process down: with ``blocking`` every wait blocks the host
    and raises on the timeout; without it (for code that overlaps collectives
    with other streams) the timed-out communicator is aborted and later calls
    raise.  Call before the process group is created."""
    if blocking:
        os.environ.setdefault("TORCH_NCCL_BLOCKING_WAIT", "1")
        os.environ.setdefault("TORCH_NCCL_ASYNC_ERROR_HANDLING", "0")
    else:
        os.environ.setdefault("TORCH_NCCL_ASYNC_ERROR_HANDLING", "2")


class PeerFailed(RuntimeError):
    """A peer rank flagged a failure; this rank must not launch again."""


class RankGuard:
    def __init__(self, store, rank: int, world: int, prefix: str = "aotk_guard",
                 grace_s: float = 5.0, timeout_s: float = 120.0):
        self.store = store
        self.rank, self.world = rank, world
        self.failed_key = f"{prefix}/failed"
        self.done_key = f"{prefix}/done"
        self.released_key = f"{prefix}/released"
        self.grace_s, self.timeout_s = grace_s, timeout_s

    # ---- between steps
    def peer_failed(self) -> bool:
        return self.store.check([self.failed_key])

    def check(self) -> None:
        if self.peer_failed():
            raise PeerFailed(f"rank {self.store.get(self.failed_key).decode()} flagged a failure")

    def flag_failure(self) -> None:
        try:
            if not self.store.check([self.failed_key]):
                self.store.set(self.failed_key, str(self.rank))
        except Exception:  # noqa: BLE001  (store gone: peers time out on their own)
            pass

    # ---- end of the run
    def _count_to(self, key: str, deadline: float) -> bool:
        self.store.add(key, 1)
        while time.monotonic() < deadline:
            if self.store.add(key, 0) >= self.world:
                return True
            if key == self.done_key and self.peer_failed():
                return False
            time.sleep(0.005)
        return False

    def finish(self, ok: bool, release: Callable[[], None],
               sync: Callable[[], None] | None = None) -> bool:
        """Ends this rank's part of the run.  ``sync`` waits for this rank's
        kernels (all of which end on their own); ``release`` frees the shared
        buffers.  Returns True when every rank finished cleanly."""
        clean = False
        deadline = time.monotonic() + self.timeout_s
        if ok:
            try:
                if sync:
                    sync()
                clean = self._count_to(self.done_key, deadline)
            except Exception:  # noqa: BLE001
                clean = False
        if not clean:
            self.flag_failure()
            try:
                if sync:
                    sync()
            except Exception:  # noqa: BLE001  (a device error: nothing more runs here)
                pass
            # Peers' kernels give up their waits within about a second; the
            # grace period covers that and their next check between steps.
            time.sleep(self.grace_s)
        try:
            release()
        finally:
            try:
                # Leave only when every rank has released (or the bound runs
                # out), so that no launcher tears down a peer that still
                # holds bound buffers because this rank exited first.
                self._count_to(self.released_key, deadline + self.grace_s)
            except Exception:  # noqa: BLE001
                pass
        return clean


def make_store(rank: int, world: int, port: int, host: str = "127.0.0.1",
               timeout_s: float = 60.0):
    """A TCP store for the group; rank 0 serves it."""
    import torch.distributed as dist

    return dist.TCPStore(host, port, world, rank == 0, timeout=timedelta(seconds=timeout_s))
