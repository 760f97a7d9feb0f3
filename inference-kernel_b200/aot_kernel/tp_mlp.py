"""Tensor-parallel Llama MLP block on the aot_kernel ops.

    y = down( silu(x_n @ W_gate) * (x_n @ W_up) ),   x_n = rms_norm(x, w_norm)

Megatron layout over a process group of W ranks (one process per GPU):
rank r owns the gate and up columns [r*I/W, (r+1)*I/W) - stored side by side
as one [H, 2*I/W] matrix so the two projections are a single GEMM - and the
same rows of W_down ([I/W, H]).  rms_norm and silu_mul are local; the only
exchange is one all-reduce (sum) of the [T, H] partial outputs over NCCL.
With ``chunks > 1`` the token dimension is cut into slices whose all-reduce
(asynchronous, on NCCL's stream) overlaps the down projection of the next
slice.  With ``allreduce="fused"`` the down projection and the all-reduce are
one kernel (``aotk_gemm_allreduce``): partial tiles are summed through
NVSwitch multicast memory while the rest of the GEMM runs.  A shard built
with ``fused_silu=True`` (``shard_gate_up_interleaved``) runs the gate/up
projection and silu(gate) * up as one kernel (``gemm_silu_mul``); one built
with ``fold_norm=True`` (``shard_gate_up_folded``) also takes rms_norm into
that kernel: the norm weight is folded into the rows of the gate/up weight
once, and each step only computes the row statistic rstd (``rms_rstd``), which
the GEMM epilogue applies - the normalised activations are never written.

The reference has no multi-GPU code; its oracle for this block is the
unsharded composition of ref.rmsnorm, ref.gemm and ref.silu.
"""

from __future__ import annotations

from dataclasses import dataclass
from types import SimpleNamespace

import torch
import torch.distributed as dist


def default_ops() -> SimpleNamespace:
    from . import gemm, gemm_silu_mul, rms_norm, rms_rstd, silu_mul

    return SimpleNamespace(rms_norm=rms_norm, gemm=gemm, silu_mul=silu_mul,
                           gemm_silu_mul=gemm_silu_mul, rms_rstd=rms_rstd)


def shard_gate_up(w_gate_up: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """[H, 2I] = [W_gate | W_up]  ->  rank's [H, 2I/W] = [W_gate[:, s] | W_up[:, s]]."""
    inter = w_gate_up.shape[1] // 2
    if inter % world:
        raise ValueError(f"intermediate size {inter} does not split over {world} ranks")
    s = inter // world
    gate = w_gate_up[:, rank * s:(rank + 1) * s]
    up = w_gate_up[:, inter + rank * s: inter + (rank + 1) * s]
    return torch.cat([gate, up], dim=1).contiguous()


def shard_gate_up_interleaved(w_gate_up: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """Rank's gate/up shard in the interleaved layout of ``gemm_silu_mul``."""
    from .gemm import interleave_gate_up

    shard = shard_gate_up(w_gate_up, rank, world)
    s = shard.shape[1] // 2
    return interleave_gate_up(shard[:, :s], shard[:, s:])


def shard_gate_up_folded(w_gate_up: torch.Tensor, norm_weight: torch.Tensor, rank: int,
                         world: int) -> torch.Tensor:
    """``shard_gate_up_interleaved`` with the rms_norm weight folded into its
    rows (``fold_norm_weight``), for ``MLPShard(..., fold_norm=True)``."""
    from .gemm import fold_norm_weight

    return fold_norm_weight(shard_gate_up_interleaved(w_gate_up, rank, world), norm_weight)


def shard_down(w_down: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """[I, H] -> rank's rows [r*I/W, (r+1)*I/W)."""
    inter = w_down.shape[0]
    if inter % world:
        raise ValueError(f"intermediate size {inter} does not split over {world} ranks")
    s = inter // world
    return w_down[rank * s:(rank + 1) * s].contiguous()


class FusedDownAllReduce:
    """Symmetric buffers and call state of ``aotk_gemm_allreduce`` for one
    [tokens, hidden] output on one process group.

    ``part`` and ``out`` are allocated with torch's symmetric memory and bound
    to NVSwitch multicast objects; the arrival counters and the done word live
    in one zero-initialised symmetric int32 buffer.  The returned output is
    ``out`` itself and is overwritten by the next call.
    """

    def __init__(self, tokens: int, hidden: int, dtype, device, group=None):
        import torch.distributed._symmetric_memory as symm_mem

        from . import capi

        self.capi = capi
        self.group = group or dist.group.WORLD
        self.rank = dist.get_rank(self.group)
        self.world = dist.get_world_size(self.group)
        self.M, self.N = tokens, hidden
        self.dtype = dtype
        self.tiles = capi.gemm_allreduce_tiles(tokens, hidden)
        self.part = symm_mem.empty((tokens, hidden), dtype=dtype, device=device)
        self.out = symm_mem.empty((tokens, hidden), dtype=dtype, device=device)
        self.sig = symm_mem.empty((self.tiles + 64,), dtype=torch.int32, device=device)
        self.sig.zero_()
        torch.cuda.synchronize(device)
        hp = symm_mem.rendezvous(self.part, self.group)
        ho = symm_mem.rendezvous(self.out, self.group)
        hs = symm_mem.rendezvous(self.sig, self.group)
        if not hp.multicast_ptr or not ho.multicast_ptr:
            raise RuntimeError("NVSwitch multicast (NVLS) is not available on this group")
        self._handles = (hp, ho, hs)
        done_off = self.tiles * 4
        self.peer_counters = torch.tensor(list(hs.buffer_ptrs), dtype=torch.int64, device=device)
        self.peer_done = torch.tensor([p + done_off for p in hs.buffer_ptrs], dtype=torch.int64,
                                      device=device)
        self.epoch = 0
        self.bufs = capi.AllReduceBuffers(
            rank=self.rank, world=self.world, part=self.part.data_ptr(),
            part_multicast=hp.multicast_ptr, out_multicast=ho.multicast_ptr,
            counters=self.sig.data_ptr(), peer_counters=self.peer_counters.data_ptr(),
            done=self.sig.data_ptr() + done_off, peer_done=self.peer_done.data_ptr(), epoch=0)
        dist.barrier(self.group)  # every rank's counters are zero before the first call

    def __call__(self, act: torch.Tensor, w_down: torch.Tensor) -> torch.Tensor:
        if act.shape[0] != self.M or w_down.shape[1] != self.N or act.dtype != self.dtype:
            raise ValueError("shape/dtype differs from the one the buffers were built for")
        self.epoch += 1
        self.bufs.epoch = self.epoch
        self.capi.gemm_allreduce(act, w_down, self.M, self.N, act.shape[1],
                                 self.capi.dtype_code(act.dtype), self.bufs)
        return self.out


@dataclass
class MLPShard:
    norm_weight: torch.Tensor  # [H]
    w_gate_up: torch.Tensor    # [H, 2*I/W]; interleaved in 128-column blocks when fused_silu
    w_down: torch.Tensor       # [I/W, H]
    fused_silu: bool = False   # w_gate_up is in the gemm_silu_mul layout
    fold_norm: bool = False    # w_gate_up also carries norm_weight in its rows (needs fused_silu)


class TensorParallelMLP:
    def __init__(self, shard: MLPShard, group=None, eps: float = 1e-6, chunks: int = 1,
                 ops: SimpleNamespace | None = None, allreduce: str = "nccl"):
        self.shard = shard
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.eps = eps
        self.chunks = max(1, chunks)
        self.ops = ops or default_ops()
        self.inter_local = shard.w_down.shape[0]
        if shard.w_gate_up.shape[1] != 2 * self.inter_local:
            raise ValueError("gate/up shard must be [H, 2 * I_local]")
        if allreduce not in ("nccl", "fused"):
            raise ValueError(f"allreduce must be 'nccl' or 'fused', got {allreduce!r}")
        self.allreduce = allreduce
        if shard.fold_norm and not shard.fused_silu:
            raise ValueError("fold_norm needs the fused gate/up + silu layout (fused_silu=True)")
        self._fused: FusedDownAllReduce | None = None

    def gate_up_act(self, x: torch.Tensor, gate_up_events=None) -> torch.Tensor:
        """rms_norm, gate/up projection and silu(gate) * up of one step.
        ``gate_up_events`` (a pair of CUDA events) is recorded on the current
        stream around the gate/up GEMM launch, for timing that kernel alone."""
        ops, s = self.ops, self.shard
        ev = gate_up_events or ()

        def mark(i):
            if ev:
                ev[i].record()

        if s.fold_norm:
            rstd = ops.rms_rstd(x, self.eps)
            mark(0)
            act = ops.gemm_silu_mul(x, s.w_gate_up, rstd)
            mark(1)
            return act
        h = ops.rms_norm(x, s.norm_weight, self.eps)
        mark(0)
        if s.fused_silu:
            act = ops.gemm_silu_mul(h, s.w_gate_up)
            mark(1)
            return act
        gu = ops.gemm(h, s.w_gate_up)
        mark(1)
        return ops.silu_mul(gu[:, :self.inter_local], gu[:, self.inter_local:])

    def launches_per_step(self) -> int:
        """Kernels one ``forward`` launches (NCCL's all-reduce kernels not counted)."""
        s = self.shard
        n = 2 if s.fused_silu else 3          # rms_norm / rms_rstd, gate/up (+ silu_mul)
        return n + (self.chunks if self.world > 1 and self.allreduce == "nccl" else 1)

    def forward(self, x: torch.Tensor, gate_up_events=None) -> torch.Tensor:
        ops, s = self.ops, self.shard
        act = self.gate_up_act(x, gate_up_events)
        if self.world == 1:
            return ops.gemm(act, s.w_down)
        if self.allreduce == "fused":
            if self._fused is None or self._fused.M != act.shape[0]:
                self._fused = FusedDownAllReduce(act.shape[0], s.w_down.shape[1], act.dtype,
                                                 act.device, self.group)
            return self._fused(act, s.w_down)
        if self.chunks == 1:
            out = ops.gemm(act, s.w_down)
            dist.all_reduce(out, op=dist.ReduceOp.SUM, group=self.group)
            return out
        tokens = act.shape[0]
        out = torch.empty((tokens, s.w_down.shape[1]), dtype=act.dtype, device=act.device)
        bounds = [tokens * i // self.chunks for i in range(self.chunks + 1)]
        works = []
        for lo, hi in zip(bounds[:-1], bounds[1:]):
            if hi == lo:
                continue
            ops.gemm(act[lo:hi], s.w_down, out=out[lo:hi])
            works.append(dist.all_reduce(out[lo:hi], op=dist.ReduceOp.SUM, group=self.group,
                                         async_op=True))
        for w in works:
            w.wait()
        return out

    __call__ = forward


class HostStream:
    """Runs a ``TensorParallelMLP`` on batches that live in pinned HOST memory,
    the way a serving loop feeds it: ``submit(x_host, out_host)`` enqueues one
    batch and returns; batch i+1's copy-in and batch i-1's copy-out run on
    their own streams while batch i's kernels run.

    Over W ranks the host link carries every input row once: rank r copies
    rows [r*T/W, (r+1)*T/W) of ``x_host`` in, the ranks all-gather x over
    NVLink (NCCL, on the block's stream), the block runs, and rank r copies the
    same rows of the (all-reduced, replicated) output back into ``out_host``,
    so the W ranks' host buffers together hold the whole result.  Two device
    slots per rank; a slot is reused only after the batch that used it has
    been read back.
    """

    def __init__(self, block: TensorParallelMLP, tokens: int, hidden: int, device,
                 dtype=torch.bfloat16, group=None, slots: int = 2):
        self.block, self.group = block, group
        self.world = block.world
        self.rank = dist.get_rank(group) if self.world > 1 else 0
        if tokens % self.world:
            raise ValueError(f"{tokens} tokens do not split over {self.world} ranks")
        rows = tokens // self.world
        self.lo, self.hi = self.rank * rows, (self.rank + 1) * rows
        self.shape = (tokens, hidden)
        self.slots = slots
        self.x = [torch.empty((tokens, hidden), dtype=dtype, device=device) for _ in range(slots)]
        self.xin = [self.x[i][self.lo:self.hi] if self.world == 1 else
                    torch.empty((rows, hidden), dtype=dtype, device=device) for i in range(slots)]
        self.stage = [torch.empty((rows, hidden), dtype=dtype, device=device) for _ in range(slots)]
        self.h2d = torch.cuda.Stream(device)
        self.d2h = torch.cuda.Stream(device)
        self.x_free = [torch.cuda.Event() for _ in range(slots)]
        self.stage_free = [torch.cuda.Event() for _ in range(slots)]
        self.n = 0

    def h2d_bytes(self) -> int:
        return self.xin[0].nbytes

    def d2h_bytes(self) -> int:
        return self.stage[0].nbytes

    def submit(self, x_host: torch.Tensor, out_host: torch.Tensor) -> None:
        if tuple(x_host.shape) != self.shape or tuple(out_host.shape) != self.shape:
            raise ValueError(f"host batches must be {list(self.shape)}")
        if x_host.device.type != "cpu" or out_host.device.type != "cpu":
            raise ValueError("submit takes host tensors (pinned for asynchronous copies)")
        s = self.n % self.slots
        cur = torch.cuda.current_stream()
        with torch.cuda.stream(self.h2d):
            if self.n >= self.slots:
                self.h2d.wait_event(self.x_free[s])
            self.xin[s].copy_(x_host[self.lo:self.hi], non_blocking=True)
            landed = torch.cuda.Event()
            landed.record(self.h2d)
        cur.wait_event(landed)
        if self.world > 1:
            # On the block's own stream, never beside it: the fused down
            # GEMM + all-reduce needs all its CTAs resident at once, and an
            # NCCL kernel that held SMs while waiting for a peer (whose own
            # fused kernel waits for this rank) would deadlock the two.
            dist.all_gather_into_tensor(self.x[s], self.xin[s], group=self.group)
        y = self.block(self.x[s])
        self.x_free[s].record(cur)
        if self.n >= self.slots:
            cur.wait_event(self.stage_free[s])
        self.stage[s].copy_(y[self.lo:self.hi])
        staged = torch.cuda.Event()
        staged.record(cur)
        with torch.cuda.stream(self.d2h):
            self.d2h.wait_event(staged)
            out_host[self.lo:self.hi].copy_(self.stage[s], non_blocking=True)
            self.stage_free[s].record(self.d2h)
        self.n += 1

    def drain(self) -> None:
        """Makes the current stream wait for every submitted batch's copy-out."""
        torch.cuda.current_stream().wait_stream(self.d2h)
