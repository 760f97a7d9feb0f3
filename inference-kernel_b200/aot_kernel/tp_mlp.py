"""Tensor-parallel Llama MLP block on the aot_kernel ops.

    y = down( silu(x_n @ W_gate) * (x_n @ W_up) ),   x_n = rms_norm(x, w_norm)

Megatron layout over a process group of W ranks (one process per GPU):
rank r owns the gate and up columns [r*I/W, (r+1)*I/W) - stored side by side
as one [H, 2*I/W] matrix so the two projections are a single GEMM - and the
same rows of W_down ([I/W, H]).  rms_norm and silu_mul are local; the only
exchange is one all-reduce (sum) of the [T, H] partial outputs over NCCL.
With ``chunks > 1`` the token dimension is cut into slices whose all-reduce
(asynchronous, on NCCL's stream) overlaps the down projection of the next
slice.

The reference has no multi-GPU code; its oracle for this block is the
unsharded composition of ref.rmsnorm, ref.gemm and ref.silu.
"""

from __future__ import annotations

from dataclasses import dataclass
from types import SimpleNamespace

import torch
import torch.distributed as dist


def default_ops() -> SimpleNamespace:
    from . import gemm, rms_norm, silu_mul

    return SimpleNamespace(rms_norm=rms_norm, gemm=gemm, silu_mul=silu_mul)


def shard_gate_up(w_gate_up: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """[H, 2I] = [W_gate | W_up]  ->  rank's [H, 2I/W] = [W_gate[:, s] | W_up[:, s]]."""
    inter = w_gate_up.shape[1] // 2
    if inter % world:
        raise ValueError(f"intermediate size {inter} does not split over {world} ranks")
    s = inter // world
    gate = w_gate_up[:, rank * s:(rank + 1) * s]
    up = w_gate_up[:, inter + rank * s: inter + (rank + 1) * s]
    return torch.cat([gate, up], dim=1).contiguous()


def shard_down(w_down: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """[I, H] -> rank's rows [r*I/W, (r+1)*I/W)."""
    inter = w_down.shape[0]
    if inter % world:
        raise ValueError(f"intermediate size {inter} does not split over {world} ranks")
    s = inter // world
    return w_down[rank * s:(rank + 1) * s].contiguous()


@dataclass
class MLPShard:
    norm_weight: torch.Tensor  # [H]
    w_gate_up: torch.Tensor    # [H, 2*I/W]
    w_down: torch.Tensor       # [I/W, H]


class TensorParallelMLP:
    def __init__(self, shard: MLPShard, group=None, eps: float = 1e-6, chunks: int = 1,
                 ops: SimpleNamespace | None = None):
        self.shard = shard
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.eps = eps
        self.chunks = max(1, chunks)
        self.ops = ops or default_ops()
        self.inter_local = shard.w_down.shape[0]
        if shard.w_gate_up.shape[1] != 2 * self.inter_local:
            raise ValueError("gate/up shard must be [H, 2 * I_local]")

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        ops, s = self.ops, self.shard
        h = ops.rms_norm(x, s.norm_weight, self.eps)
        gu = ops.gemm(h, s.w_gate_up)
        act = ops.silu_mul(gu[:, :self.inter_local], gu[:, self.inter_local:])
        if self.world == 1:
            return ops.gemm(act, s.w_down)
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
