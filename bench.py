#!/usr/bin/env python
"""Benchmark of the dense-linear inference path on B200.

Headline (one JSON line on rank 0): tokens/s of the Llama-3-70B MLP block -
x[4096 tokens, 8192] -> rms_norm -> gate/up GEMM 8192 -> 2 x 28672 ->
silu(gate) * up -> down GEMM 28672 -> 8192 -> all-reduce - tensor-parallel
over the N ranks of one node (N = 1, 2, 4, 8; strong scaling: the same 4096
tokens per step at every N).  A step is one pass of the block over inputs
already resident in HBM; ``value`` is 4096 * steps / (max over ranks of the
CUDA-event time of the timed steps).  Per rank the block is three kernels:
rms_rstd (rms_norm's row statistic), the gate/up GEMM with rms_norm folded in
and silu(gate) * up in its epilogue, and the down GEMM fused with an NVSwitch
all-reduce (N > 1) or the plain down GEMM (N = 1).  The line also carries:

* ``roofline``  - the gate/up GEMM (the dominant kernel, 2/3 of the flops):
  2 * T * H * 2I / N flops per launch / its mean CUDA-event duration in the
  timed steps, against the measured sustained bf16 GEMM peak (the block runs
  back to back at the power cap; the burst fraction is given beside it);
* ``e2e``       - the same tokens/s through ``aot_kernel.tp_mlp.HostStream``
  with pinned HOST batches: every step copies its input rows in, runs the
  block, and copies its output rows back, inside the timed region;
* ``tp_parity`` - sampled rows of the block's output against the reference
  composition (ref.rmsnorm -> ref.gemm -> ref.silu(gate) * up -> ref.gemm)
  run on CPU by torch, max|err| <= 2e-2 * max|ref|;
* ``cpu_baseline`` - that reference composition timed on the host's cores on
  the full 4096-token block (rank 0, N = 1);
* ``kernels`` (N = 1) - every other configured workload with its roofline
  fraction: the square GEMM sweep, the Llama-3-8B linears from decode to
  prefill, rms_norm, silu, silu(gate) * up, 8-bit GEMMs, and ``gemm_8192``.

``--impl reference`` times that reference composition on the host's cores on
the same block and metric instead; under torchrun only rank 0 runs it.

``--case NAME`` runs only NAME's launches (warmup + steps) and prints nothing
else: the command the committed ncu summaries under profiles/ were made with.
"""

from __future__ import annotations

import argparse
import gc
import json
import os
import statistics
import sys
import time
import traceback
from datetime import timedelta
from pathlib import Path

REPO = Path(__file__).resolve().parent
for _p in (REPO, REPO / "inference-kernel_b200"):
    if str(_p) not in sys.path:
        sys.path.insert(0, str(_p))

FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
L2_BYTES = 126 * 1024 * 1024
TOKENS, HIDDEN, INTER = 4096, 8192, 28672
EPS = 1e-6
BLOCK_FLOPS = 2.0 * TOKENS * HIDDEN * 2 * INTER + 2.0 * TOKENS * INTER * HIDDEN
PARITY_ROWS = 32
PARITY_TOL = 2e-2

# --case workloads: name -> (kind, shape)
CASES = {
    "gemm_8192": ("gemm", (8192, 8192, 8192)),
    "gemm_4096": ("gemm", (4096, 4096, 4096)),
    "gemm_tc2_8192": ("gemm_tc2", (8192, 8192, 8192)),
    "cublas_8192": ("cublas", (8192, 8192, 8192)),  # torch.matmul, for comparison
    "gemm_decode_m1": ("gemm", (1, 4096, 28672)),
    "gemm_decode_m16": ("gemm", (16, 4096, 28672)),
    "gemm_qkv_m1": ("gemm", (1, 4096, 6144)),
    "gemm_qkv_m128": ("gemm", (128, 4096, 6144)),
    "gemm_m128_down": ("gemm", (128, 14336, 4096)),
    "gate_up_silu_2048": ("gate_up_silu", (2048, 4096, 14336)),
    "tp_gate_up_tp1": ("tp_gate_up", (TOKENS, HIDDEN, INTER)),
    "tp_gate_up_tp2": ("tp_gate_up", (TOKENS, HIDDEN, INTER // 2)),
    "tp_gate_up_tp4": ("tp_gate_up", (TOKENS, HIDDEN, INTER // 4)),
    "tp_gate_up_tp8": ("tp_gate_up", (TOKENS, HIDDEN, INTER // 8)),
    "tp_down_tp1": ("gemm", (TOKENS, INTER, HIDDEN)),
    "scaled_gemm_fp8_8192": ("scaled_gemm_e4m3", (8192, 8192, 8192)),
    "scaled_gemm_fp8_4096": ("scaled_gemm_e4m3", (4096, 4096, 4096)),
    "scaled_gemm_int8_4096": ("scaled_gemm_int8", (4096, 4096, 4096)),
    "rms_norm": ("rms_norm", (8192, 4096)),
    "rms_rstd": ("rms_rstd", (8192, 4096)),
    "rms_rstd_tp": ("rms_rstd", (TOKENS, HIDDEN)),
    "add_rms_norm": ("add_rms_norm", (8192, 4096)),
    "silu": ("silu", (8192, 14336)),
    "silu_mul": ("silu_mul", (8192, 14336)),
}


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=int(os.environ.get("WORLD_SIZE", "1")))
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-kernels", action="store_true", help="skip the per-workload table")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline")
    ap.add_argument("--tp-chunks", type=int, default=1)
    ap.add_argument("--tp-allreduce", choices=["nccl", "fused"], default="fused",
                    help="down projection + all-reduce: NCCL after the GEMM, or one fused kernel")
    ap.add_argument("--tp-unfused-silu", action="store_true",
                    help="gate/up GEMM then silu_mul, instead of the fused gate/up + silu kernel")
    ap.add_argument("--tp-unfolded-norm", action="store_true",
                    help="run rms_norm as its own kernel instead of folding it into the fused "
                         "gate/up kernel (norm weight in the weight rows, rstd in the epilogue)")
    ap.add_argument("--case", choices=sorted(CASES), default=None,
                    help="run only this workload's launches (for profilers)")
    return ap.parse_args()


def load_peaks() -> tuple[dict, str]:
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            d = json.loads(p.read_text())
            return {k: float(d[k]) for k in FALLBACK_PEAKS}, "measured"
        except (KeyError, ValueError):
            pass
    return dict(FALLBACK_PEAKS), "fallback"


# ---------------------------------------------------------------- clocks

# The sampling loop runs in a child process: NVML queries take milliseconds
# and, in the process that launches the kernels, stall its launches; with the
# ranks of a tensor-parallel step coupled through the all-reduce, a stall on
# any rank idles all of them.
_SAMPLER_CHILD = r"""
import sys, time, pynvml
pynvml.nvmlInit()
h = pynvml.nvmlDeviceGetHandleByPciBusId(sys.argv[1].encode())
period = float(sys.argv[2])
while True:
    try:
        sm = pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)
        pw = pynvml.nvmlDeviceGetPowerUsage(h) / 1000.0
        rs = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
        print(f"{sm},{pw},{rs}", flush=True)
    except pynvml.NVMLError:
        pass
    time.sleep(period)
"""


class ClockSampler:
    """Samples this rank's GPU clock, power and clock-event reasons through NVML
    (read-only queries) every 10 ms while the timed region runs, from a child
    process (``_SAMPLER_CHILD``)."""

    REASONS = {"hw_slowdown": "nvmlClocksEventReasonHwSlowdown",
               "hw_thermal_slowdown": "nvmlClocksEventReasonHwThermalSlowdown",
               "sw_thermal_slowdown": "nvmlClocksEventReasonSwThermalSlowdown",
               "sw_power_cap": "nvmlClocksEventReasonSwPowerCap",
               "hw_power_brake": "nvmlClocksEventReasonHwPowerBrakeSlowdown"}

    def __init__(self, device: int = 0, period_s: float = 0.01):
        self.device, self.period = device, period_s
        self.samples: list[tuple[float, float, int]] = []
        self.max_mhz = None
        self._proc = None
        self._nvml = None
        self._bus_id = None

    def _handle(self):
        import pynvml
        import torch

        pynvml.nvmlInit()
        p = torch.cuda.get_device_properties(self.device)
        # torch reports the PCI location as integers; NVML wants "DDDDDDDD:BB:DD.0".
        self._bus_id = (f"{int(p.pci_domain_id):08X}:{int(p.pci_bus_id):02X}:"
                        f"{int(p.pci_device_id):02X}.0")
        return pynvml.nvmlDeviceGetHandleByPciBusId(self._bus_id.encode())

    def __enter__(self):
        import subprocess

        try:
            import pynvml

            self._nvml = pynvml
            h = self._handle()
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))
            self._proc = subprocess.Popen(
                [sys.executable, "-c", _SAMPLER_CHILD, self._bus_id, str(self.period)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            # Sampling has begun once the child's first line arrives.
            import select

            if select.select([self._proc.stdout], [], [], 10.0)[0]:
                self._keep(self._proc.stdout.readline())
        except Exception:  # noqa: BLE001
            self._nvml = None
        return self

    def _keep(self, line: str) -> None:
        try:
            sm, pw, rs = line.split(",")
            self.samples.append((float(sm), float(pw), int(rs)))
        except ValueError:
            pass

    def __exit__(self, *exc):
        if self._proc is not None:
            self._proc.terminate()  # this sampler's own child, by its PID
            try:
                out, _ = self._proc.communicate(timeout=10)
            except Exception:  # noqa: BLE001
                self._proc.kill()
                out, _ = self._proc.communicate()
            for line in (out or "").splitlines():
                self._keep(line)
        return False

    def nvlink_kib(self):
        """This GPU's NVLink data counters (TX, RX; KiB, summed over its
        links) through NVML field values, or None where NVML does not
        report them."""
        if self._nvml is None:
            return None
        nv = self._nvml
        try:
            h = self._handle()
            tx = rx = 0
            for link in range(18):
                vals = nv.nvmlDeviceGetFieldValues(h, [
                    (nv.NVML_FI_DEV_NVLINK_THROUGHPUT_DATA_TX, link),
                    (nv.NVML_FI_DEV_NVLINK_THROUGHPUT_DATA_RX, link)])
                if vals[0].nvmlReturn or vals[1].nvmlReturn:
                    continue
                tx += int(vals[0].value.ullVal)
                rx += int(vals[1].value.ullVal)
            return tx, rx
        except Exception:  # noqa: BLE001
            return None

    def summary(self) -> dict:
        if self._nvml is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvml unavailable"]}
        loaded = [s for s in self.samples if s[1] > 250.0] or self.samples
        reasons = set()
        for _, _, bits in loaded:
            for name, const in self.REASONS.items():
                if bits & int(getattr(self._nvml, const, 0)):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(s[0] for s in loaded) if loaded else None,
                "sm_max_mhz": self.max_mhz, "reasons": sorted(reasons),
                "samples": len(self.samples), "samples_under_load": len(loaded),
                "power_w_max": max((s[1] for s in self.samples), default=None)}


# ---------------------------------------------------------------- workloads

def rand_bf16(shape, seed: int, std: float = 1.0, mean: float = 0.0):
    import torch

    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    x = torch.randn(shape, generator=g, device="cuda", dtype=torch.float32)
    if std != 1.0:
        x.mul_(std)
    if mean != 0.0:
        x.add_(mean)
    return x.to(torch.bfloat16)


def rand_q(shape, seed: int, qdtype: str):
    """8-bit GEMM operands drawn as the reference's scaled-GEMM benchmark draws
    them: N(0, 1) converted to float8_e4m3fn, or integers in [-8, 8)."""
    import torch

    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    if qdtype == "int8":
        return torch.randint(-8, 8, shape, generator=g, device="cuda", dtype=torch.int8)
    return torch.randn(shape, generator=g, device="cuda").to(torch.float8_e4m3fn)


def row_scales(M: int, N: int, seed: int):
    import torch

    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    sa = torch.rand(M, generator=g, device="cuda") * 0.1 + 0.01
    sb = torch.rand(N, generator=g, device="cuda") * 0.1 + 0.01
    return sa, sb


# ---------------------------------------------------------------- the block on the GPU

def tp_build(args, rank: int, world: int):
    """The block's inputs drawn on the device (seeded Philox), sharded for this
    rank.  Rank 0 keeps host copies of x, the norm weight and the full
    weights for the parity check and the CPU baseline."""
    import torch

    from aot_kernel.tp_mlp import (MLPShard, TensorParallelMLP, shard_down, shard_gate_up,
                                   shard_gate_up_folded, shard_gate_up_interleaved)

    x = rand_bf16((TOKENS, HIDDEN), 30)
    nw = rand_bf16((HIDDEN,), 31, std=0.1, mean=1.0)
    w_gu = rand_bf16((HIDDEN, 2 * INTER), 32, std=0.02)
    host = {}
    if rank == 0:
        host.update(x=x.cpu(), nw=nw.cpu(), wgu=w_gu.cpu())
    fused_silu = not args.tp_unfused_silu
    fold_norm = fused_silu and not args.tp_unfolded_norm
    if fold_norm:
        wgu_r = shard_gate_up_folded(w_gu, nw, rank, world)
    else:
        wgu_r = (shard_gate_up_interleaved if fused_silu else shard_gate_up)(w_gu, rank, world)
    del w_gu
    w_d = rand_bf16((INTER, HIDDEN), 33, std=0.02)
    if rank == 0:
        host["wd"] = w_d.cpu()
    wd_r = shard_down(w_d, rank, world)
    del w_d
    torch.cuda.empty_cache()
    allreduce = args.tp_allreduce if world > 1 else "nccl"
    block = TensorParallelMLP(MLPShard(nw, wgu_r, wd_r, fused_silu=fused_silu, fold_norm=fold_norm),
                              eps=EPS, chunks=args.tp_chunks, allreduce=allreduce)
    return x, block, host


def _max_over_ranks(vals: list[float], world: int) -> list[float]:
    import torch
    import torch.distributed as dist

    t = torch.tensor(vals, device="cuda", dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


def _meet(world: int) -> None:
    import torch
    import torch.distributed as dist

    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()


def tp_timed(args, block, x, world: int, peaks: dict, guard) -> dict:
    """Exactly ``args.steps`` block steps between two events, after
    ``args.warmup`` untimed ones.  Inside every timed step, events before the
    block, around its gate/up GEMM launch and after it split the step into
    rms_rstd | gate/up GEMM | down GEMM (+ all-reduce)."""
    import torch

    for _ in range(args.warmup):
        block(x)

    def ev():
        return torch.cuda.Event(enable_timing=True)

    # The sampler starts (NVML set-up can take a second) before the ranks
    # meet, so that every rank enters the timed steps at the same moment.
    with ClockSampler(torch.cuda.current_device()) as clocks:
        evs = [(ev(), ev(), ev(), ev()) for _ in range(args.steps)]
        nv0 = clocks.nvlink_kib() if world > 1 else None
        _meet(world)
        guard.check()
        t0, t1 = ev(), ev()
        t0.record()
        for a, b, c, d in evs:
            a.record()
            block(x, gate_up_events=(b, c))
            d.record()
        t1.record()
        torch.cuda.synchronize()
        nv1 = clocks.nvlink_kib() if nv0 is not None else None
    total_ms = t0.elapsed_time(t1)
    down_alone = down_gemm_alone_ms(block, x) if world > 1 else -1.0
    ar_alone = nccl_allreduce_ms(world) if world > 1 else -1.0
    pre = statistics.mean(a.elapsed_time(b) for a, b, _, _ in evs)
    gu_ms = statistics.mean(b.elapsed_time(c) for _, b, c, _ in evs)
    post = statistics.mean(c.elapsed_time(d) for _, _, c, d in evs)
    total_ms, pre, gu_ms, post, down_alone, ar_alone = _max_over_ranks(
        [total_ms, pre, gu_ms, post, down_alone, ar_alone], world)
    s = block.shard
    first = "rms_rstd" if s.fold_norm else "rms_norm"
    mid = "gate_up+norm+silu" if s.fold_norm else ("gate_up+silu" if s.fused_silu else "gate_up")
    last = ("" if s.fused_silu else "silu_mul+") + ("down" if world == 1 else "down+all_reduce")
    gu_flops = 2.0 * TOKENS * HIDDEN * 2 * INTER / world
    achieved = gu_flops / (gu_ms * 1e-3) / 1e12
    return {"ms_per_step": total_ms / args.steps,
            "value": TOKENS * args.steps / (total_ms * 1e-3),
            "phases_ms": {first: round(pre, 4), mid: round(gu_ms, 4), last: round(post, 4),
                          **({"down_gemm_alone": round(down_alone, 4),
                              "nccl_all_reduce_alone": round(ar_alone, 4)} if world > 1 else {})},
            "roofline": {"bound": "tensor", "achieved": round(achieved, 1),
                         "peak": peaks["bf16_tflops_sustained"], "unit": "TFLOP/s",
                         "frac": round(achieved / peaks["bf16_tflops_sustained"], 4),
                         "frac_of_burst_peak": round(achieved / peaks["bf16_tflops"], 4),
                         "traffic": traffic_per_launch(f"tp_gate_up_tp{world}"),
                         "kernel": f"gemm_silu_mul + folded rms_norm, M={TOKENS} K={HIDDEN} "
                                   f"N={2 * INTER // world}"},
            "gpu_launches": block.launches_per_step() * args.steps,
            "clocks": clocks.summary(),
            "nvlink": nvlink_per_step(nv0, nv1, args.steps, world)}


def down_gemm_alone_ms(block, x, reps: int = 10) -> float:
    """This rank's down projection without the all-reduce (the plain GEMM on
    the same shard and activations), mean CUDA-event time: what the fused
    down GEMM + all-reduce would take if the exchange were free."""
    import torch

    act = block.gate_up_act(x)
    w = block.shard.w_down
    for _ in range(2):
        block.ops.gemm(act, w)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(reps):
        block.ops.gemm(act, w)
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / reps


def nccl_allreduce_ms(world: int, reps: int = 10) -> float:
    """One NCCL all-reduce (sum) of the block's [4096, 8192] bf16 output on
    its own, mean CUDA-event time: the box's collective speed for the same
    bytes, beside the fused kernel (every rank takes part)."""
    import torch
    import torch.distributed as dist

    t = torch.zeros((TOKENS, HIDDEN), dtype=torch.bfloat16, device="cuda")
    for _ in range(2):
        dist.all_reduce(t)
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(reps):
        dist.all_reduce(t)
    e.record()
    torch.cuda.synchronize()
    del t
    return s.elapsed_time(e) / reps


def nvlink_per_step(nv0, nv1, steps: int, world: int):
    """NVLink data bytes per timed step per GPU (the largest over the ranks)
    from the NVML counters read around the timed steps; every rank takes
    part in the reduction, null where a rank had no counters."""
    if world == 1:
        return None
    have = nv0 is not None and nv1 is not None
    tx = (nv1[0] - nv0[0]) * 1024.0 / steps if have else -1.0
    rx = (nv1[1] - nv0[1]) * 1024.0 / steps if have else -1.0
    lo = _max_over_ranks([-tx, -rx], world)  # any rank without counters shows as +1
    tx, rx = _max_over_ranks([tx, rx], world)
    if lo[0] > 0 or lo[1] > 0 or tx <= 0:
        return None
    payload = 2.0 * TOKENS * HIDDEN
    return {"tx_mb": round(tx / 1e6, 1), "rx_mb": round(rx / 1e6, 1),
            "all_reduce_payload_mb": round(payload / 1e6, 1)}


def tp_e2e(args, block, x, rank: int, world: int, guard) -> dict:
    """The block through ``HostStream``: pinned host batch in, block, output
    rows back to pinned host memory, every step, inside the timed region."""
    import torch

    from aot_kernel.tp_mlp import HostStream

    hs = HostStream(block, TOKENS, HIDDEN, x.device)
    x_host = x.cpu().pin_memory()
    out_host = torch.empty((TOKENS, HIDDEN), dtype=torch.bfloat16).pin_memory()
    for _ in range(2):
        hs.submit(x_host, out_host)
    hs.drain()
    _meet(world)
    guard.check()
    cur = torch.cuda.current_stream()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    hs.h2d.wait_stream(cur)  # the first copy-in starts after the start event
    for _ in range(args.steps):
        hs.submit(x_host, out_host)
    hs.drain()
    e.record()
    torch.cuda.synchronize()
    (ms,) = _max_over_ranks([s.elapsed_time(e) / args.steps], world)
    # the rows this rank read back equal the device-resident block's output
    y = block(x)
    diff = (out_host[hs.lo:hs.hi].float() - y[hs.lo:hs.hi].float().cpu()).abs().max().item()
    (diff,) = _max_over_ranks([diff], world)
    return {"value": TOKENS / (ms * 1e-3), "unit": "tokens/s",
            "h2d_bytes_per_step": hs.h2d_bytes() * world, "d2h_bytes_per_step": hs.d2h_bytes() * world,
            "ms_per_step": round(ms, 4), "max_abs_diff_vs_device": diff,
            "api": "tp_mlp.HostStream.submit: 1/N of the pinned rows in per rank, all-gather, "
                   "block, 1/N out"}


def tp_parity(block, x, host: dict, rank: int) -> dict | None:
    """Sampled output rows against the reference composition on CPU."""
    import torch

    y = block(x)  # every rank takes part (the all-reduce)
    torch.cuda.synchronize()
    if rank != 0:
        return None
    rows = torch.randperm(TOKENS, generator=torch.Generator().manual_seed(5))[:PARITY_ROWS].sort().values
    got = y[rows.cuda()].float().cpu()
    ref = reference_block_cpu(host["x"][rows], host["nw"], host["wgu"], host["wd"]).float()
    err = (got - ref).abs().max().item()
    scale = ref.abs().max().item()
    return {"rows": PARITY_ROWS, "max_abs_err": err, "max_abs_ref": scale,
            "err_frac": round(err / scale, 6), "tol_frac": PARITY_TOL,
            "pass": bool(err <= PARITY_TOL * scale),
            "reference": "ref ops on CPU"}


# ---------------------------------------------------------------- the reference on the host

def reference_block_cpu(x, nw, wgu, wd, eps: float = EPS):
    """The reference's MLP block on CPU tensors, one torch call per reference
    op: ref.rmsnorm = F.rms_norm(x, (H,), w, eps) (ref/norm.py:11-12),
    ref.gemm = a @ b (ref/gemm.py:4-5), ref.silu = F.silu
    (ref/activation.py:15-16); silu(gate) * up as ref.silu(gate) * up."""
    import torch.nn.functional as F

    h = F.rms_norm(x, (x.shape[-1],), nw, eps)
    gu = h @ wgu
    inter = wgu.shape[1] // 2
    act = F.silu(gu[:, :inter]) * gu[:, inter:]
    return act @ wd


def _cpu_inputs(seed: int = 0):
    """Block inputs for a CPU-only run, bf16: x ~ N(0, 1), norm weight
    N(1, 0.1), weights N(0, 0.02).  The weights are tiled from a seeded pool
    of 2^24 samples (drawing 700 M samples one by one would take longer than
    the timing itself; the GEMM's speed does not depend on the values)."""
    import torch

    g = torch.Generator().manual_seed(seed)
    pool = torch.randn(1 << 24, generator=g)

    def tiled(shape, std, offset):
        n = shape[0] * shape[1]
        reps = -(-(n + offset) // pool.numel())
        flat = pool.repeat(reps)[offset:offset + n]
        return (flat * std).to(torch.bfloat16).reshape(shape)

    x = torch.randn((TOKENS, HIDDEN), generator=g).to(torch.bfloat16)
    nw = (torch.randn((HIDDEN,), generator=g) * 0.1 + 1.0).to(torch.bfloat16)
    return x, nw, tiled((HIDDEN, 2 * INTER), 0.02, 12345), tiled((INTER, HIDDEN), 0.02, 777)


def cpu_block_times(x, nw, wgu, wd, steps: int, warmup: int, budget_s: float | None = None):
    """Seconds per reference block step on the host, all threads."""
    import torch

    torch.set_num_threads(os.cpu_count() or 1)
    for _ in range(warmup):
        reference_block_cpu(x, nw, wgu, wd)
    times = []
    t_all = time.perf_counter()
    for _ in range(steps):
        t0 = time.perf_counter()
        reference_block_cpu(x, nw, wgu, wd)
        times.append(time.perf_counter() - t0)
        if budget_s is not None and time.perf_counter() - t_all >= budget_s:
            break
    return times, torch.get_num_threads()


def cpu_baseline(host: dict) -> dict:
    """The reference composition on the host's cores, on the same 4096-token
    block and weights as the GPU run (a bounded number of steps)."""
    times, cores = cpu_block_times(host["x"], host["nw"], host["wgu"], host["wd"], steps=8,
                                   warmup=1, budget_s=15.0)
    mean = statistics.mean(times)
    return {"value": TOKENS / mean, "unit": "tokens/s", "cores": cores, "kind": "port",
            "sample": f"the full block (4096 tokens, same inputs) x {len(times)} steps, "
                      f"{mean * 1e3:.0f} ms per step; torch CPU composition of ref.rmsnorm, "
                      f"ref.gemm, ref.silu",
            "cpu_count": os.cpu_count()}


# ---------------------------------------------------------------- per-workload table (N = 1)

def traffic_per_launch(key: str):
    p = REPO / "profiles" / "traffic.json"
    if not p.exists():
        return None
    try:
        return json.loads(p.read_text()).get(key)
    except ValueError:
        return None


def graph_launch_ms(calls, replays: int = 4) -> float:
    """Mean device time of one launch: the launches in `calls` (one per input
    set, the sets together larger than L2) are captured once into a CUDA graph
    and the graph is replayed back to back; host dispatch is not timed."""
    import torch

    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for c in calls:  # first calls set per-device kernel attributes
            c()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for c in calls:
            c()
    g.replay()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(replays):
        g.replay()
    e.record()
    torch.cuda.synchronize()
    ms = s.elapsed_time(e) / (replays * len(calls))
    del g
    return ms


def _sets_for(nbytes: int, cap: int = 16) -> int:
    """Input copies needed for a rotation of at least 2x L2."""
    return max(1, min(cap, -(-2 * L2_BYTES // max(1, nbytes))))


def gemm_8192(args, peaks: dict) -> dict:
    """The square 8192^3 bf16 GEMM through aot_kernel.gemm: args.steps launches
    after args.warmup, each bracketed by CUDA events (operands 256 MB > L2)."""
    import torch

    import aot_kernel

    n = 8192
    a = rand_bf16((n, n), 1)
    b = rand_bf16((n, n), 2, std=n ** -0.5)
    for _ in range(args.warmup):
        aot_kernel.gemm(a, b)
    torch.cuda.synchronize()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(args.steps)]
    for s, e in evs:
        s.record()
        aot_kernel.gemm(a, b)
        e.record()
    torch.cuda.synchronize()
    ms = statistics.mean(s.elapsed_time(e) for s, e in evs)
    tf = 2.0 * n ** 3 / (ms * 1e-3) / 1e12
    return {"ms": round(ms, 4), "tflops": round(tf, 1), "frac": round(tf / peaks["bf16_tflops"], 4),
            "traffic": traffic_per_launch("gemm_8192")}


def kernel_table(peaks: dict) -> dict:
    """Every configured workload of the path, timed from CUDA-graph replays.
    Entries are [ms, TFLOP/s or GB/s, fraction of the measured peak] (the
    8-bit GEMMs: [ms, TFLOP/s, ratio to the library kernel])."""
    import torch

    import aot_kernel

    out = {}
    ridge = peaks["bf16_tflops"] * 1e12 / (peaks["hbm_gbs"] * 1e9)

    def gemm_entry(M, K, N, seed, b_std):
        nbytes = 2 * (M * K + K * N)
        R = _sets_for(nbytes)
        sets = [(rand_bf16((M, K), seed + 2 * i), rand_bf16((K, N), seed + 2 * i + 1, std=b_std))
                for i in range(R)]
        outs = [torch.empty((M, N), device="cuda", dtype=torch.bfloat16) for _ in range(R)]
        calls = [lambda a=a, b=b, c=c: aot_kernel.gemm(a, b, out=c) for (a, b), c in zip(sets, outs)]
        ms = graph_launch_ms(calls)
        # cuBLAS (torch.matmul) on the same operands: its time / ours
        lib = [lambda a=a, b=b, c=c: torch.matmul(a, b, out=c) for (a, b), c in zip(sets, outs)]
        try:
            vs_lib = round(graph_launch_ms(lib) / ms, 3)
        except Exception:  # noqa: BLE001  (library path unavailable on this build)
            vs_lib = None
        del sets, outs, calls, lib
        flops = 2.0 * M * N * K
        nbytes = 2.0 * (M * K + K * N + M * N)
        if flops / nbytes >= ridge:
            tf = flops / (ms * 1e-3) / 1e12
            return [round(ms, 5), round(tf, 1), round(tf / peaks["bf16_tflops"], 3), vs_lib]
        gbs = nbytes / (ms * 1e-3) / 1e9
        return [round(ms, 5), round(gbs, 1), round(gbs / peaks["hbm_gbs"], 3), vs_lib]

    for n in (2048, 4096, 8192, 16384):
        out[f"gemm_{n}^3"] = gemm_entry(n, n, n, 10 + n, n ** -0.5)
    for K, N in ((4096, 6144), (4096, 28672), (14336, 4096)):
        for M in (1, 16, 128, 2048, 8192):
            out[f"lin_M{M}_K{K}_N{N}"] = gemm_entry(M, K, N, M + K + N, 0.02)
    for M in (2048, 8192):  # Llama-3-8B gate/up (I = 14336) with the fused silu epilogue
        K, inter = 4096, 14336
        a = rand_bf16((M, K), 50 + M)
        w = rand_bf16((K, 2 * inter), 51 + M, std=0.02)
        o = torch.empty((M, inter), device="cuda", dtype=torch.bfloat16)
        ms = graph_launch_ms([lambda: torch.ops.aot_kernel.gemm_silu_mul(o, a, w)])
        tf = 2.0 * M * K * 2 * inter / (ms * 1e-3) / 1e12
        out[f"gate_up_silu_M{M}_K{K}_I{inter}"] = [round(ms, 5), round(tf, 1),
                                                   round(tf / peaks["bf16_tflops"], 3)]
        del a, w, o
    torch.cuda.empty_cache()

    # 8-bit scaled GEMM (rowwise scales, bf16 out) beside the library kernel
    # for the same operation on the same box: cuBLASLt fp8 through
    # torch._scaled_mm (B column-major, as it requires) and torch._int_mm plus
    # a dequantising multiply for int8 - the baselines of the reference's
    # benchmarks/gemm/bench_scaled_gemm.py.
    def scaled_entry(n, qdtype, seed):
        M = K = N = n
        R = _sets_for(M * K + K * N)
        sets = [(rand_q((M, K), seed + 2 * i, qdtype), rand_q((K, N), seed + 2 * i + 1, qdtype))
                for i in range(R)]
        sa, sb = row_scales(M, N, seed + 99)
        outs = [torch.empty((M, N), device="cuda", dtype=torch.bfloat16) for _ in range(R)]
        calls = [lambda a=a, b=b, c=c: torch.ops.aot_kernel.scaled_gemm(c, a, b, sa, sb, True)
                 for (a, b), c in zip(sets, outs)]
        ms = graph_launch_ms(calls)
        tf = 2.0 * M * N * K / (ms * 1e-3) / 1e12
        entry = [round(ms, 5), round(tf, 1), None]
        cols = [b.t().contiguous().t() for _, b in sets]  # [K, N] views of [N, K] storage
        del outs, calls
        try:
            if qdtype == "int8":
                lib = [lambda a=a, bc=bc: (torch._int_mm(a, bc).float() * sa[:, None] * sb[None, :])
                       .to(torch.bfloat16) for (a, _), bc in zip(sets, cols)]
            else:
                sa2, sb2 = sa.reshape(M, 1), sb.reshape(1, N)
                lib = [lambda a=a, bc=bc: torch._scaled_mm(a, bc, scale_a=sa2, scale_b=sb2,
                                                           out_dtype=torch.bfloat16)
                       for (a, _), bc in zip(sets, cols)]
            entry[2] = round(graph_launch_ms(lib) / ms, 3)
        except Exception:  # noqa: BLE001  (library path unavailable on this build)
            pass
        del sets, cols
        torch.cuda.empty_cache()
        return entry

    for n in (4096, 8192):
        out[f"fp8_{n}^3_vs_cublaslt"] = scaled_entry(n, "e4m3", 70 + n)
        out[f"int8_{n}^3_vs_torch"] = scaled_entry(n, "int8", 80 + n)

    def hbm_entry(calls, nbytes):
        ms = graph_launch_ms(calls)
        gbs = nbytes / (ms * 1e-3) / 1e9
        return [round(ms, 5), round(gbs, 1), round(gbs / peaks["hbm_gbs"], 3)]

    rows, cols = 8192, 4096
    R = _sets_for(rows * cols * 2)
    w = rand_bf16((cols,), 21, std=0.1, mean=1.0)
    xs = [rand_bf16((rows, cols), 20 + 2 * i) for i in range(R)]
    out["rms_norm_8192x4096"] = hbm_entry([lambda x=x: aot_kernel.rms_norm(x, w) for x in xs],
                                          2.0 * rows * cols * 2 + cols * 2)
    out["rms_rstd_8192x4096"] = hbm_entry([lambda x=x: aot_kernel.rms_rstd(x) for x in xs],
                                          1.0 * rows * cols * 2 + rows * 4)
    rs = [rand_bf16((rows, cols), 40 + 2 * i) for i in range(R)]
    out["add_rms_norm_8192x4096"] = hbm_entry(
        [lambda x=x, r=r: aot_kernel.add_rmsnorm(x, r, w) for x, r in zip(xs, rs)],
        4.0 * rows * cols * 2 + cols * 2)
    del xs, rs
    rows, cols = 8192, 14336
    g = rand_bf16((rows, cols), 22, std=2.0)
    u = rand_bf16((rows, cols), 23, std=2.0)
    out["silu_8192x14336"] = hbm_entry([lambda: aot_kernel.silu(g), lambda: aot_kernel.silu(u)],
                                       2.0 * rows * cols * 2)
    out["silu_mul_8192x14336"] = hbm_entry([lambda: aot_kernel.silu_mul(g, u),
                                            lambda: aot_kernel.silu_mul(u, g)],
                                           3.0 * rows * cols * 2)
    del g, u
    torch.cuda.empty_cache()
    return out


# ---------------------------------------------------------------- main

def base_line(args, world: int) -> dict:
    return {
        "metric": "TP MLP tokens/s (Llama-3-70B MLP block, 4096 tokens, bf16)",
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic: seeded x ~ N(0,1), norm weight N(1,0.1), weights N(0,0.02)",
        "config": {"workload": "Llama-3-70B MLP block: x[4096,8192] -> rms_norm -> gate/up "
                               "8192->2x28672 -> silu(gate)*up -> down 28672->8192 -> all-reduce",
                   "tokens": TOKENS, "hidden": HIDDEN, "intermediate": INTER,
                   "l2": "weights 1.41 GB split over the ranks plus activations exceed the 126 MB "
                         "L2; every step re-reads them"},
    }


def run_reference(args) -> None:
    """The reference composition on the host's cores, rank 0 only."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    world = int(os.environ.get("WORLD_SIZE", "1"))
    x, nw, wgu, wd = _cpu_inputs()
    times, cores = cpu_block_times(x, nw, wgu, wd, steps=args.steps, warmup=args.warmup)
    mean = statistics.mean(times)
    value = TOKENS / mean
    line = base_line(args, world)
    line.update({
        "impl": "reference", "parallelism": "host CPU, all threads (one process)",
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": "port",
                         "sample": f"the full block (4096 tokens) x {len(times)} timed steps after "
                                   f"{args.warmup} warm-up; torch CPU composition of ref.rmsnorm, "
                                   f"ref.gemm, ref.silu"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "gpu_launches": 0,
        "value": value, "ms_per_step": mean * 1e3,
    })
    print(json.dumps(line), flush=True)


def run_case(args) -> None:
    import torch

    import aot_kernel
    from aot_kernel import capi

    kind, shape = CASES[args.case]
    if kind == "gemm":
        M, K, N = shape
        a = rand_bf16((M, K), 1)
        b = rand_bf16((K, N), 2, std=0.02)
        fn = lambda: aot_kernel.gemm(a, b)  # noqa: E731
    elif kind == "cublas":
        M, K, N = shape
        a = rand_bf16((M, K), 1)
        b = rand_bf16((K, N), 2, std=0.02)
        c = torch.empty((M, N), device="cuda", dtype=torch.bfloat16)
        fn = lambda: torch.matmul(a, b, out=c)  # noqa: E731
    elif kind == "gemm_tc2":
        M, K, N = shape
        a = rand_bf16((M, K), 1)
        b = rand_bf16((K, N), 2, std=0.02)
        c = torch.empty((M, N), device="cuda", dtype=torch.bfloat16)
        fn = lambda: capi.gemm_tc2(c, a, b, M, N, K, capi.dtype_code(a.dtype))  # noqa: E731
    elif kind == "gate_up_silu":
        M, K, inter = shape
        a = rand_bf16((M, K), 1)
        w = rand_bf16((K, 2 * inter), 2, std=0.02)
        fn = lambda: aot_kernel.gemm_silu_mul(a, w)  # noqa: E731
    elif kind == "tp_gate_up":
        M, K, inter = shape
        a = rand_bf16((M, K), 1)
        w = rand_bf16((K, 2 * inter), 2, std=0.02)
        rstd = aot_kernel.rms_rstd(a)
        fn = lambda: aot_kernel.gemm_silu_mul(a, w, rstd)  # noqa: E731
    elif kind.startswith("scaled_gemm"):
        M, K, N = shape
        q = kind.rsplit("_", 1)[1]
        a, b = rand_q((M, K), 1, q), rand_q((K, N), 2, q)
        sa, sb = row_scales(M, N, 3)
        fn = lambda: aot_kernel.scaled_gemm(a, b, sa, sb)  # noqa: E731
    elif kind == "rms_norm":
        x = rand_bf16(shape, 3)
        w = rand_bf16((shape[1],), 4, std=0.1, mean=1.0)
        fn = lambda: aot_kernel.rms_norm(x, w)  # noqa: E731
    elif kind == "rms_rstd":
        x = rand_bf16(shape, 3)
        fn = lambda: aot_kernel.rms_rstd(x)  # noqa: E731
    elif kind == "add_rms_norm":
        x = rand_bf16(shape, 3)
        r = rand_bf16(shape, 8)
        w = rand_bf16((shape[1],), 4, std=0.1, mean=1.0)
        fn = lambda: aot_kernel.add_rmsnorm(x, r, w)  # noqa: E731
    elif kind == "silu":
        x = rand_bf16(shape, 5, std=2.0)
        fn = lambda: aot_kernel.silu(x)  # noqa: E731
    else:
        g = rand_bf16(shape, 6, std=2.0)
        u = rand_bf16(shape, 7, std=2.0)
        fn = lambda: aot_kernel.silu_mul(g, u)  # noqa: E731
    for _ in range(args.warmup + args.steps):
        fn()
    torch.cuda.synchronize()


def run_ours(args, rank: int, world: int, local: int, guard, held: dict) -> dict:
    import torch

    from aot_kernel import capi

    peaks, peak_src = load_peaks()
    x, block, host = tp_build(args, rank, world)
    held["block"] = block
    head = tp_timed(args, block, x, world, peaks, guard)
    # The block runs back to back for the whole timed region (seconds at the
    # power cap), so its kernels are held against the sustained GEMM peak.
    head["roofline"]["peak_source"] = f"{peak_src} (sustained bf16 GEMM)"
    guard.check()
    e2e = tp_e2e(args, block, x, rank, world, guard)
    guard.check()
    parity = tp_parity(block, x, host, rank)
    line = base_line(args, world)
    line["parallelism"] = (f"tp{world}: column-split gate/up, row-split down, "
                           + ("down GEMM fused with an NVSwitch all-reduce" if world > 1 and
                              block.allreduce == "fused" else
                              "NCCL all-reduce" if world > 1 else "one GPU"))
    tensor_frac = round(BLOCK_FLOPS / world / (peaks["bf16_tflops_sustained"] * 1e12)
                        / (head["ms_per_step"] * 1e-3), 4)
    if rank == 0 and world == 1 and not args.no_kernels:
        del block, held["block"]
        gc.collect()
        torch.cuda.empty_cache()
        line["kernels_fields"] = ("[ms, TFLOP/s or GB/s, fraction of the measured peak"
                                  "(, 16-bit GEMMs: cuBLAS time / ours)]")
        line["kernels"] = kernel_table(peaks)
        line["gemm_8192"] = gemm_8192(args, peaks)
    if rank == 0 and world == 1 and not args.no_cpu:
        line["cpu_baseline"] = cpu_baseline(host)
    wd = capi.watchdog_status(local)
    if wd:
        line["watchdog"] = wd
    line.update({k: head[k] for k in ("gpu_launches", "clocks", "roofline")})
    line["e2e"] = e2e
    line["tp_parity"] = parity
    # Last, and short: the figures a reader of the line's tail needs.
    line["phases_ms"] = head["phases_ms"]
    line["tensor_frac_per_gpu"] = tensor_frac
    if head["nvlink"] is not None:
        line["nvlink_per_step_per_gpu"] = head["nvlink"]
    if "kernels" in line:
        line["glance"] = glance(line)
    line.update({k: head[k] for k in ("value", "ms_per_step")})
    return line


GLANCE = {"gemm_8192^3": "gemm_8192", "gemm_2048^3": "gemm_2048",
          "lin_M1_K4096_N28672": "m1_n28672", "lin_M16_K4096_N28672": "m16_n28672",
          "lin_M1_K4096_N6144": "m1_n6144", "lin_M128_K4096_N6144": "m128_n6144",
          "lin_M1_K14336_N4096": "m1_down", "lin_M128_K14336_N4096": "m128_down",
          "gate_up_silu_M8192_K4096_I14336": "gate_up_silu", "rms_norm_8192x4096": "rms_norm",
          "rms_rstd_8192x4096": "rms_rstd", "add_rms_norm_8192x4096": "add_rms_norm",
          "silu_8192x14336": "silu", "silu_mul_8192x14336": "silu_mul"}


def glance(line: dict) -> dict:
    """Roofline fraction (and cuBLAS time / ours where timed) of the kernels
    a reader checks first."""
    out = {}
    for key, short in GLANCE.items():
        e = line["kernels"].get(key)
        if e:
            out[short] = e[2] if len(e) < 4 or e[3] is None else [e[2], e[3]]
    return out


def main() -> None:
    args = parse_args()
    if args.impl == "reference":
        run_reference(args)
        return
    if args.case:
        run_case(args)
        return
    from aot_kernel.rank_guard import RankGuard, nccl_env

    nccl_env(blocking=False)
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
        store = dist.distributed_c10d._get_default_store()
    else:
        store = dist.HashStore()
    import aot_kernel  # noqa: F401  (fails loudly when the extension is missing)

    guard = RankGuard(store, rank, world, prefix="bench")
    held: dict = {}
    line, ok = None, False
    try:
        line = run_ours(args, rank, world, local, guard, held)
        ok = True
    except BaseException:  # noqa: BLE001  (reported below; the rank leaves through the guard)
        traceback.print_exc()

    def release():
        held.clear()
        gc.collect()
        torch.cuda.synchronize()

    clean = guard.finish(ok, release, sync=torch.cuda.synchronize)
    if world > 1 and clean:
        dist.destroy_process_group()
    if rank == 0 and clean and line is not None:
        print(json.dumps(line), flush=True)
    sys.stdout.flush()
    if not clean:
        sys.stderr.flush()
        os._exit(1)


if __name__ == "__main__":
    main()
