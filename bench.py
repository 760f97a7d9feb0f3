#!/usr/bin/env python
"""Benchmark of the dense-linear inference path on B200.

Headline (one JSON line on rank 0): bf16 GEMM TFLOP/s on the square
M = N = K = 8192 problem (fp32 accumulation, bf16 output) through the
``aot_kernel`` public API.  A step is one GEMM over operands already resident
in HBM; at N GPUs every rank runs its own GEMM (independent replicas, weak
scaling) and ``value`` is the sum over ranks.  The same line carries:

* ``roofline``  - the GEMM kernel's achieved TFLOP/s (2*M*N*K / mean CUDA-event
  duration of its launches) against the measured bf16 peak;
* ``e2e``       - the same metric through the public API with pinned host
  buffers: host->device copy of A and B, the GEMM, device->host copy of C;
* ``cpu_baseline`` - the reference's CPU GEMM (``a @ b`` on CPU bf16 tensors,
  all host threads) on a bounded row sample of the same problem, with the
  numpy oracle's rate beside it (rank 0, N = 1);
* ``kernels``   - the remaining workloads of the path at their configured sizes:
  the square sweep, the Llama-3-8B linear layers from decode to prefill,
  rms_norm, silu and silu(gate)*up, each with its roofline fraction (N = 1);
* ``tp_mlp``    - tokens/s of the Llama-3-70B MLP block (4096 tokens,
  hidden 8192, intermediate 28672) tensor-parallel over the N ranks with one
  NCCL all-reduce (the multi-GPU path; strong scaling in tokens).

``--impl reference`` times the reference's CPU path (``ref.gemm`` = ``a @ b``
on CPU tensors, all host threads) on the same metric instead; under torchrun
only rank 0 runs it.

``--case NAME`` runs only NAME's launches (warmup + steps) and prints nothing
else: the command the committed ncu summaries under profiles/ were made with.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import time
from datetime import timedelta
from pathlib import Path

REPO = Path(__file__).resolve().parent
for _p in (REPO, REPO / "inference-kernel_b200"):
    if str(_p) not in sys.path:
        sys.path.insert(0, str(_p))

FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
HEADLINE = (8192, 8192, 8192)
L2_BYTES = 126 * 1024 * 1024


# --case workloads: name -> (kind, shape)
CASES = {
    "gemm_8192": ("gemm", (8192, 8192, 8192)),
    "gemm_4096": ("gemm", (4096, 4096, 4096)),
    "gemm_decode_m1": ("gemm", (1, 4096, 28672)),
    "gemm_decode_m16": ("gemm", (16, 4096, 28672)),
    "gemm_m128_down": ("gemm", (128, 14336, 4096)),
    "gate_up_silu_2048": ("gate_up_silu", (2048, 4096, 14336)),
    "scaled_gemm_fp8_8192": ("scaled_gemm_e4m3", (8192, 8192, 8192)),
    "scaled_gemm_fp8_4096": ("scaled_gemm_e4m3", (4096, 4096, 4096)),
    "scaled_gemm_int8_4096": ("scaled_gemm_int8", (4096, 4096, 4096)),
    "rms_norm": ("rms_norm", (8192, 4096)),
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
    ap.add_argument("--no-tp", action="store_true", help="skip the tensor-parallel MLP block")
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

class ClockSampler:
    """Samples this rank's GPU clock, power and clock-event reasons through NVML
    (read-only queries) every 10 ms while the timed region runs."""

    REASONS = {"hw_slowdown": "nvmlClocksEventReasonHwSlowdown",
               "hw_thermal_slowdown": "nvmlClocksEventReasonHwThermalSlowdown",
               "sw_thermal_slowdown": "nvmlClocksEventReasonSwThermalSlowdown",
               "sw_power_cap": "nvmlClocksEventReasonSwPowerCap",
               "hw_power_brake": "nvmlClocksEventReasonHwPowerBrakeSlowdown"}

    def __init__(self, device: int = 0, period_s: float = 0.01):
        self.device, self.period = device, period_s
        self.samples: list[tuple[float, float, int]] = []
        self.max_mhz = None
        self._stop = None
        self._thread = None
        self._nvml = None

    def _handle(self):
        import pynvml
        import torch

        pynvml.nvmlInit()
        p = torch.cuda.get_device_properties(self.device)
        # torch reports the PCI location as integers; NVML wants "DDDDDDDD:BB:DD.0".
        bus_id = f"{int(p.pci_domain_id):08X}:{int(p.pci_bus_id):02X}:{int(p.pci_device_id):02X}.0"
        try:
            return pynvml.nvmlDeviceGetHandleByPciBusId(bus_id.encode())
        except pynvml.NVMLError:
            return pynvml.nvmlDeviceGetHandleByIndex(self.device)

    def _run(self, h):
        nv = self._nvml
        while not self._stop.is_set():
            try:
                sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                pw = nv.nvmlDeviceGetPowerUsage(h) / 1000.0
                rs = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                self.samples.append((float(sm), pw, int(rs)))
            except Exception:  # noqa: BLE001
                pass
            self._stop.wait(self.period)

    def __enter__(self):
        import threading

        try:
            import pynvml

            self._nvml = pynvml
            h = self._handle()
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))
        except Exception:  # noqa: BLE001
            self._nvml = None
            return self
        self._stop = threading.Event()
        self._thread = threading.Thread(target=self._run, args=(h,), daemon=True)
        self._thread.start()
        return self

    def __exit__(self, *exc):
        if self._thread is not None:
            self._stop.set()
            self._thread.join(timeout=5)
        return False

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


def headline_gemm(args, rank: int, world: int, peaks: dict):
    import torch
    import torch.distributed as dist

    import aot_kernel

    M, N, K = HEADLINE
    a = rand_bf16((M, K), 1 + rank)
    b = rand_bf16((K, N), 2 + rank, std=K ** -0.5)
    flops = 2.0 * M * N * K

    def step():
        return aot_kernel.gemm(a, b)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(torch.cuda.current_device()) as clocks:
        events = []
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record()
        for _ in range(args.steps):
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            step()
            e.record()
            events.append((s, e))
        t1.record()
        torch.cuda.synchronize()
    total_ms = t0.elapsed_time(t1)
    launch_ms = statistics.mean(s.elapsed_time(e) for s, e in events)
    if world > 1:
        dist.barrier()
    t = torch.tensor([total_ms, launch_ms], device="cuda", dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_ms, launch_ms = t.tolist()

    # End to end through the public host-buffer API (aot_kernel.gemm_host ->
    # aotk_gemm_host): every step copies A and B in from pinned host memory and
    # C back out, overlapped with the GEMM row blocks.
    a_h = a.cpu().pin_memory()
    b_h = b.cpu().pin_memory()
    c_h = torch.empty((M, N), dtype=torch.bfloat16).pin_memory()

    def e2e_step():
        aot_kernel.gemm_host(a_h, b_h, out=c_h)

    e2e_steps = max(3, min(args.steps, 20))
    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(e2e_steps):
        e2e_step()
    e.record()
    torch.cuda.synchronize()
    e2e_ms = torch.tensor([s.elapsed_time(e) / e2e_steps], device="cuda", dtype=torch.float64)
    if world > 1:
        dist.all_reduce(e2e_ms, op=dist.ReduceOp.MAX)
    e2e_ms = float(e2e_ms.item())

    achieved = flops / (launch_ms * 1e-3) / 1e12
    res = {
        "value": world * flops * args.steps / (total_ms * 1e-3) / 1e12,
        "ms_per_step": total_ms / args.steps,
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peaks["bf16_tflops"],
                     "unit": "TFLOP/s", "frac": achieved / peaks["bf16_tflops"],
                     "traffic": traffic_per_launch("gemm_tc_8192")},
        "e2e": {"value": world * flops / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
                "h2d_bytes_per_step": a.nbytes + b.nbytes, "d2h_bytes_per_step": M * N * 2,
                "ms_per_step": e2e_ms,
                "api": "aot_kernel.gemm_host (C ABI aotk_gemm_host): pinned host A, B, C; "
                       "B then 128-row-multiple blocks of A copied in, C blocks copied out, "
                       "overlapped with the GEMM blocks"},
        "gpu_launches": args.steps,
        "clocks": clocks.summary(),
    }
    del a_h, b_h, c_h
    return res


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


def kernel_table(peaks: dict) -> dict:
    """Every configured workload of the path, timed from CUDA-graph replays."""
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
        del sets, outs, calls
        flops = 2.0 * M * N * K
        nbytes = 2.0 * (M * K + K * N + M * N)
        tf = flops / (ms * 1e-3) / 1e12
        gbs = nbytes / (ms * 1e-3) / 1e9
        bound = "tensor" if flops / nbytes >= ridge else "hbm"
        frac = tf / peaks["bf16_tflops"] if bound == "tensor" else gbs / peaks["hbm_gbs"]
        return {"ms": round(ms, 5), "tflops": round(tf, 2), "gbs": round(gbs, 1), "bound": bound,
                "frac": round(frac, 4), "input_sets": R}

    for n in (2048, 4096, 8192, 16384):
        out[f"gemm_{n}^3"] = gemm_entry(n, n, n, 10 + n, n ** -0.5)
    for K, N in ((4096, 6144), (4096, 28672), (14336, 4096)):
        for M in (1, 16, 128, 2048, 8192):
            out[f"linear_M{M}_K{K}_N{N}"] = gemm_entry(M, K, N, M + K + N, 0.02)
    for M in (2048, 8192):  # Llama-3-8B gate/up (I = 14336) with the fused silu epilogue
        K, inter = 4096, 14336
        a = rand_bf16((M, K), 50 + M)
        w = rand_bf16((K, 2 * inter), 51 + M, std=0.02)
        o = torch.empty((M, inter), device="cuda", dtype=torch.bfloat16)
        ms = graph_launch_ms([lambda: torch.ops.aot_kernel.gemm_silu_mul(o, a, w)])
        tf = 2.0 * M * K * 2 * inter / (ms * 1e-3) / 1e12
        out[f"gate_up_silu_M{M}_K{K}_I{inter}"] = {"ms": round(ms, 5), "tflops": round(tf, 2),
                                                   "bound": "tensor",
                                                   "frac": round(tf / peaks["bf16_tflops"], 4)}
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
        entry = {"ms": round(ms, 5), "tflops": round(tf, 2), "bound": "tensor", "input_sets": R}
        cols = [b.t().contiguous().t() for _, b in sets]  # [K, N] views of [N, K] storage
        del outs, calls
        try:
            if qdtype == "int8":
                lib = [lambda a=a, bc=bc: (torch._int_mm(a, bc).float() * sa[:, None] * sb[None, :])
                       .to(torch.bfloat16) for (a, _), bc in zip(sets, cols)]
                name = "torch._int_mm + dequant"
            else:
                sa2, sb2 = sa.reshape(M, 1), sb.reshape(1, N)
                lib = [lambda a=a, bc=bc: torch._scaled_mm(a, bc, scale_a=sa2, scale_b=sb2,
                                                           out_dtype=torch.bfloat16)
                       for (a, _), bc in zip(sets, cols)]
                name = "torch._scaled_mm (cuBLASLt)"
            lms = graph_launch_ms(lib)
            ltf = 2.0 * M * N * K / (lms * 1e-3) / 1e12
            entry["library"] = {"name": name, "ms": round(lms, 5), "tflops": round(ltf, 2)}
            entry["frac_of_library"] = round(tf / ltf, 4)
        except Exception as e:  # noqa: BLE001  (library path unavailable on this build)
            entry["library"] = {"unavailable": str(e).splitlines()[0][:160]}
        del sets, cols
        torch.cuda.empty_cache()
        return entry

    for n in (4096, 8192):
        out[f"scaled_gemm_fp8_{n}^3"] = scaled_entry(n, "e4m3", 70 + n)
        out[f"scaled_gemm_int8_{n}^3"] = scaled_entry(n, "int8", 80 + n)

    def hbm_entry(calls, nbytes, R):
        ms = graph_launch_ms(calls)
        gbs = nbytes / (ms * 1e-3) / 1e9
        return {"ms": round(ms, 5), "gbs": round(gbs, 1), "bound": "hbm",
                "frac": round(gbs / peaks["hbm_gbs"], 4), "bytes": int(nbytes), "input_sets": R}

    rows, cols = 8192, 4096
    R = _sets_for(rows * cols * 2)
    w = rand_bf16((cols,), 21, std=0.1, mean=1.0)
    xs = [rand_bf16((rows, cols), 20 + 2 * i) for i in range(R)]
    out["rms_norm_8192x4096"] = hbm_entry([lambda x=x: aot_kernel.rms_norm(x, w) for x in xs],
                                          2.0 * rows * cols * 2 + cols * 2, R)
    out["rms_rstd_8192x4096"] = hbm_entry([lambda x=x: aot_kernel.rms_rstd(x) for x in xs],
                                          1.0 * rows * cols * 2 + rows * 4, R)
    rs = [rand_bf16((rows, cols), 40 + 2 * i) for i in range(R)]
    out["add_rms_norm_8192x4096"] = hbm_entry(
        [lambda x=x, r=r: aot_kernel.add_rmsnorm(x, r, w) for x, r in zip(xs, rs)],
        4.0 * rows * cols * 2 + cols * 2, R)
    del xs, rs
    rows, cols = 8192, 14336
    g = rand_bf16((rows, cols), 22, std=2.0)
    u = rand_bf16((rows, cols), 23, std=2.0)
    out["silu_8192x14336"] = hbm_entry([lambda: aot_kernel.silu(g), lambda: aot_kernel.silu(u)],
                                       2.0 * rows * cols * 2, 2)
    out["silu_mul_8192x14336"] = hbm_entry([lambda: aot_kernel.silu_mul(g, u),
                                            lambda: aot_kernel.silu_mul(u, g)],
                                           3.0 * rows * cols * 2, 2)
    del g, u
    torch.cuda.empty_cache()
    return out


def tp_mlp(args, rank: int, world: int, peaks: dict) -> dict:
    import torch
    import torch.distributed as dist

    from aot_kernel.tp_mlp import (MLPShard, TensorParallelMLP, shard_down, shard_gate_up,
                                   shard_gate_up_folded, shard_gate_up_interleaved)

    T, H, inter = 4096, 8192, 28672
    x = rand_bf16((T, H), 30)
    nw = rand_bf16((H,), 31, std=0.1, mean=1.0)
    w_gu = rand_bf16((H, 2 * inter), 32, std=0.02)
    fused_silu = not args.tp_unfused_silu
    fold_norm = fused_silu and not args.tp_unfolded_norm
    if fold_norm:
        wgu_r = shard_gate_up_folded(w_gu, nw, rank, world)
    else:
        wgu_r = (shard_gate_up_interleaved if fused_silu else shard_gate_up)(w_gu, rank, world)
    del w_gu
    w_d = rand_bf16((inter, H), 33, std=0.02)
    wd_r = shard_down(w_d, rank, world)
    del w_d
    torch.cuda.empty_cache()
    allreduce = args.tp_allreduce if world > 1 else "nccl"
    block = TensorParallelMLP(MLPShard(nw, wgu_r, wd_r, fused_silu=fused_silu, fold_norm=fold_norm),
                              eps=1e-6, chunks=args.tp_chunks, allreduce=allreduce)
    for _ in range(max(3, args.warmup)):
        block(x)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    steps = max(5, min(args.steps, 30))
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(steps):
        block(x)
    e.record()
    torch.cuda.synchronize()
    ms = torch.tensor([s.elapsed_time(e) / steps], device="cuda", dtype=torch.float64)
    if world > 1:
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    ms = float(ms.item())
    phases = tp_phase_breakdown(block, x, world)
    flops = 2.0 * T * H * 2 * inter + 2.0 * T * inter * H
    per_gpu_ideal_ms = flops / world / (peaks["bf16_tflops"] * 1e12) * 1e3
    return {"tokens_per_s": T / (ms * 1e-3), "ms_per_step": ms, "tokens": T, "hidden": H,
            "intermediate": inter, "tp": world, "chunks": args.tp_chunks,
            "allreduce": allreduce if world > 1 else None, "fused_silu": fused_silu,
            "fold_norm": fold_norm,
            "gpu_launches_per_step": (2 if fused_silu else 3)
            + (1 if world == 1 or allreduce == "fused" else args.tp_chunks),
            "tensor_frac_per_gpu": per_gpu_ideal_ms / ms, "allreduce_bytes": T * H * 2,
            "phases_ms": phases}


def tp_phase_breakdown(block, x, world: int, reps: int = 5) -> dict:
    """Device time of each op of one block step (mean of `reps` passes outside
    the timed region, CUDA events between ops, max over ranks).  A sleep
    kernel queued first keeps the host ahead so dispatch gaps are not timed."""
    import torch
    import torch.distributed as dist

    ops, s = block.ops, block.shard
    fused = world > 1 and block.allreduce == "fused"
    fsilu = s.fused_silu
    if s.fold_norm:
        names = ["rms_rstd", "gemm_gate_up+rms_norm+silu_mul (fused)"]
    else:
        names = ["rms_norm"] + (["gemm_gate_up+silu_mul (fused)"] if fsilu else
                                ["gemm_gate_up", "silu_mul"])
    names += ["gemm_down+all_reduce (fused)"] if fused else ["gemm_down", "all_reduce"]
    acc = torch.zeros(len(names), dtype=torch.float64, device="cuda")
    for _ in range(reps):
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(len(names) + 1)]
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        torch.cuda._sleep(2_000_000)
        i = 0
        ev[i].record()
        if s.fold_norm:
            rstd = ops.rms_rstd(x, block.eps)
            i += 1
            ev[i].record()
            act = ops.gemm_silu_mul(x, s.w_gate_up, rstd)
        elif fsilu:
            h = ops.rms_norm(x, s.norm_weight, block.eps)
            i += 1
            ev[i].record()
            act = ops.gemm_silu_mul(h, s.w_gate_up)
        else:
            h = ops.rms_norm(x, s.norm_weight, block.eps)
            i += 1
            ev[i].record()
            gu = ops.gemm(h, s.w_gate_up)
            i += 1
            ev[i].record()
            act = ops.silu_mul(gu[:, :block.inter_local], gu[:, block.inter_local:])
        i += 1
        ev[i].record()
        if fused:
            block._fused(act, s.w_down)
        else:
            out = ops.gemm(act, s.w_down)
            i += 1
            ev[i].record()
            if world > 1:
                dist.all_reduce(out)
        i += 1
        ev[i].record()
        torch.cuda.synchronize()
        acc += torch.tensor([ev[i].elapsed_time(ev[i + 1]) for i in range(len(names))],
                            dtype=torch.float64, device="cuda")
    acc /= reps
    if world > 1:
        dist.all_reduce(acc, op=dist.ReduceOp.MAX)
    return {n: round(v, 4) for n, v in zip(names, acc.tolist())}


def cpu_baseline(target_s: float = 8.0) -> dict:
    """The reference's CPU GEMM on a bounded row sample of the 8192^3 problem.

    ``ref.gemm`` is ``a @ b`` (ref/gemm.py:4-5); on CPU bf16 tensors torch runs
    it through its own bf16 GEMM with every host thread.  That call, ported
    as one line, is the timed value.  The numpy oracle (float32 BLAS) is timed
    beside it for reference.
    """
    import torch

    from oracle import ops

    M, N, K = HEADLINE
    rows = 1024
    torch.set_num_threads(os.cpu_count() or 1)
    g = torch.Generator().manual_seed(0)
    a = torch.randn((rows, K), generator=g).to(torch.bfloat16)
    b = (torch.randn((K, N), generator=g) * K ** -0.5).to(torch.bfloat16)

    def timed(fn, budget):
        fn()  # warm thread pools / packing
        n, t0 = 0, time.perf_counter()
        while True:
            fn()
            n += 1
            el = time.perf_counter() - t0
            if el >= budget or n >= 500:
                return n, el

    n, el = timed(lambda: a @ b, target_s)
    a_np, b_np = a.float().numpy(), b.float().numpy()
    n_np, el_np = timed(lambda: ops.gemm(a_np, b_np, "bfloat16"), target_s / 2)
    flops = 2.0 * rows * N * K
    return {"value": flops * n / el / 1e12, "unit": "TFLOP/s", "cores": torch.get_num_threads(),
            "kind": "port",
            "sample": f"A[{rows} of {M} rows, {K}] @ B[{K},{N}] bf16 on CPU via torch (the call "
                      f"ref.gemm makes), {n} repetitions in {el:.1f} s",
            "oracle_numpy_tflops": flops * n_np / el_np / 1e12,
            "cpu_count": os.cpu_count()}


# ---------------------------------------------------------------- main

def base_line(args, world: int) -> dict:
    M, N, K = HEADLINE
    return {
        "metric": "bf16 GEMM TFLOP/s (M=N=K=8192, fp32 accumulate, bf16 out)",
        "unit": "TFLOP/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic: seeded A ~ N(0,1), B ~ N(0,1/K) (Philox on device)",
        "config": {"workload": "square bf16 GEMM C[8192,8192] = A[8192,8192] B[8192,8192]",
                   "M": M, "N": N, "K": K,
                   "parallelism": f"replicas x{world} (one independent GEMM per GPU)",
                   "l2": "operands 256 MB > 126 MB L2 (no reuse across steps)"},
    }


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    cb = None
    per_step = []
    for i in range(args.warmup + args.steps):
        r = cpu_baseline(target_s=1.0)
        if i >= args.warmup:
            per_step.append(r)
        cb = r
    value = statistics.mean(r["value"] for r in per_step)
    line = base_line(args, int(os.environ.get("WORLD_SIZE", "1")))
    line.update({
        "impl": "reference", "value": value,
        "ms_per_step": statistics.mean(2.0 * 1024 * 8192 * 8192 / (r["value"] * 1e12) * 1e3
                                       for r in per_step),
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": cb["cores"], "kind": "port",
                         "sample": cb["sample"]},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "gpu_launches": 0,
    })
    line["config"]["parallelism"] = "host CPU, all threads (ref.gemm = a @ b on CPU tensors)"
    print(json.dumps(line), flush=True)


def run_case(args) -> None:
    import torch

    import aot_kernel

    kind, shape = CASES[args.case]
    if kind == "gemm":
        M, K, N = shape
        a = rand_bf16((M, K), 1)
        b = rand_bf16((K, N), 2, std=0.02)
        fn = lambda: aot_kernel.gemm(a, b)  # noqa: E731
    elif kind == "gate_up_silu":
        M, K, inter = shape
        a = rand_bf16((M, K), 1)
        w = rand_bf16((K, 2 * inter), 2, std=0.02)
        fn = lambda: aot_kernel.gemm_silu_mul(a, w)  # noqa: E731
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


def main() -> None:
    args = parse_args()
    if args.impl == "reference":
        run_reference(args)
        return
    if args.case:
        run_case(args)
        return
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    import aot_kernel  # noqa: F401  (fails loudly when the extension is missing)
    from aot_kernel import capi

    peaks, peak_src = load_peaks()
    line = base_line(args, world)
    head = headline_gemm(args, rank, world, peaks)
    line.update({k: head[k] for k in ("value", "ms_per_step", "roofline", "e2e", "gpu_launches",
                                      "clocks")})
    line["roofline"]["peak_source"] = f"{peak_src} (burst bf16 GEMM)"
    if not args.no_tp:
        line["tp_mlp"] = tp_mlp(args, rank, world, peaks)
    if rank == 0 and world == 1 and not args.no_kernels:
        line["kernels"] = kernel_table(peaks)
        line["kernels"]["peaks"] = {"hbm_gbs": peaks["hbm_gbs"], "bf16_tflops": peaks["bf16_tflops"],
                                    "source": peak_src}
    if rank == 0 and world == 1 and not args.no_cpu:
        line["cpu_baseline"] = cpu_baseline()
    wd = capi.watchdog_status(local)
    if wd:
        line["watchdog"] = wd
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
