"""Parity cases shared by the golden-vector generator and the tests.

Shapes follow the reference's own tests (tests/gemm/test_cuda.py:16-27,
tests/gemm/test_triton.py:110-121, tests/norm/test_cuda.py:11,
tests/activation/test_cuda.py:12 and :45) and its
CPU-runnable configuration (ref.gemm on A[1024,1024], B[1024,1024] bf16,
N(0,1), seed 0).  Inputs come from ``oracle.inputs.randn`` with a seed derived
from the case id, so any machine regenerates identical bits.
"""

from __future__ import annotations

import zlib
from dataclasses import dataclass, field

DTYPES = ("float32", "float16", "bfloat16")


def seed_of(case_id: str) -> int:
    return zlib.crc32(case_id.encode())


@dataclass(frozen=True)
class Case:
    op: str                     # gemm | rmsnorm | add_rmsnorm | silu | relu | silu_mul | scaled_gemm
    shape: tuple                # gemm, scaled_gemm: (M, K, N); others: input shape
    dtype: str                  # scaled_gemm: the output dtype
    eps: float = 1e-6
    x_std: float = 1.0
    w_mean: float = 0.0
    w_std: float = 1.0
    sample_rows: int = 0        # >0: golden keeps every `sample_rows`-th output row + a hash
    tags: tuple = field(default_factory=tuple)
    qdtype: str = ""            # scaled_gemm: e4m3 | e5m2 | int8
    scale_mode: str = ""        # scaled_gemm: tensor | row

    @property
    def id(self) -> str:
        dims = "x".join(str(d) for d in self.shape)
        extra = f"-eps{self.eps:g}" if self.eps != 1e-6 else ""
        extra += f"-xs{self.x_std:g}" if self.x_std != 1.0 else ""
        extra += f"-w{self.w_mean:g},{self.w_std:g}" if (self.w_mean, self.w_std) != (0.0, 1.0) else ""
        if self.op == "scaled_gemm":
            extra += f"-{self.qdtype}-{self.scale_mode}"
        return f"{self.op}-{dims}-{self.dtype}{extra}"


GEMM_SHAPES = [(8, 16, 8), (32, 64, 32), (17, 33, 23), (64, 128, 32), (128, 256, 128),
               (130, 64, 130), (256, 256, 256)]
RMSNORM_SHAPES = [(8, 16), (32, 64), (4, 16, 128), (2, 3, 1023), (8, 8, 8, 16384)]
ACT_SHAPES = [(1024,), (32, 1024), (4, 16, 1024), (1023,)]
SILU_MUL_SHAPES = [(4, 1024), (3, 1000), (2, 14336)]
ADD_RMSNORM_SHAPES = [(4, 4096), (3, 1000), (2, 3, 1023)]
# tests/gemm/test_triton.py:110-121 (M, K, N)
SCALED_GEMM_SHAPES = [(64, 64, 64), (128, 256, 128), (130, 64, 130), (256, 256, 256),
                      (129, 257, 193)]


def all_cases() -> list[Case]:
    cases: list[Case] = []
    for dt in DTYPES:
        cases += [Case("gemm", s, dt) for s in GEMM_SHAPES]
        for s in RMSNORM_SHAPES:
            cases.append(Case("rmsnorm", s, dt, sample_rows=61 if s[-1] >= 16384 else 0))
        cases += [Case("silu", s, dt) for s in ACT_SHAPES]
        cases += [Case("relu", s, dt) for s in ACT_SHAPES]
        cases += [Case("silu_mul", s, dt, x_std=2.0) for s in SILU_MUL_SHAPES]
        cases += [Case("add_rmsnorm", s, dt, w_mean=1.0, w_std=0.1) for s in ADD_RMSNORM_SHAPES]
    for s in SCALED_GEMM_SHAPES:
        for q in ("e4m3", "int8"):
            for mode in ("tensor", "row"):
                cases.append(Case("scaled_gemm", s, "bfloat16", qdtype=q, scale_mode=mode))
    for q in ("e5m2",):
        cases.append(Case("scaled_gemm", (128, 256, 128), "bfloat16", qdtype=q, scale_mode="row"))
    for out in ("float16", "float32"):
        cases.append(Case("scaled_gemm", (128, 256, 128), out, qdtype="e4m3", scale_mode="row"))
        cases.append(Case("scaled_gemm", (130, 64, 130), out, qdtype="int8", scale_mode="tensor"))
    # custom eps (tests/norm/test_cuda.py:37-46)
    cases.append(Case("rmsnorm", (4, 32), "float32", eps=1e-3))
    # the CPU-runnable configuration: ref.gemm 1024^3 bf16, N(0,1)
    cases.append(Case("gemm", (1024, 1024, 1024), "bfloat16", sample_rows=31, tags=("config",)))
    # rms_norm configuration: x[8192,4096] N(0,1), weight N(1, 0.1), eps 1e-6
    cases.append(Case("rmsnorm", (8192, 4096), "bfloat16", w_mean=1.0, w_std=0.1, sample_rows=257,
                      tags=("config",)))
    return cases


def make_inputs(case: Case):
    """numpy float32 inputs of `case` (values representable in case.dtype)."""
    from oracle.inputs import quantized, randn, scales

    s = seed_of(case.id)
    if case.op == "scaled_gemm":
        M, K, N = case.shape
        sa, sb = scales(M, N, case.scale_mode, s + 2)
        return (quantized((M, K), s, case.qdtype), quantized((K, N), s + 1, case.qdtype), sa, sb)
    if case.op == "gemm":
        M, K, N = case.shape
        return (randn((M, K), s, case.dtype), randn((K, N), s + 1, case.dtype))
    if case.op == "rmsnorm":
        x = randn(case.shape, s, case.dtype, std=case.x_std)
        w = randn((case.shape[-1],), s + 1, case.dtype, mean=case.w_mean, std=case.w_std)
        return (x, w)
    if case.op == "add_rmsnorm":
        return (randn(case.shape, s, case.dtype, std=case.x_std),
                randn(case.shape, s + 2, case.dtype, std=case.x_std),
                randn((case.shape[-1],), s + 1, case.dtype, mean=case.w_mean, std=case.w_std))
    if case.op in ("silu", "relu"):
        return (randn(case.shape, s, case.dtype, std=case.x_std),)
    if case.op == "silu_mul":
        return (randn(case.shape, s, case.dtype, std=case.x_std),
                randn(case.shape, s + 1, case.dtype, std=case.x_std))
    raise ValueError(case.op)


def oracle_output(case: Case, inputs):
    from oracle import ops

    if case.op == "gemm":
        return ops.gemm(*inputs, case.dtype)
    if case.op == "rmsnorm":
        return ops.rmsnorm(*inputs, case.eps, case.dtype)
    if case.op == "add_rmsnorm":
        return ops.add_rmsnorm(*inputs, case.eps, case.dtype)[0]
    if case.op == "silu":
        return ops.silu(*inputs, case.dtype)
    if case.op == "relu":
        return ops.relu(*inputs, case.dtype)
    if case.op == "silu_mul":
        return ops.silu_mul_composed(*inputs, case.dtype)
    if case.op == "scaled_gemm":
        return ops.scaled_gemm(*inputs, case.qdtype, case.dtype)
    raise ValueError(case.op)


def sampled(case: Case, out):
    """The rows of `out` the golden file keeps for sampled cases (all rows otherwise)."""
    if not case.sample_rows:
        return out
    flat = out.reshape(-1, out.shape[-1])
    return flat[:: case.sample_rows]
