"""B200 (sm_100a) kernels for the dense-linear inference path, behind the
``aot_kernel`` operator API of gongyisheng/inference-kernel.

Importing the package loads ``_C`` (the torch operator library, built in place
by ``inference-kernel_b200/build.py``), which registers ``torch.ops.aot_kernel.*``
and pulls in ``libaotk.so`` (the CUDA kernels and their C ABI).  Names and
signatures follow the reference's ``aot_kernel/__init__.py:8-20``; ``rms_norm``
is an alias of ``rmsnorm``; ``silu_mul``, ``add_rmsnorm`` and ``gemm_silu_mul``
are new fused ops (``interleave_gate_up`` builds the fused gate/up weight,
``fold_norm_weight`` and ``rms_rstd`` fold rms_norm into it); ``scaled_gemm`` is
the reference's 8-bit GEMM (``jit_kernel.gemm.scaled_gemm``, a Triton kernel
there) with the same signature; ``gemm_host`` runs ``gemm`` on host-resident
operands with the copies overlapped.
"""

from .activation import relu, silu, silu_mul
from .gemm import (fold_norm_weight, gemm, gemm_host, gemm_naive, gemm_silu_mul,
                   interleave_gate_up, scaled_gemm)
from .norm import add_rmsnorm, rms_norm, rms_rstd, rmsnorm

__version__ = "0.1.0"

__all__ = [
    "add_rmsnorm",
    "fold_norm_weight",
    "gemm",
    "gemm_host",
    "gemm_naive",
    "gemm_silu_mul",
    "interleave_gate_up",
    "relu",
    "rms_norm",
    "rms_rstd",
    "rmsnorm",
    "scaled_gemm",
    "silu",
    "silu_mul",
]
