"""CPU oracle for the dense-linear path - TEST INFRASTRUCTURE, not product code.

A numpy restatement of what the reference's torch oracle computes
(ref/gemm.py:4-5, ref/norm.py:11-12, ref/activation.py:11-16 of
gongyisheng/inference-kernel).  The arithmetic of those call sites lives in
PyTorch 2.11.0 (pinned by the reference's uv.lock:1736-1737), which is not part
of the reference tree; ``ops`` restates its published semantics for CPU
tensors and ``tests/golden`` pins the restatement to outputs of the reference's
own ``ref`` package run in the build container.

Only tests, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` may import this package, and only as the checker / the timed CPU
baseline; the kernels in ``aot_kernel`` never call it.
"""

from . import inputs, ops

__all__ = ["inputs", "ops"]
