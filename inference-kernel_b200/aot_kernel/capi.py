"""ctypes binding of the C ABI in ``include/aotk.h`` (``libaotk.so``).

This is the binding a non-torch host would write; the parity tests call the
kernels through it so that what they check is the C ABI itself.  Every
wrapper takes device pointers as integers (or torch tensors, converted with
``data_ptr()``) and a stream handle (default: torch's current stream when
torch is importable, else the legacy default stream), and raises
``AotkError`` with ``aotk_last_error()`` on a non-zero status.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libaotk.so"

FLOAT32, FLOAT16, BFLOAT16 = 0, 1, 2
FLOAT8_E4M3, INT8, FLOAT8_E5M2 = 3, 4, 5  # inputs of aotk_scaled_gemm
SCALE_TENSOR, SCALE_ROW = 0, 1
OK, ERR_INVALID_ARGUMENT, ERR_UNSUPPORTED, ERR_CUDA, ERR_DEVICE = 0, 1, 2, 3, 4

_i64 = ctypes.c_int64
_int = ctypes.c_int
_ptr = ctypes.c_void_p

# name -> argument types (all return int except aotk_last_error)
SIGNATURES: dict[str, list] = {
    "aotk_version": [],
    "aotk_silu_forward": [_ptr, _ptr, _i64, _int, _ptr],
    "aotk_relu_forward": [_ptr, _ptr, _i64, _int, _ptr],
    "aotk_silu_mul_forward": [_ptr, _i64, _ptr, _i64, _ptr, _i64, _i64, _i64, _int, _ptr],
    "aotk_rmsnorm_forward": [_ptr, _ptr, _ptr, _i64, _i64, ctypes.c_double, _int, _ptr],
    "aotk_add_rmsnorm_forward": [_ptr, _ptr, _ptr, _ptr, _ptr, _i64, _i64, ctypes.c_double, _int,
                                 _ptr],
    "aotk_gemm_opt": [_ptr, _ptr, _ptr, _i64, _i64, _i64, _int, _ptr],
    "aotk_gemm_opt_ws": [_ptr, _ptr, _ptr, _i64, _i64, _i64, _int, _ptr, ctypes.c_size_t, _ptr],
    "aotk_gemm_opt_workspace_size": [_i64, _i64, _i64, _int, ctypes.POINTER(ctypes.c_size_t)],
    "aotk_gemm_opt_noalloc": [_ptr, _ptr, _ptr, _i64, _i64, _i64, _int, _ptr],
    "aotk_gemm": [_ptr, _ptr, _ptr, _i64, _i64, _i64, _int, _ptr],
    "aotk_gemm_tc": [_ptr, _ptr, _ptr, _i64, _i64, _i64, _int, _ptr],
    "aotk_gemm_tc2": [_ptr, _ptr, _ptr, _i64, _i64, _i64, _int, _ptr],
    "aotk_gemm_tc2w": [_ptr, _ptr, _ptr, _i64, _i64, _i64, _int, _ptr],
    "aotk_gemm_path": [_i64, _i64, _i64, _int, _int, ctypes.POINTER(ctypes.c_int)],
    "aotk_gemm_skinny": [_ptr, _ptr, _ptr, _i64, _i64, _i64, _int, _ptr],
    "aotk_watchdog_status": [_int, ctypes.POINTER(ctypes.c_uint32), _int],
    "aotk_gemm_allreduce_tiles": [_i64, _i64, ctypes.POINTER(ctypes.c_int64)],
    "aotk_watchdog_selftest": [_ptr],
    "aotk_gemm_silu_mul": [_ptr, _ptr, _ptr, _i64, _i64, _i64, _int, _ptr, ctypes.c_size_t, _ptr],
    "aotk_gemm_silu_mul_workspace_size": [_i64, _i64, _i64, _int, ctypes.POINTER(ctypes.c_size_t)],
    "aotk_gemm_allreduce": [_ptr, _ptr, _i64, _i64, _i64, _int, ctypes.c_void_p, _ptr],
    "aotk_gemm_schedule": [_i64, _i64, _i64, _int, _int, _int, ctypes.POINTER(ctypes.c_int64)],
    "aotk_rmsnorm_rstd": [_ptr, _ptr, _i64, _i64, ctypes.c_double, _int, _ptr],
    "aotk_gemm_silu_mul_rowscale": [_ptr, _ptr, _ptr, _ptr, _i64, _i64, _i64, _int, _ptr,
                                    ctypes.c_size_t, _ptr],
    "aotk_gemm_host": [_ptr, _ptr, _ptr, _i64, _i64, _i64, _int, _ptr, _ptr, _ptr, _ptr,
                       ctypes.c_size_t, _ptr],
    "aotk_gemm_host_workspace_size": [_i64, _i64, _i64, _int, ctypes.POINTER(ctypes.c_size_t)],
    "aotk_scaled_gemm": [_ptr, _ptr, _ptr, _ptr, _ptr, _i64, _i64, _i64, _int, _int, _int, _ptr,
                         ctypes.c_size_t, _ptr],
    "aotk_scaled_gemm_workspace_size": [_i64, _i64, _i64, _int, ctypes.POINTER(ctypes.c_size_t)],
    "aotk_scaled_gemm_tc": [_ptr, _ptr, _ptr, _ptr, _ptr, _i64, _i64, _i64, _int, _int, _int, _ptr,
                            ctypes.c_size_t, _ptr],
    "aotk_scaled_gemm_simt": [_ptr, _ptr, _ptr, _ptr, _ptr, _i64, _i64, _i64, _int, _int, _int,
                              _ptr],
}


class AllReduceBuffers(ctypes.Structure):
    """aotk_allreduce_buffers (include/aotk.h)."""

    _fields_ = [
        ("rank", ctypes.c_int),
        ("world", ctypes.c_int),
        ("part", ctypes.c_void_p),
        ("part_multicast", ctypes.c_uint64),
        ("out_multicast", ctypes.c_uint64),
        ("counters", ctypes.c_void_p),
        ("peer_counters", ctypes.c_void_p),
        ("done", ctypes.c_void_p),
        ("peer_done", ctypes.c_void_p),
        ("epoch", ctypes.c_uint32),
    ]


class AotkError(RuntimeError):
    def __init__(self, fn: str, status: int, message: str):
        super().__init__(f"{fn} returned {status}: {message}")
        self.status = status


_lib: ctypes.CDLL | None = None


def load(path: str | Path | None = None) -> ctypes.CDLL:
    """Loads libaotk.so once and declares every entry point's signature."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    lib = ctypes.CDLL(str(path or LIB_PATH))
    lib.aotk_last_error.restype = ctypes.c_char_p
    lib.aotk_last_error.argtypes = []
    for name, argtypes in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = ctypes.c_int
        fn.argtypes = argtypes
    if path is None:
        _lib = lib
    return lib


def dtype_code(dtype) -> int:
    import torch

    return {
        torch.float32: FLOAT32,
        torch.float16: FLOAT16,
        torch.bfloat16: BFLOAT16,
        torch.float8_e4m3fn: FLOAT8_E4M3,
        torch.float8_e5m2: FLOAT8_E5M2,
        torch.int8: INT8,
    }[dtype]


def _p(x) -> int | None:
    if x is None:
        return None
    if isinstance(x, int):
        return x
    return x.data_ptr()


def _stream(stream) -> int | None:
    if stream is not None:
        return int(stream)
    try:
        import torch

        if torch.cuda.is_available():
            return torch.cuda.current_stream().cuda_stream
    except ImportError:
        pass
    return None


def _call(name: str, *args) -> None:
    lib = load()
    status = getattr(lib, name)(*args)
    if status != OK:
        raise AotkError(name, status, lib.aotk_last_error().decode())


def silu_forward(out, x, n: int, dtype: int, stream=None) -> None:
    _call("aotk_silu_forward", _p(out), _p(x), n, dtype, _stream(stream))


def relu_forward(out, x, n: int, dtype: int, stream=None) -> None:
    _call("aotk_relu_forward", _p(out), _p(x), n, dtype, _stream(stream))


def silu_mul_forward(out, out_stride, gate, gate_stride, up, up_stride, rows, cols, dtype,
                     stream=None) -> None:
    _call("aotk_silu_mul_forward", _p(out), out_stride, _p(gate), gate_stride, _p(up), up_stride,
          rows, cols, dtype, _stream(stream))


def rmsnorm_forward(out, x, weight, rows: int, cols: int, eps: float, dtype: int,
                    stream=None) -> None:
    _call("aotk_rmsnorm_forward", _p(out), _p(x), _p(weight), rows, cols, eps, dtype,
          _stream(stream))


def add_rmsnorm_forward(out, residual_out, x, residual, weight, rows: int, cols: int, eps: float,
                        dtype: int, stream=None) -> None:
    _call("aotk_add_rmsnorm_forward", _p(out), _p(residual_out), _p(x), _p(residual), _p(weight),
          rows, cols, eps, dtype, _stream(stream))


def _gemm(name, c, a, b, M, N, K, dtype, stream) -> None:
    _call(name, _p(c), _p(a), _p(b), M, N, K, dtype, _stream(stream))


def gemm_opt(c, a, b, M, N, K, dtype, stream=None) -> None:
    _gemm("aotk_gemm_opt", c, a, b, M, N, K, dtype, stream)


def gemm_opt_workspace_size(M, N, K, dtype) -> int:
    n = ctypes.c_size_t(0)
    _call("aotk_gemm_opt_workspace_size", M, N, K, dtype, ctypes.byref(n))
    return n.value


def gemm_opt_ws(c, a, b, M, N, K, dtype, workspace, workspace_bytes, stream=None) -> None:
    _call("aotk_gemm_opt_ws", _p(c), _p(a), _p(b), M, N, K, dtype, _p(workspace), workspace_bytes,
          _stream(stream))


def gemm_opt_noalloc(c, a, b, M, N, K, dtype, stream=None) -> None:
    """aotk_gemm_opt_ws with the library's built-in scratch; allocates nothing."""
    _gemm("aotk_gemm_opt_noalloc", c, a, b, M, N, K, dtype, stream)


def gemm(c, a, b, M, N, K, dtype, stream=None) -> None:
    _gemm("aotk_gemm", c, a, b, M, N, K, dtype, stream)


def gemm_tc(c, a, b, M, N, K, dtype, stream=None) -> None:
    _gemm("aotk_gemm_tc", c, a, b, M, N, K, dtype, stream)


def gemm_tc2(c, a, b, M, N, K, dtype, stream=None) -> None:
    _gemm("aotk_gemm_tc2", c, a, b, M, N, K, dtype, stream)


def gemm_tc2w(c, a, b, M, N, K, dtype, stream=None) -> None:
    _gemm("aotk_gemm_tc2w", c, a, b, M, N, K, dtype, stream)


PATHS = {0: "simt", 1: "skinny", 2: "tc", 3: "tc2_wide", 4: "tc2"}


def gemm_path(M, N, K, sm_count, with_workspace=True) -> str:
    """The kernel aotk_gemm_opt_ws picks for a 16-bit problem (host arithmetic)."""
    p = ctypes.c_int(-1)
    _call("aotk_gemm_path", M, N, K, sm_count, int(bool(with_workspace)), ctypes.byref(p))
    return PATHS[p.value]


def gemm_skinny(c, a, b, M, N, K, dtype, stream=None) -> None:
    _gemm("aotk_gemm_skinny", c, a, b, M, N, K, dtype, stream)


def gemm_silu_mul_workspace_size(M, I, K, dtype) -> int:
    n = ctypes.c_size_t(0)
    _call("aotk_gemm_silu_mul_workspace_size", M, I, K, dtype, ctypes.byref(n))
    return n.value


def gemm_silu_mul(act, a, b_gate_up, M, I, K, dtype, workspace=None, workspace_bytes=0,
                  stream=None) -> None:
    _call("aotk_gemm_silu_mul", _p(act), _p(a), _p(b_gate_up), M, I, K, dtype, _p(workspace),
          workspace_bytes, _stream(stream))


SCHEDULE_FIELDS = ("grid", "tiles", "full_rounds", "split_begin", "halves", "splits",
                   "kb_per_split", "units", "kblocks", "ws_bytes")


def gemm_schedule(M: int, N: int, K: int, elem_bytes: int, sm_count: int,
                  with_workspace: bool) -> dict:
    out = (ctypes.c_int64 * len(SCHEDULE_FIELDS))()
    _call("aotk_gemm_schedule", M, N, K, elem_bytes, sm_count, int(with_workspace), out)
    return dict(zip(SCHEDULE_FIELDS, list(out)))


def rmsnorm_rstd(rstd, x, rows: int, cols: int, eps: float, dtype: int, stream=None) -> None:
    _call("aotk_rmsnorm_rstd", _p(rstd), _p(x), rows, cols, eps, dtype, _stream(stream))


def gemm_silu_mul_rowscale(act, a, b_gate_up, row_scale, M, I, K, dtype, workspace=None,
                           workspace_bytes=0, stream=None) -> None:
    _call("aotk_gemm_silu_mul_rowscale", _p(act), _p(a), _p(b_gate_up), _p(row_scale), M, I, K,
          dtype, _p(workspace), workspace_bytes, _stream(stream))


def gemm_host_workspace_size(M, N, K, dtype) -> int:
    n = ctypes.c_size_t(0)
    _call("aotk_gemm_host_workspace_size", M, N, K, dtype, ctypes.byref(n))
    return n.value


def gemm_host(c_host, a_host, b_host, M, N, K, dtype, a_dev, b_dev, c_dev, workspace=None,
              workspace_bytes=0, stream=None) -> None:
    _call("aotk_gemm_host", _p(c_host), _p(a_host), _p(b_host), M, N, K, dtype, _p(a_dev),
          _p(b_dev), _p(c_dev), _p(workspace), workspace_bytes, _stream(stream))


def scaled_gemm_workspace_size(M, N, K, in_dtype) -> int:
    n = ctypes.c_size_t(0)
    _call("aotk_scaled_gemm_workspace_size", M, N, K, in_dtype, ctypes.byref(n))
    return n.value


def scaled_gemm(c, a, b, scale_a, scale_b, M, N, K, in_dtype, out_dtype, scale_mode,
                workspace=None, workspace_bytes=0, stream=None) -> None:
    _call("aotk_scaled_gemm", _p(c), _p(a), _p(b), _p(scale_a), _p(scale_b), M, N, K, in_dtype,
          out_dtype, scale_mode, _p(workspace), workspace_bytes, _stream(stream))


def scaled_gemm_tc(c, a, b, scale_a, scale_b, M, N, K, in_dtype, out_dtype, scale_mode,
                   workspace=None, workspace_bytes=0, stream=None) -> None:
    _call("aotk_scaled_gemm_tc", _p(c), _p(a), _p(b), _p(scale_a), _p(scale_b), M, N, K, in_dtype,
          out_dtype, scale_mode, _p(workspace), workspace_bytes, _stream(stream))


def scaled_gemm_simt(c, a, b, scale_a, scale_b, M, N, K, in_dtype, out_dtype, scale_mode,
                     stream=None) -> None:
    _call("aotk_scaled_gemm_simt", _p(c), _p(a), _p(b), _p(scale_a), _p(scale_b), M, N, K,
          in_dtype, out_dtype, scale_mode, _stream(stream))


def gemm_allreduce_tiles(M: int, N: int) -> int:
    n = ctypes.c_int64(0)
    _call("aotk_gemm_allreduce_tiles", M, N, ctypes.byref(n))
    return n.value


def gemm_allreduce(a, b, M, N, K, dtype, bufs: AllReduceBuffers, stream=None) -> None:
    _call("aotk_gemm_allreduce", _p(a), _p(b), M, N, K, dtype, ctypes.addressof(bufs),
          _stream(stream))


def watchdog_selftest(stream=None) -> None:
    _call("aotk_watchdog_selftest", _stream(stream))


def watchdog_status(device: int = 0, clear: bool = True) -> int:
    """Bit mask of tensor-core pipeline waits that timed out (0 = healthy)."""
    v = ctypes.c_uint32(0)
    _call("aotk_watchdog_status", device, ctypes.byref(v), 1 if clear else 0)
    return v.value
