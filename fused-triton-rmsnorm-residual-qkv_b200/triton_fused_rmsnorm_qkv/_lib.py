"""ctypes binding of ``libfqkv.so`` (C ABI declared in ``include/fused_rmsnorm_qkv.h``).

The library is built in-tree by ``build.py`` next to this file.  Loading it never
falls back to anything else: if the shared object is missing the import of the GPU
entry points raises, with the build command in the message.

Error mapping of ``fqkv_launch`` return codes:
  FQKV_ERR_DTYPE -> TypeError, other codes > 0 -> ValueError, codes < 0 (CUDA
  runtime errors) -> RuntimeError.  The message is ``fqkv_last_error()``.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

# Constants mirrored from include/fused_rmsnorm_qkv.h.
F16, BF16, F32 = 0, 1, 2
SCHED_AUTO, SCHED_SIMT, SCHED_DECODE, SCHED_SPLIT, SCHED_PREFILL, SCHED_GRID = -1, 0, 1, 2, 3, 4
FLAG_PDL, FLAG_STATIC_WEIGHTS, FLAG_TEST_WITHHOLD = 1, 2, 4
ERR_NULL, ERR_SHAPE, ERR_DTYPE, ERR_ALIGN, ERR_WORKSPACE, ERR_SCHEDULE, ERR_DEVICE, ERR_DEVICE_TIMEOUT, ERR_ALIAS = (
    1, 2, 3, 4, 5, 6, 7, 8, 9)
STATUS_WAIT_TIMEOUT = 1

SCHEDULE_NAMES = {SCHED_SIMT: "simt", SCHED_DECODE: "decode", SCHED_SPLIT: "split", SCHED_PREFILL: "prefill",
                  SCHED_GRID: "grid"}
SCHEDULE_BY_NAME = {v: k for k, v in SCHEDULE_NAMES.items()}
SCHEDULE_BY_NAME["auto"] = SCHED_AUTO
SCHEDULE_BY_NAME["naive"] = SCHED_SIMT

LIB_PATH = Path(__file__).resolve().parent / "libfqkv.so"

EXPORTED_SYMBOLS = (
    "fqkv_launch",
    "fqkv_launch_noalloc",
    "fqkv_launch_fp8w",
    "fqkv_rope_split",
    "fqkv_launch_rope",
    "fqkv_workspace_bytes",
    "fqkv_query_schedule",
    "fqkv_last_error",
    "fqkv_device_status",
    "fqkv_stream_capture_id",
    "fqkv_test_set_wait_limit_ns",
    "fqkv_version",
)


class ScheduleInfo(ctypes.Structure):
    """``fqkv_schedule_info``."""

    _fields_ = [(name, ctypes.c_int32) for name in (
        "schedule", "block_m", "block_n", "block_k", "stages", "split_k", "grid", "threads",
        "smem_bytes", "uses_prepass")]

    def as_dict(self) -> dict:
        return {name: getattr(self, name) for name, _ in self._fields_}


_lib = None
# CPython fast path for fqkv_launch (csrc/fqkv_pycall.c, built by build.py); ctypes otherwise.
try:
    from . import _fqkv_pycall as _pycall
except ImportError:
    _pycall = None


def load() -> ctypes.CDLL:
    """Load (once) and return the library, declaring every entry point's signature."""
    global _lib
    if _lib is not None:
        return _lib
    path = Path(os.environ.get("FQKV_LIB", LIB_PATH))
    if not path.exists():
        raise RuntimeError(
            f"{path} is missing: build the CUDA library first "
            f"(python {Path(__file__).resolve().parent.parent / 'build.py'})")
    lib = ctypes.CDLL(str(path))
    i64, i32, vp, f32 = ctypes.c_int64, ctypes.c_int, ctypes.c_void_p, ctypes.c_float
    lib.fqkv_launch.argtypes = [vp, vp, vp, i32, vp, vp, vp, i64, i64, i64, i64, i64, i64, i64, i64, f32, i32,
                                i32, i32, vp, i64, vp]
    lib.fqkv_launch.restype = i32
    lib.fqkv_workspace_bytes.argtypes = [i64, i64, i64, i32, i32]
    lib.fqkv_workspace_bytes.restype = i64
    lib.fqkv_query_schedule.argtypes = [i64, i64, i64, i32, i32, ctypes.POINTER(ScheduleInfo)]
    lib.fqkv_query_schedule.restype = i32
    lib.fqkv_last_error.argtypes = []
    lib.fqkv_last_error.restype = ctypes.c_char_p
    lib.fqkv_device_status.argtypes = [vp, ctypes.POINTER(ctypes.c_int)]
    lib.fqkv_device_status.restype = i32
    lib.fqkv_test_set_wait_limit_ns.argtypes = [ctypes.c_ulonglong]
    lib.fqkv_test_set_wait_limit_ns.restype = i32
    lib.fqkv_stream_capture_id.argtypes = [vp, ctypes.POINTER(ctypes.c_ulonglong)]
    lib.fqkv_stream_capture_id.restype = i32
    lib.fqkv_version.argtypes = []
    lib.fqkv_version.restype = i32
    lib.fqkv_launch_fp8w.argtypes = [vp, vp, vp, i32, vp, vp, vp, vp, i64, i64, i64, i64, i64, i64, i64, i64, f32,
                                     i32, i32, vp]
    lib.fqkv_launch_fp8w.restype = i32
    lib.fqkv_rope_split.argtypes = [vp, i64, vp, vp, i64, vp, vp, vp, i64, i64, i32, i32, i32, i32, vp]
    lib.fqkv_rope_split.restype = i32
    lib.fqkv_launch_rope.argtypes = [vp, vp, vp, i32, vp, vp, vp, vp, vp, i64, i64, i64, i64, i64, i64, i64, vp, vp,
                                     i64, i32, i32, i32, f32, i32, i32, vp]
    lib.fqkv_launch_rope.restype = i32
    if _pycall is not None:
        _pycall.set_launch(ctypes.cast(lib.fqkv_launch, ctypes.c_void_p).value)
    _lib = lib
    return lib


def last_error() -> str:
    return load().fqkv_last_error().decode(errors="replace")


def check(rc: int, what: str = "fqkv_launch") -> None:
    """Raise the Python exception matching a C-ABI return code."""
    if rc == 0:
        return
    msg = f"{what}: {last_error()} (code {rc})"
    if rc == ERR_DTYPE:
        raise TypeError(msg)
    if rc > 0:
        raise ValueError(msg)
    raise RuntimeError(msg)


def launch(x_ptr, r_ptr, g_ptr, g_dtype, w_ptr, out_ptr, rout_ptr, M, H, N, ldx, ldr, ldw, ldo, ldro, eps,
           dtype, schedule, flags, ws_ptr, ws_bytes, stream) -> int:
    lib = _lib if _lib is not None else load()
    if _pycall is not None:  # the same library call, its arguments converted by the CPython module
        return _pycall.launch(x_ptr, r_ptr, g_ptr, g_dtype, w_ptr, out_ptr, rout_ptr, M, H, N, ldx, ldr, ldw, ldo,
                              ldro, eps, dtype, schedule, flags, ws_ptr, ws_bytes, stream)
    return lib.fqkv_launch(x_ptr, r_ptr, g_ptr, g_dtype, w_ptr, out_ptr, rout_ptr, M, H, N, ldx, ldr, ldw,
                           ldo, ldro, ctypes.c_float(eps), dtype, schedule, flags, ws_ptr, ws_bytes, stream)


def launch_fp8w(x_ptr, r_ptr, g_ptr, g_dtype, w_ptr, scale_ptr, out_ptr, rout_ptr, M, H, N, ldx, ldr, ldw, ldo,
                ldro, eps, dtype, flags, stream) -> int:
    return load().fqkv_launch_fp8w(x_ptr, r_ptr, g_ptr, g_dtype, w_ptr, scale_ptr, out_ptr, rout_ptr, M, H, N, ldx,
                                   ldr, ldw, ldo, ldro, ctypes.c_float(eps), dtype, flags, stream)


def rope_split(qkv_ptr, ldq, cos_ptr, sin_ptr, cos_batch, q_ptr, k_ptr, v_ptr, B, S, n_q, n_kv, head_dim,
               dtype, stream) -> int:
    return load().fqkv_rope_split(qkv_ptr, ldq, cos_ptr, sin_ptr, cos_batch, q_ptr, k_ptr, v_ptr, B, S, n_q, n_kv,
                                  head_dim, dtype, stream)


def set_wait_limit_ns(ns: int) -> None:
    """Tests of the failure path: the bounded-wait limit of kernels launched from now on
    (current device); 0 restores the default of 1 s."""
    check(load().fqkv_test_set_wait_limit_ns(ns), "fqkv_test_set_wait_limit_ns")


def stream_capture_id(stream: int) -> int:
    """Id of the capture active on ``stream``, or 0 when it is not being captured."""
    cid = ctypes.c_ulonglong(0)
    check(load().fqkv_stream_capture_id(stream, ctypes.byref(cid)), "fqkv_stream_capture_id")
    return cid.value


def launch_rope(x_ptr, r_ptr, g_ptr, g_dtype, w_ptr, q_ptr, k_ptr, v_ptr, rout_ptr, B, S, H, ldx, ldr, ldw, ldro,
                cos_ptr, sin_ptr, cos_batch, n_q, n_kv, head_dim, eps, dtype, flags, stream) -> int:
    return load().fqkv_launch_rope(x_ptr, r_ptr, g_ptr, g_dtype, w_ptr, q_ptr, k_ptr, v_ptr, rout_ptr, B, S, H, ldx,
                                   ldr, ldw, ldro, cos_ptr, sin_ptr, cos_batch, n_q, n_kv, head_dim,
                                   ctypes.c_float(eps), dtype, flags, stream)


def workspace_bytes(M: int, H: int, N: int, dtype: int, schedule: int) -> int:
    n = load().fqkv_workspace_bytes(M, H, N, dtype, schedule)
    if n < 0:
        check(-n, "fqkv_workspace_bytes")
    return n


def query_schedule(M: int, H: int, N: int, dtype: int, schedule: int = SCHED_AUTO) -> dict:
    info = ScheduleInfo()
    check(load().fqkv_query_schedule(M, H, N, dtype, schedule, ctypes.byref(info)), "fqkv_query_schedule")
    return info.as_dict()


def device_status(stream: int) -> int:
    v = ctypes.c_int(0)
    check(load().fqkv_device_status(stream, ctypes.byref(v)), "fqkv_device_status")
    return v.value


def version() -> int:
    return load().fqkv_version()
