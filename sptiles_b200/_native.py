"""ctypes binding of the C ABI declared in include/sptiles_b200.h.

The library (libsptiles_b200.so, built in-tree by ``sptiles_b200.build``) is
the only compute path: if it is missing or cannot be loaded, every call
raises -- there is no Python or CPU fallback.
"""
from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

_PKG = Path(__file__).resolve().parent
LIB_PATH = _PKG / "libsptiles_b200.so"

ST_OK = 0
ST_ERR_INVALID_ARGUMENT = 1
ST_ERR_UNKNOWN_ENTRY = 2
ST_ERR_UNSUPPORTED = 3
ST_ERR_CUDA = 4
ST_ERR_NO_DEVICE = 5
ST_ERR_OUT_OF_MEMORY = 6
ST_ERR_TIMEOUT = 7
ST_ERR_DEVICE_ABORT = 8

ST_F32, ST_F16, ST_BF16, ST_I32 = 0, 1, 2, 3
ST_PARAM_BUFFER, ST_PARAM_I32 = 0, 1
ST_MODULE_PARAM_BUFFER, ST_MODULE_PARAM_I32, ST_MODULE_PARAM_OTHER = 0, 1, 2
ST_EXEC_SYNC, ST_EXEC_HOST_BUFFERS, ST_EXEC_DETERMINISTIC, ST_EXEC_ALL_DEVICES = 1, 2, 4, 8

# Every symbol the header declares; the CPU test suite checks the library exports them all.
EXPORTED = (
    "st_version", "st_last_error", "st_device_count", "st_kernel_launches", "st_init", "st_shutdown", "st_sync", "st_stream",
    "st_alloc", "st_free", "st_upload", "st_download", "st_launch", "st_grid_from_dispatch",
    "st_vector_add", "st_matmul", "st_vector_add_host", "st_matmul_host", "st_tile_raster",
    "st_matmul_plan", "st_stream_k_split", "st_shard_range", "st_matmul_static_scratch", "st_vector_fma", "st_cast",
    "st_ipc_handle", "st_ipc_open", "st_ipc_close", "st_matmul_allgather",
    "st_module_load", "st_module_load_file", "st_module_free", "st_module_version", "st_module_entry_count",
    "st_module_entry", "st_module_param", "st_launch_module", "st_check_device_wait",
)


class StParam(ctypes.Structure):
    _fields_ = [("kind", ctypes.c_int32), ("dtype", ctypes.c_int32), ("data", ctypes.c_void_p),
                ("bytes", ctypes.c_uint64), ("value", ctypes.c_int64)]


class StTensor(ctypes.Structure):
    _fields_ = [("data", ctypes.c_void_p), ("dtype", ctypes.c_int32), ("rank", ctypes.c_int32),
                ("shape", ctypes.c_int64 * 2), ("strides", ctypes.c_int64 * 2)]


class StGrid(ctypes.Structure):
    _fields_ = [("x", ctypes.c_uint32), ("y", ctypes.c_uint32), ("z", ctypes.c_uint32)]


class StExec(ctypes.Structure):
    _fields_ = [("stream", ctypes.c_void_p), ("device", ctypes.c_int32), ("flags", ctypes.c_int32),
                ("timeout_ms", ctypes.c_uint32), ("output_indices", ctypes.POINTER(ctypes.c_int32)),
                ("n_outputs", ctypes.c_int32)]


class StModuleEntryInfo(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char_p), ("n_params", ctypes.c_int32), ("n_arrays", ctypes.c_int32),
                ("array_rank", ctypes.c_int32 * 8), ("array_dtype", ctypes.c_int32 * 8),
                ("n_constants", ctypes.c_int32), ("constants", ctypes.c_int32 * 3),
                ("num_cta_in_cga", ctypes.c_int32), ("occupancy", ctypes.c_int32),
                ("backend_entry", ctypes.c_char_p)]


class NativeError(RuntimeError):
    """A failed call into the native library; ``code`` is the ST_* status."""

    def __init__(self, code: int, message: str):
        super().__init__(message)
        self.code = code


class DeviceAbort(NativeError):
    """A kernel gave up one of its bounded on-device waits."""


_lib = None
_lock = threading.Lock()

_P = ctypes.POINTER
_c = ctypes


def _declare(L: ctypes.CDLL) -> None:
    vp, i32, i64, u32, u64 = _c.c_void_p, _c.c_int32, _c.c_int64, _c.c_uint32, _c.c_uint64
    sig = {
        "st_version": ([], _c.c_char_p),
        "st_last_error": ([], _c.c_char_p),
        "st_device_count": ([_P(i32)], _c.c_int),
        "st_kernel_launches": ([_P(u64)], _c.c_int),
        "st_init": ([_P(i32), i32, _P(vp)], _c.c_int),
        "st_shutdown": ([vp], _c.c_int),
        "st_sync": ([vp, i32, u32], _c.c_int),
        "st_stream": ([vp, i32, _P(vp)], _c.c_int),
        "st_alloc": ([vp, i32, u64, _P(vp)], _c.c_int),
        "st_free": ([vp, i32, vp], _c.c_int),
        "st_upload": ([vp, i32, vp, vp, u64], _c.c_int),
        "st_download": ([vp, i32, vp, vp, u64], _c.c_int),
        "st_launch": ([vp, _c.c_char_p, _P(StGrid), _P(StParam), i32, _P(StExec)], _c.c_int),
        "st_grid_from_dispatch": ([_c.c_char_p, _P(u32), i64, _P(StGrid)], _c.c_int),
        "st_vector_add": ([vp, _P(StTensor), _P(StTensor), _P(StTensor), _P(StExec)], _c.c_int),
        "st_matmul": ([vp, _P(StTensor), _P(StTensor), _P(StTensor), _P(StTensor), _P(StExec)], _c.c_int),
        "st_vector_add_host": ([vp, _P(StTensor), _P(StTensor), _P(StTensor), _P(StExec)], _c.c_int),
        "st_matmul_host": ([vp, _P(StTensor), _P(StTensor), _P(StTensor), _P(StTensor), _P(StExec)], _c.c_int),
        "st_vector_fma": ([vp, _P(StTensor), _P(StTensor), _P(StTensor), _P(StTensor), _P(StExec)], _c.c_int),
        "st_cast": ([vp, _P(StTensor), _P(StTensor), _P(StExec)], _c.c_int),
        "st_ipc_handle": ([vp, i32, vp, _P(_c.c_uint8)], _c.c_int),
        "st_ipc_open": ([vp, i32, _P(_c.c_uint8), _P(vp)], _c.c_int),
        "st_ipc_close": ([vp, i32, vp], _c.c_int),
        "st_matmul_allgather": ([vp, _P(StTensor), _P(StTensor), _P(StTensor), _P(StTensor), _P(vp), i32, i64,
                                 _P(StExec)], _c.c_int),
        "st_tile_raster": ([i64, i64, i64, i64, i64, i64, _P(i64), _P(i64)], _c.c_int),
        "st_matmul_plan": ([i32, i64, i64, i64, i32, _P(i32), _P(i32), _P(i32), _P(i32), _P(i32)], _c.c_int),
        "st_stream_k_split": ([i32, i32, i32, _P(i32), _P(i32), _P(i64)], _c.c_int),
        "st_shard_range": ([i64, i32, i32, i64, _P(i64), _P(i64)], _c.c_int),
        "st_matmul_static_scratch": ([_P(StTensor), _P(StTensor), _P(StTensor), _P(StTensor), _P(StExec)],
                                     _c.c_int),
        "st_check_device_wait": ([vp, i32, u32, _P(StExec)], _c.c_int),
        "st_module_load": ([vp, u64, _P(vp)], _c.c_int),
        "st_module_load_file": ([_c.c_char_p, _P(vp)], _c.c_int),
        "st_module_free": ([vp], _c.c_int),
        "st_module_version": ([vp, _P(i32), _P(i32), _P(i32)], _c.c_int),
        "st_module_entry_count": ([vp, _P(i32)], _c.c_int),
        "st_module_entry": ([vp, i32, _P(StModuleEntryInfo)], _c.c_int),
        "st_module_param": ([vp, i32, i32, _P(i32), _P(i32)], _c.c_int),
        "st_launch_module": ([vp, vp, _c.c_char_p, _P(StGrid), _P(StParam), i32, _P(StExec)], _c.c_int),
    }
    for name, (args, res) in sig.items():
        fn = getattr(L, name)
        fn.argtypes = args
        fn.restype = res


def lib() -> ctypes.CDLL:
    """The loaded native library.  Raises if it was not built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            path = Path(os.environ.get("SPTILES_B200_LIB", LIB_PATH))
            if not path.exists():
                raise RuntimeError(
                    f"native library {path} is missing: build it with `python -m sptiles_b200.build` "
                    "(there is no fallback path)")
            L = ctypes.CDLL(str(path))
            _declare(L)
            _lib = L
    return _lib


def last_error() -> str:
    msg = lib().st_last_error()
    return msg.decode() if msg else ""


def check(code: int, what: str = "") -> None:
    """Raise the Python exception that matches an ST_* status."""
    if code == ST_OK:
        return
    msg = last_error() or f"status {code}"
    if what:
        msg = f"{what}: {msg}"
    if code in (ST_ERR_INVALID_ARGUMENT, ST_ERR_UNKNOWN_ENTRY):
        raise ValueError(msg)
    if code == ST_ERR_UNSUPPORTED:
        raise NotImplementedError(msg)
    if code == ST_ERR_TIMEOUT:
        raise TimeoutError(msg)
    if code == ST_ERR_OUT_OF_MEMORY:
        raise MemoryError(msg)
    if code == ST_ERR_DEVICE_ABORT:
        raise DeviceAbort(code, msg)
    raise NativeError(code, msg)
