"""Host runtime front end: contexts, argument descriptors and launch by entry name.

Mirror of the reference's shaders/spirv_runtime.py for the B200 backend:

* ``tensor_1d_descriptor`` / ``tensor_2d_descriptor`` build the same
  cutile_python_v1 argument lists (data, size, stride) and (data, dim0, dim1,
  stride0, stride1) as spirv_runtime.py:107-128;
* ``run_tile_kernel`` takes the place of ``run_spirv_kernel``
  (spirv_runtime.py:153-174): host arrays in, a named kernel, a dispatch,
  the requested output arrays back -- but the kernel is a registered sm_100a
  kernel reached through the C ABI instead of a SPIR-V module run by Kompute.
"""
from __future__ import annotations

import atexit
import ctypes
from typing import Iterable, Sequence

import numpy as np

from . import _native as N

LOCAL_SIZE_X = 1024  # invocations per workgroup of the reference's dispatches (lower.hpp:277-290)

_contexts: dict[int, int] = {}


def ceil_div(lhs: int, rhs: int) -> int:
    return (lhs + rhs - 1) // rhs


def device_count() -> int:
    n = ctypes.c_int32(0)
    N.check(N.lib().st_device_count(ctypes.byref(n)), "st_device_count")
    return n.value


def kernel_launches() -> int:
    """Kernels the native library has launched in this process so far."""
    n = ctypes.c_uint64(0)
    N.check(N.lib().st_kernel_launches(ctypes.byref(n)), "st_kernel_launches")
    return n.value


def context(device: int = 0) -> int:
    """The process-wide native context of one CUDA device (created on first use)."""
    ctx = _contexts.get(device)
    if ctx is None:
        handle = ctypes.c_void_p()
        devs = (ctypes.c_int32 * 1)(device)
        N.check(N.lib().st_init(devs, 1, ctypes.byref(handle)), f"st_init(device {device})")
        ctx = handle.value
        _contexts[device] = ctx
    return ctx


_group_contexts: dict[tuple[int, ...], int] = {}


def context_group(devices: Sequence[int]) -> int:
    """A process-wide native context over several CUDA devices (created on
    first use; peer access between them is enabled), for calls split over
    all of them (ST_EXEC_ALL_DEVICES)."""
    key = tuple(int(d) for d in devices)
    if not key:
        raise ValueError("devices must name at least one CUDA device")
    ctx = _group_contexts.get(key)
    if ctx is None:
        handle = ctypes.c_void_p()
        devs = (ctypes.c_int32 * len(key))(*key)
        N.check(N.lib().st_init(devs, len(key), ctypes.byref(handle)), f"st_init(devices {key})")
        ctx = handle.value
        _group_contexts[key] = ctx
    return ctx


def shutdown() -> None:
    for dev, ctx in list(_contexts.items()):
        N.lib().st_shutdown(ctx)
        del _contexts[dev]
    for key, ctx in list(_group_contexts.items()):
        N.lib().st_shutdown(ctx)
        del _group_contexts[key]


atexit.register(shutdown)


def sync(device: int = 0, timeout_ms: int = 60000) -> None:
    N.check(N.lib().st_sync(context(device), device, timeout_ms), "st_sync")


# ----------------------------------------------------------------- descriptors
def tensor_1d_descriptor(tensor: np.ndarray) -> list[np.ndarray]:
    """(data, size, stride) of a 1D array, as cutile_python_v1 binds it."""
    data = np.ascontiguousarray(tensor).reshape(-1)
    stride = data.strides[0] // data.itemsize
    return [data, np.array([data.shape[0]], dtype=np.int32), np.array([stride], dtype=np.int32)]


def tensor_2d_descriptor(tensor: np.ndarray) -> list[np.ndarray]:
    """(data, dim0, dim1, stride0, stride1) of a 2D array."""
    data = np.ascontiguousarray(tensor)
    dim0, dim1 = data.shape
    s0, s1 = (s // data.itemsize for s in data.strides)
    return [data.reshape(-1), np.array([dim0], dtype=np.int32), np.array([dim1], dtype=np.int32),
            np.array([s0], dtype=np.int32), np.array([s1], dtype=np.int32)]


def _np_dtype_code(a: np.ndarray) -> int:
    if a.dtype == np.float32:
        return N.ST_F32
    if a.dtype == np.float16:
        return N.ST_F16
    if a.dtype == np.uint16:  # bfloat16 bit patterns
        return N.ST_BF16
    raise ValueError(f"unsupported buffer dtype {a.dtype}")


def _is_scalar(a: np.ndarray) -> bool:
    return a.dtype == np.int32 and a.size == 1


def grid_from_dispatch(entry_name: str, dispatch: Sequence[int], tile_elems: int) -> tuple[int, int, int]:
    """cuda_tile grid of an entry from a reference dispatch of 1024-wide workgroups."""
    d = (ctypes.c_uint32 * 3)(*[int(x) for x in dispatch])
    g = N.StGrid()
    N.check(N.lib().st_grid_from_dispatch(entry_name.encode(), d, int(tile_elems), ctypes.byref(g)),
            "st_grid_from_dispatch")
    return (g.x, g.y, g.z)


def run_tile_kernel(*, entry_name: str | None = None, parameter_arrays: Iterable[np.ndarray],
                    output_indices: Iterable[int], dispatch: tuple[int, int, int] | None = None,
                    grid: tuple[int, int, int] | None = None, tile_elems: int | None = None, device: int = 0,
                    timeout_ms: int = 60000, spirv_path=None, module=None,
                    devices: Sequence[int] | None = None) -> list[np.ndarray]:
    """Run a registered kernel on host arrays and return the output arrays.

    Same contract as run_spirv_kernel (spirv_runtime.py:153-174): every
    parameter array is bound in order (1-element int32 arrays are the i32
    scalars of the cutile_python_v1 convention), the kernel runs once, and
    the arrays at ``output_indices`` come back as new numpy arrays.  Give
    either the cuda_tile ``grid`` or the reference's ``dispatch`` (1024-wide
    workgroups; converted with ``tile_elems``, default: the entry's tile).
    ``spirv_path`` is accepted for signature compatibility and ignored: the
    kernel is found by ``entry_name`` in the native registry.

    ``module`` (a .tilebc path, its bytes, or a ``TileModule``) takes the
    place of the SPIR-V module: ``entry_name`` (optional for a one-entry
    module) then names one of its entries, the bindings are checked against
    that entry's parameters, the module's tile sizes are the kernel
    constants, and ``tile_elems`` defaults to the module's tile.

    ``devices`` splits the launch over those GPUs in this process
    (ST_EXEC_ALL_DEVICES; vector_add and matmul entries): the region the
    grid covers is divided by element ranges or 128-row blocks.
    """
    arrays = [np.ascontiguousarray(a) for a in parameter_arrays]
    outs = [int(i) for i in output_indices]
    for i in outs:
        if not (0 <= i < len(arrays)) or _is_scalar(arrays[i]):
            raise ValueError(f"output index {i} does not name a buffer parameter")
    # outputs are written in place into private copies
    arrays = [a.copy() if i in outs else a for i, a in enumerate(arrays)]
    params = (N.StParam * len(arrays))()
    for i, a in enumerate(arrays):
        if _is_scalar(a):
            params[i].kind = N.ST_PARAM_I32
            params[i].value = int(a.reshape(-1)[0])
        else:
            params[i].kind = N.ST_PARAM_BUFFER
            params[i].dtype = _np_dtype_code(a)
            params[i].data = a.ctypes.data
            params[i].bytes = a.nbytes
    out_idx = (ctypes.c_int32 * len(outs))(*outs)
    ex = N.StExec(None, device, N.ST_EXEC_HOST_BUFFERS | N.ST_EXEC_SYNC, timeout_ms, out_idx, len(outs))
    ctx = context(device)
    if devices is not None:
        ex.device, ex.flags = -1, ex.flags | N.ST_EXEC_ALL_DEVICES
        ctx = context_group(devices)
    if module is not None:
        from .module import TileModule

        mod = module if isinstance(module, TileModule) else TileModule(module)
        ent = mod.entry(entry_name)
        if grid is None:
            if dispatch is None:
                raise ValueError("give the cuda_tile grid or the reference dispatch")
            if tile_elems is None:
                tile_elems = ent.tile_elems
            if tile_elems is None or ent.backend_entry is None:
                raise ValueError(f"entry {ent.name}: pass tile_elems or grid (the module does not fix its tile)")
            grid = grid_from_dispatch(ent.backend_entry, dispatch, tile_elems)
        mod.launch(ctx, ent.name, grid, params, ex)
        return [arrays[i] for i in outs]
    if entry_name is None:
        raise ValueError("entry_name is required without a module")
    if grid is None:
        if dispatch is None:
            raise ValueError("give the cuda_tile grid or the reference dispatch")
        if tile_elems is None:
            tile_elems = _default_tile_elems(entry_name)
        grid = grid_from_dispatch(entry_name, dispatch, tile_elems)
    g = N.StGrid(*[int(x) for x in grid])
    N.check(N.lib().st_launch(ctx, entry_name.encode(), ctypes.byref(g), params, len(arrays),
                              ctypes.byref(ex)), f"st_launch({entry_name})")
    return [arrays[i] for i in outs]


def _default_tile_elems(entry_name: str) -> int:
    if entry_name == "vector_add":
        return 1024
    if "matmul" in entry_name:
        tm, tn = (32, 32) if entry_name.endswith(("fp32", "fp32_bias")) else (128, 256)
        return tm * tn
    raise ValueError(f"no default tile for {entry_name!r}; pass tile_elems or grid")


# ----------------------------------------------------------------- policy
def tile_raster(m: int, n: int, tm: int, tn: int, group_m: int, bid: int) -> tuple[int, int]:
    bm, bn = ctypes.c_int64(), ctypes.c_int64()
    N.check(N.lib().st_tile_raster(m, n, tm, tn, group_m, bid, ctypes.byref(bm), ctypes.byref(bn)), "st_tile_raster")
    return bm.value, bn.value


def matmul_plan(in_dtype: int, m: int, n: int, k: int, sm_count: int = 148) -> dict:
    out = [ctypes.c_int32() for _ in range(5)]
    N.check(N.lib().st_matmul_plan(in_dtype, m, n, k, sm_count, *[ctypes.byref(o) for o in out]), "st_matmul_plan")
    return dict(zip(("block_m", "block_n", "block_k", "stages", "ctas"), (o.value for o in out)))


def stream_k_split(tiles: int, pairs: int, k_blocks: int) -> tuple[int, int, int]:
    """(dp_tiles, sk_pairs, sk_iters) of the CTA-pair kernel's work split."""
    dp, skp, ski = ctypes.c_int32(), ctypes.c_int32(), ctypes.c_int64()
    N.check(N.lib().st_stream_k_split(tiles, pairs, k_blocks, ctypes.byref(dp), ctypes.byref(skp), ctypes.byref(ski)),
            "st_stream_k_split")
    return dp.value, skp.value, ski.value


def shard_range(total: int, count: int, rank: int, align: int = 1) -> tuple[int, int]:
    b, e = ctypes.c_int64(), ctypes.c_int64()
    N.check(N.lib().st_shard_range(total, count, rank, align, ctypes.byref(b), ctypes.byref(e)), "st_shard_range")
    return b.value, e.value
