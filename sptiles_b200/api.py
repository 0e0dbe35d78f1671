"""Torch-facing operator API of the B200 backend.

Same names, argument meaning and error behaviour as the reference's Python
operators, so existing callers switch by changing an import:

* ``spirv_vector_add``     shaders/spirv_vector_add.py:44-92
* ``spirv_matmul``         shaders/spirv_matmul.py:48-98
* ``cutile_matmul_spirv``  shaders/spirv_matmul.py:101-113
* ``cutile_matmul``        shaders/matmul.py:181-253 (the cuTile host wrapper)

Device (CUDA) tensors are used in place on torch's current stream; host
tensors go through the C ABI's host-memory calls, which copy in, compute and
copy out (the reference routes every call through the CPU,
spirv_vector_add.py:37,89-92).  ``spirv_path`` is accepted and ignored: the
kernels are native sm_100a code selected by ``entry_name``.
"""
from __future__ import annotations

import ctypes
import struct
from pathlib import Path
from typing import Sequence

import torch

from . import _native as N
from .runtime import context, context_group

VECTOR_ADD_TILE_SIZE = 16  # spirv_vector_add.py:27
MATMUL_TILE_M = 32  # spirv_matmul.py:27
MATMUL_TILE_N = 32  # spirv_matmul.py:28

CUDA_STREAM_LEGACY = 0x1  # cudaStreamLegacy: the implicitly synchronising NULL stream

_CODES = {torch.float32: N.ST_F32, torch.float16: N.ST_F16, torch.bfloat16: N.ST_BF16}


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return _CODES[dtype]
    except KeyError:
        raise ValueError(f"unsupported dtype {dtype}") from None


def tensor_view(t: torch.Tensor) -> N.StTensor:
    """The C ABI view (data, dtype, rank, shape, strides) of a torch tensor."""
    if t.dim() not in (1, 2):
        raise ValueError("tensors must be rank 1 or 2")
    v = N.StTensor()
    v.data = t.data_ptr() if t.numel() else None
    v.dtype = dtype_code(t.dtype)
    v.rank = t.dim()
    for i in range(t.dim()):
        v.shape[i] = t.shape[i]
        v.strides[i] = t.stride(i)
    return v


def _det_flag() -> int:
    """ST_EXEC_DETERMINISTIC while torch.use_deterministic_algorithms(True) is in force."""
    return N.ST_EXEC_DETERMINISTIC if torch.are_deterministic_algorithms_enabled() else 0


def _exec_for(t: torch.Tensor, flags: int = 0) -> N.StExec:
    ex = N.StExec()
    ex.flags = flags | _det_flag()
    ex.timeout_ms = 60000
    if t.is_cuda:
        ex.device = t.device.index if t.device.index is not None else torch.cuda.current_device()
        handle = torch.cuda.current_stream(t.device).cuda_stream
        # torch's default stream is the legacy NULL stream; NULL would select
        # the context's own stream, so name it explicitly (cudaStreamLegacy)
        ex.stream = handle if handle else CUDA_STREAM_LEGACY
    else:  # host tensors: the process's current GPU (one rank per GPU), the context's own stream
        ex.device = torch.cuda.current_device() if torch.cuda.is_available() else 0
        ex.stream = None
    return ex


def _ctx(ex: N.StExec) -> int:
    return context(ex.device)


def _all_devices_exec() -> N.StExec:
    """st_exec of a call split over every device of its context (each on the context's stream)."""
    return N.StExec(None, -1, N.ST_EXEC_ALL_DEVICES | _det_flag(), 60000, None, 0)


# ----------------------------------------------------------------- lean calls
# CUDA tensors go to the same C ABI entry points with their st_tensor and
# st_exec descriptors packed by struct -- one C-level call per descriptor
# instead of field-by-field ctypes assignment, and torch's raw current
# stream instead of a Stream object: about 15 us less host time per call,
# most of what a 1024^3 fp32 matmul spends in Python.
_TENSOR_DESC = struct.Struct("@Pii2q2q")  # data, dtype, rank, shape[2], strides[2]
_EXEC_DESC = struct.Struct("@PiiIPi4x")  # stream, device, flags, timeout_ms, output_indices, n_outputs
assert _TENSOR_DESC.size == ctypes.sizeof(N.StTensor) and _EXEC_DESC.size == ctypes.sizeof(N.StExec)
_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)
_lean_fns: dict = {}


def _lean_fn(name: str, n_desc: int):
    """`name` from the native library, taking a context and `n_desc` descriptor pointers."""
    fn = _lean_fns.get(name)
    if fn is None:
        proto = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_void_p, *([ctypes.c_char_p] * n_desc))
        fn = _lean_fns[name] = proto((name, N.lib()))
    return fn


def _desc(t: torch.Tensor) -> bytes:
    """The st_tensor descriptor of `t`, packed (the bytes of tensor_view(t))."""
    shape, strides = t.shape, t.stride()
    code = _CODES.get(t.dtype)
    if code is None:
        raise ValueError(f"unsupported dtype {t.dtype}")
    if len(shape) == 2:
        return _TENSOR_DESC.pack(t.data_ptr() if shape[0] and shape[1] else 0, code, 2, shape[0], shape[1],
                                 strides[0], strides[1])
    if len(shape) == 1:
        return _TENSOR_DESC.pack(t.data_ptr() if shape[0] else 0, code, 1, shape[0], 0, strides[0], 0)
    raise ValueError("tensors must be rank 1 or 2")


def _exec_desc(device: int) -> bytes:
    """st_exec for torch's current stream on `device` (asynchronous, 60 s host waits)."""
    handle = _raw_stream(device) if _raw_stream is not None else torch.cuda.current_stream(device).cuda_stream
    return _EXEC_DESC.pack(handle or CUDA_STREAM_LEGACY, device, _det_flag(), 60000, 0, 0)


# ----------------------------------------------------------------- vector add
def vector_add(A: torch.Tensor, B: torch.Tensor, out: torch.Tensor | None = None, *,
               devices: Sequence[int] | None = None) -> torch.Tensor:
    """C = A + B (f32, rank 1 or 2, any strides), bit-exact IEEE adds.

    ``devices`` (host tensors only): split the add over those GPUs by element
    ranges, in this process (ST_EXEC_ALL_DEVICES).
    """
    if A.shape != B.shape:
        raise ValueError(f"Input tensors must have the same shape: {A.shape} != {B.shape}")
    dev = A.get_device()
    if B.get_device() != dev or A.device != B.device:
        raise ValueError("Input tensors must be on the same torch device.")
    C = out if out is not None else torch.empty(A.shape, dtype=A.dtype, device=A.device,
                                                 pin_memory=A.device.type == "cpu" and A.is_pinned())
    if devices is not None:
        if dev >= 0:
            raise ValueError("devices= splits calls on host tensors; CUDA tensors run on their own device")
        va, vb, vc = tensor_view(A), tensor_view(B), tensor_view(C)
        ex = _all_devices_exec()
        N.check(N.lib().st_vector_add_host(context_group(devices), ctypes.byref(va), ctypes.byref(vb),
                                           ctypes.byref(vc), ctypes.byref(ex)), "vector_add")
        return C
    if dev >= 0:
        rc = _lean_fn("st_vector_add", 4)(context(dev), _desc(A), _desc(B), _desc(C), _exec_desc(dev))
        if rc != N.ST_OK:
            N.check(rc, "vector_add")
        return C
    ex = _exec_for(A)
    va, vb, vc = tensor_view(A), tensor_view(B), tensor_view(C)
    fn = N.lib().st_vector_add if A.is_cuda else N.lib().st_vector_add_host
    N.check(fn(_ctx(ex), ctypes.byref(va), ctypes.byref(vb), ctypes.byref(vc), ctypes.byref(ex)), "vector_add")
    return C


def spirv_vector_add(A: torch.Tensor, B: torch.Tensor, *, spirv_path: str | Path | None = None,
                     entry_name: str = "vector_add") -> torch.Tensor:
    """Drop-in for the reference's spirv_vector_add (spirv_vector_add.py:44-92).

    Checks the same preconditions with the same messages (equal shapes, same
    device, 1D float32, size divisible by the exported tile size 16) and
    returns the sum on the inputs' device.
    """
    if A.shape != B.shape:
        raise ValueError(f"Input tensors must have the same shape: {A.shape} != {B.shape}")
    if A.device != B.device:
        raise ValueError("Input tensors must be on the same torch device.")
    for t, name in ((A, "A"), (B, "B")):
        if t.ndim != 1:
            raise ValueError(f"{name} must be a 1D tensor.")
        if t.dtype != torch.float32:
            raise ValueError(f"{name} must be torch.float32; the current SPIR-V lowering is f32-only.")
    if entry_name != "vector_add":
        raise ValueError(f"Entry point {entry_name!r} was not found in the SPIR-V module.")
    element_count = A.shape[0]
    if element_count % VECTOR_ADD_TILE_SIZE != 0:
        raise ValueError(f"vector_add expects a size divisible by {VECTOR_ADD_TILE_SIZE}; got {element_count}.")
    return vector_add(A, B)


def vector_fma(A: torch.Tensor, B: torch.Tensor, D: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """C = A * B + D elementwise with one rounding (f32 CUDA tensors, rank 1 or 2, any strides).

    The lowering's `fma` (tileops.hpp:616-623, GLSL.std.450 Fma) as a fused
    IEEE multiply-add.
    """
    if not (A.shape == B.shape == D.shape):
        raise ValueError(f"Input tensors must have the same shape: {A.shape}, {B.shape}, {D.shape}")
    if not (A.device == B.device == D.device) or not A.is_cuda:
        raise ValueError("Input tensors must be on the same CUDA device.")
    C = out if out is not None else torch.empty(A.shape, dtype=A.dtype, device=A.device)
    ex = _exec_for(A)
    va, vb, vd, vc = tensor_view(A), tensor_view(B), tensor_view(D), tensor_view(C)
    N.check(N.lib().st_vector_fma(_ctx(ex), ctypes.byref(va), ctypes.byref(vb), ctypes.byref(vd), ctypes.byref(vc),
                                  ctypes.byref(ex)), "vector_fma")
    return C


def cast(A: torch.Tensor, dtype: torch.dtype, out: torch.Tensor | None = None) -> torch.Tensor:
    """A converted to ``dtype`` (float32 / float16 / bfloat16) on the GPU, round to nearest even.

    The lowering's `ftof` (tileops.hpp:257-258), which the f32-only
    reference passes through unchanged.
    """
    if not A.is_cuda:
        raise ValueError("Input tensor must be on a CUDA device.")
    C = out if out is not None else torch.empty(A.shape, dtype=dtype, device=A.device)
    ex = _exec_for(A)
    va, vc = tensor_view(A), tensor_view(C)
    N.check(N.lib().st_cast(_ctx(ex), ctypes.byref(va), ctypes.byref(vc), ctypes.byref(ex)), "cast")
    return C


# ----------------------------------------------------------------- matmul
def matmul(A: torch.Tensor, B: torch.Tensor, bias: torch.Tensor | None = None, *,
           out_dtype: torch.dtype | None = None, out: torch.Tensor | None = None,
           devices: Sequence[int] | None = None) -> torch.Tensor:
    """C = A @ B (+ bias) with fp32 accumulation on the tensor cores.

    A, B: both float32 (3xTF32), both float16 or both bfloat16.  C defaults
    to A's dtype (matmul.py:245); ``out_dtype`` may ask for float32, float16
    or bfloat16.  bias (length N) is float32 or A's dtype.  ``devices`` (host
    tensors only): split the call over those GPUs by 128-row blocks of A and
    C, in this process (ST_EXEC_ALL_DEVICES).
    """
    sa, sb = A.shape, B.shape
    if len(sa) != 2 or len(sb) != 2:
        raise ValueError("A and B must be 2D tensors.")
    if sa[1] != sb[0]:
        raise ValueError(f"Incompatible matrices: K dimension of A ({sa[1]}) "
                         f"must match K dimension of B ({sb[0]})")
    dev = A.get_device()
    if B.get_device() != dev or (bias is not None and bias.get_device() != dev):
        raise ValueError("Input tensors must be on the same device.")
    if A.dtype != B.dtype:
        raise ValueError(f"A and B must have the same dtype ({A.dtype} != {B.dtype})")
    if out is None:
        out = torch.empty((sa[0], sb[1]), dtype=out_dtype or A.dtype, device=A.device,
                          pin_memory=dev < 0 and A.device.type == "cpu" and A.is_pinned())
    if devices is not None:
        if dev >= 0:
            raise ValueError("devices= splits calls on host tensors; CUDA tensors run on their own device")
        va, vb, vc = tensor_view(A), tensor_view(B), tensor_view(out)
        vbias = ctypes.byref(tensor_view(bias)) if bias is not None else None
        ex = _all_devices_exec()
        N.check(N.lib().st_matmul_host(context_group(devices), ctypes.byref(va), ctypes.byref(vb), vbias,
                                       ctypes.byref(vc), ctypes.byref(ex)), "matmul")
        return out
    if dev >= 0:
        rc = _lean_fn("st_matmul", 5)(context(dev), _desc(A), _desc(B), None if bias is None else _desc(bias),
                                      _desc(out), _exec_desc(dev))
        if rc != N.ST_OK:
            N.check(rc, "matmul")
        return out
    if A.device != B.device or (bias is not None and bias.device != A.device):
        raise ValueError("Input tensors must be on the same device.")
    ex = _exec_for(A)
    va, vb, vc = tensor_view(A), tensor_view(B), tensor_view(out)
    vbias = ctypes.byref(tensor_view(bias)) if bias is not None else None
    fn = N.lib().st_matmul if A.is_cuda else N.lib().st_matmul_host
    N.check(fn(_ctx(ex), ctypes.byref(va), ctypes.byref(vb), vbias, ctypes.byref(vc), ctypes.byref(ex)), "matmul")
    return out


def _check_spirv_matmul_args(A: torch.Tensor, B: torch.Tensor) -> None:
    if A.shape[1] != B.shape[0]:
        raise ValueError(f"Incompatible matrices: K dimension of A ({A.shape[1]}) "
                         f"must match K dimension of B ({B.shape[0]})")
    if A.device != B.device:
        raise ValueError("Input tensors must be on the same torch device.")
    for t, name in ((A, "A"), (B, "B")):
        if t.ndim != 2:
            raise ValueError(f"{name} must be a 2D tensor.")
        if t.dtype != torch.float32:
            raise ValueError(f"{name} must be torch.float32; the current SPIR-V lowering is f32-only.")


def spirv_matmul(A: torch.Tensor, B: torch.Tensor, *, spirv_path: str | Path | None = None,
                 entry_name: str = "matmul_fp32") -> torch.Tensor:
    """Drop-in for the reference's spirv_matmul (spirv_matmul.py:48-98): fp32 C = A @ B."""
    _check_spirv_matmul_args(A, B)
    if entry_name not in ("matmul_fp32", "persistent_matmul_fp32"):
        raise ValueError(f"Entry point {entry_name!r} was not found in the SPIR-V module.")
    return matmul(A, B)


def cutile_matmul_spirv(A: torch.Tensor, B: torch.Tensor, persistent: bool = False, *,
                        spirv_path: str | Path | None = None, entry_name: str = "matmul_fp32") -> torch.Tensor:
    """Drop-in for cutile_matmul_spirv (spirv_matmul.py:101-113).

    The reference raises NotImplementedError for ``persistent=True``; here
    the tensor-core kernel is persistent in every case, so both forms run and
    give the same result.
    """
    return spirv_matmul(A, B, spirv_path=spirv_path,
                        entry_name="persistent_matmul_fp32" if persistent else entry_name)


def cutile_matmul(A: torch.Tensor, B: torch.Tensor, persistent: bool = False, *,
                  bias: torch.Tensor | None = None, out_dtype: torch.dtype | None = None) -> torch.Tensor:
    """Drop-in for the cuTile host wrapper cutile_matmul (matmul.py:181-253).

    Same validation (K match, same device, CUDA tensors) and the same output
    dtype rule (C takes A's dtype, matmul.py:245) unless ``out_dtype`` says
    otherwise; tile shapes are chosen by the native runtime.
    """
    if A.shape[1] != B.shape[0]:
        raise ValueError(f"Incompatible matrices: K dimension of A ({A.shape[1]}) "
                         f"must match K dimension of B ({B.shape[0]})")
    if A.device != B.device:
        raise ValueError("Input tensors must be on the same device.")
    if not A.is_cuda or not B.is_cuda:
        raise ValueError("Input tensors must be on a CUDA device.")
    return matmul(A, B, bias, out_dtype=out_dtype)
