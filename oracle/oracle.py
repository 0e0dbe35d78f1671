"""ctypes front end of the C oracle (oracle.c) -- test infrastructure only.

Every function here takes and returns numpy arrays.  fp16 inputs are numpy
float16 arrays; bf16 inputs are numpy uint16 arrays holding bfloat16 bit
patterns (numpy has no bfloat16 type).
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import time
from pathlib import Path

import numpy as np

__all__ = [
    "F32", "F16", "BF16",
    "lib", "vector_add_1d", "vector_add_2d", "matmul", "reference_matmul_f32",
    "f32_to_bf16_bits", "bf16_bits_to_f32", "f32_to_f16_bits", "f16_bits_to_f32",
    "kat_values", "kat_iota", "matmul_kat_expected", "time_matmul_rows",
    "time_vector_add", "vector_fma_1d", "cast",
]

F32, F16, BF16 = 0, 1, 2

_HERE = Path(__file__).resolve().parent
_LIB_PATH = _HERE / "liboracle.so"
_lib = None

_i64 = ctypes.c_int64
_vp = ctypes.c_void_p
_i64p = ctypes.POINTER(ctypes.c_int64)


def _build() -> None:
    subprocess.run(["make", "-s", "-C", str(_HERE)], check=True)


def lib() -> ctypes.CDLL:
    """Load (building first if needed) liboracle.so."""
    global _lib
    if _lib is not None:
        return _lib
    src = _HERE / "oracle.c"
    if not _LIB_PATH.exists() or (src.exists() and src.stat().st_mtime > _LIB_PATH.stat().st_mtime):
        _build()
    L = ctypes.CDLL(str(_LIB_PATH))
    L.or_vector_add_1d.argtypes = [_vp, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _i64, _i64, _i64]
    L.or_vector_add_1d.restype = ctypes.c_int
    L.or_vector_add_2d.argtypes = [_vp, _i64p, _i64p, _vp, _i64p, _i64p, _vp, _i64p, _i64p,
                                   _i64, _i64, _i64, _i64]
    L.or_vector_add_2d.restype = ctypes.c_int
    L.or_matmul.argtypes = [ctypes.c_int, _vp, _i64, _i64, _vp, _i64, _i64, ctypes.c_int, _vp,
                            ctypes.c_int, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _i64, ctypes.c_int]
    L.or_matmul.restype = ctypes.c_int
    L.or_reference_matmul_f32.argtypes = [_vp, _vp, _vp, _i64, _i64, _i64]
    L.or_reference_matmul_f32.restype = ctypes.c_int
    L.or_first_mismatch_abs.argtypes = [_vp, _vp, _i64, ctypes.c_float]
    L.or_first_mismatch_abs.restype = ctypes.c_int64
    L.or_kat_values.argtypes = [_vp, _i64, _i64, _i64, ctypes.c_float]
    L.or_kat_values.restype = None
    L.or_kat_iota.argtypes = [_vp, _i64, _i64]
    L.or_kat_iota.restype = None
    L.or_vector_fma_1d.argtypes = [_vp, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _i64, _i64, _i64]
    L.or_vector_fma_1d.restype = ctypes.c_int
    L.or_cast.argtypes = [ctypes.c_int, _vp, _i64, ctypes.c_int, _vp, _i64, _i64]
    L.or_cast.restype = ctypes.c_int
    L.or_f16_to_f32.argtypes = [ctypes.c_uint16]
    L.or_f16_to_f32.restype = ctypes.c_float
    L.or_bf16_to_f32.argtypes = [ctypes.c_uint16]
    L.or_bf16_to_f32.restype = ctypes.c_float
    L.or_f32_to_f16.argtypes = [ctypes.c_float]
    L.or_f32_to_f16.restype = ctypes.c_uint16
    L.or_f32_to_bf16.argtypes = [ctypes.c_float]
    L.or_f32_to_bf16.restype = ctypes.c_uint16
    _lib = L
    return L


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


def _estrides(a: np.ndarray) -> tuple[int, ...]:
    return tuple(s // a.itemsize for s in a.strides)


def vector_add_1d(a: np.ndarray, b: np.ndarray, c: np.ndarray, tile: int, grid_tiles: int) -> np.ndarray:
    """C[i] = A[i] + B[i] for i < min(grid_tiles*tile, C.size); C is updated in place."""
    for x in (a, b, c):
        assert x.dtype == np.float32 and x.ndim == 1
    rc = lib().or_vector_add_1d(_ptr(a), a.shape[0], _estrides(a)[0], _ptr(b), b.shape[0], _estrides(b)[0],
                                _ptr(c), c.shape[0], _estrides(c)[0], tile, grid_tiles)
    if rc:
        raise ValueError(f"or_vector_add_1d failed ({rc})")
    return c


def vector_fma_1d(a: np.ndarray, b: np.ndarray, d: np.ndarray, c: np.ndarray, tile: int, grid_tiles: int) -> np.ndarray:
    """C[i] = fma(A[i], B[i], D[i]) (one rounding) over the tiles the grid covers; C updated in place."""
    for x in (a, b, d, c):
        assert x.dtype == np.float32 and x.ndim == 1
    rc = lib().or_vector_fma_1d(_ptr(a), a.shape[0], _estrides(a)[0], _ptr(b), b.shape[0], _estrides(b)[0],
                                _ptr(d), d.shape[0], _estrides(d)[0], _ptr(c), c.shape[0], _estrides(c)[0],
                                tile, grid_tiles)
    if rc:
        raise ValueError(f"or_vector_fma_1d failed ({rc})")
    return c


def cast(a: np.ndarray, out_dtype: int, *, bf16_in: bool = False) -> np.ndarray:
    """Elementwise conversion of a 1D array to F32 / F16 / BF16 (BF16 as uint16 bit patterns)."""
    a = np.ascontiguousarray(a).reshape(-1)
    in_code = _dtype_code(a, bf16_in)
    out = np.zeros(a.shape[0], dtype={F32: np.float32, F16: np.float16, BF16: np.uint16}[out_dtype])
    rc = lib().or_cast(in_code, _ptr(a), 1, out_dtype, _ptr(out), 1, a.shape[0])
    if rc:
        raise ValueError(f"or_cast failed ({rc})")
    return out


def vector_add_2d(a: np.ndarray, b: np.ndarray, c: np.ndarray, tm: int, tn: int, grid_x: int, grid_y: int) -> np.ndarray:
    for x in (a, b, c):
        assert x.dtype == np.float32 and x.ndim == 2

    def arr(v):
        return (ctypes.c_int64 * 2)(*v)

    rc = lib().or_vector_add_2d(_ptr(a), arr(a.shape), arr(_estrides(a)), _ptr(b), arr(b.shape), arr(_estrides(b)),
                                _ptr(c), arr(c.shape), arr(_estrides(c)), tm, tn, grid_x, grid_y)
    if rc:
        raise ValueError(f"or_vector_add_2d failed ({rc})")
    return c


def _dtype_code(a: np.ndarray, bf16: bool) -> int:
    if a.dtype == np.float32:
        return F32
    if a.dtype == np.float16:
        return F16
    if a.dtype == np.uint16 and bf16:
        return BF16
    raise TypeError(f"unsupported oracle dtype {a.dtype}")


def matmul(a: np.ndarray, b: np.ndarray, bias: np.ndarray | None = None, *, bf16: bool = False,
           out_dtype: int = F32, rows: tuple[int, int] | None = None, threads: int | None = None) -> np.ndarray:
    """C = A @ B (+ bias) with the reference's mmaf arithmetic.

    With ``rows=(r0, r1)`` only those rows are computed and an array of
    shape (r1 - r0, N) is returned.  ``bf16=True`` marks uint16 inputs as
    bfloat16 bit patterns.  ``out_dtype`` selects the stored type (F32, F16
    or BF16; F16 returns float16, BF16 returns uint16 bit patterns).
    """
    M, K = a.shape
    K2, N = b.shape
    assert K == K2
    in_code = _dtype_code(a, bf16)
    assert _dtype_code(b, bf16) == in_code
    r0, r1 = rows if rows is not None else (0, M)
    out_np = {F32: np.float32, F16: np.float16, BF16: np.uint16}[out_dtype]
    out = np.zeros((r1 - r0, N), dtype=out_np)
    bias_code, bias_ptr = 0, None
    if bias is not None:
        bias = np.ascontiguousarray(bias)
        bias_code = _dtype_code(bias, bf16)
        bias_ptr = _ptr(bias)
    # C rows are written at m * sc0; shift the base so row r0 lands at out[0]
    c_base = _ptr(out) - r0 * out.strides[0]
    sa, sb = _estrides(a), _estrides(b)
    n_threads = threads or os.cpu_count() or 1
    rc = lib().or_matmul(in_code, _ptr(a), sa[0], sa[1], _ptr(b), sb[0], sb[1], bias_code, bias_ptr,
                         out_dtype, c_base, N, 1, M, N, K, r0, r1, n_threads)
    if rc:
        raise ValueError(f"or_matmul failed ({rc})")
    return out


def reference_matmul_f32(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """The reference test's own naive CPU matmul (examples.cpp:533-551)."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    b = np.ascontiguousarray(b, dtype=np.float32)
    m, k = a.shape
    _, n = b.shape
    c = np.zeros((m, n), dtype=np.float32)
    lib().or_reference_matmul_f32(_ptr(a), _ptr(b), _ptr(c), m, n, k)
    return c


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round fp32 to bfloat16 (nearest even), returned as uint16 bit patterns."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def bf16_bits_to_f32(x: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(x, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_f16_bits(x: np.ndarray) -> np.ndarray:
    L = lib()
    flat = np.ascontiguousarray(x, dtype=np.float32).ravel()
    return np.array([L.or_f32_to_f16(float(v)) for v in flat], dtype=np.uint16).reshape(np.shape(x))


def f16_bits_to_f32(x: np.ndarray) -> np.ndarray:
    L = lib()
    flat = np.ascontiguousarray(x, dtype=np.uint16).ravel()
    return np.array([L.or_f16_to_f32(int(v)) for v in flat], dtype=np.float32).reshape(np.shape(x))


def kat_values(count: int, modulus: int, offset: int, scale: float) -> np.ndarray:
    out = np.empty(count, dtype=np.float32)
    lib().or_kat_values(_ptr(out), count, modulus, offset, scale)
    return out


def kat_iota(count: int, start: int) -> np.ndarray:
    out = np.empty(count, dtype=np.float32)
    lib().or_kat_iota(_ptr(out), count, start)
    return out


def matmul_kat_expected(m: int, n: int, k: int) -> np.ndarray:
    """Exact C for the reference's matmul known-answer inputs at any size.

    A[i, kk] = ((i*K + kk) % 17 - 8) * 0.25 and B[kk, j] = ((kk*N + j) % 13 - 6) * 0.5
    (examples.cpp:590-596).  Every product is a multiple of 1/8 bounded by 6,
    so every partial sum is exact in fp32 while 48*K < 2^21, and the result is
    independent of summation order.  A's residue depends on kk only through
    kk mod 17 and B's through kk mod 13, so the K sum folds into 221 residue
    classes and C depends on i only through (i*K) mod 17 and on j only
    through j mod 13: the full matrix is assembled from a 17 x 13 table.
    """
    assert 48 * k < 2 ** 24, "known-answer partial sums stop being exact in fp32"
    period = 17 * 13
    r = np.arange(period, dtype=np.int64)
    counts = (k - r + period - 1) // period  # number of kk < k with kk % 221 == r
    counts = np.maximum(counts, 0).astype(np.float64)
    ia = np.arange(17, dtype=np.int64)  # (i*K) mod 17
    jb = np.arange(13, dtype=np.int64)  # j mod 13
    fa = (((ia[:, None] + r[None, :]) % 17) - 8) * 0.25          # [17, 221]
    gb = ((((r[:, None] * n) + jb[None, :]) % 13) - 6) * 0.5      # [221, 13]
    table = (fa * counts[None, :]) @ gb                            # [17, 13], exact in f64
    rows = (np.arange(m, dtype=np.int64) * k) % 17
    cols = np.arange(n, dtype=np.int64) % 13
    return table[rows[:, None], cols[None, :]].astype(np.float32)


def time_matmul_rows(a: np.ndarray, b: np.ndarray, bias: np.ndarray | None, *, bf16: bool, out_dtype: int,
                     rows: int, threads: int) -> tuple[float, int]:
    """Run the oracle on the first ``rows`` rows; return (seconds, rows)."""
    t0 = time.perf_counter()
    matmul(a, b, bias, bf16=bf16, out_dtype=out_dtype, rows=(0, rows), threads=threads)
    return time.perf_counter() - t0, rows


def time_vector_add(a: np.ndarray, b: np.ndarray, c: np.ndarray, reps: int) -> float:
    """Seconds per full 1D vector add over the flattened arrays (single thread)."""
    a1, b1, c1 = a.reshape(-1), b.reshape(-1), c.reshape(-1)
    n = a1.shape[0]
    t0 = time.perf_counter()
    for _ in range(reps):
        vector_add_1d(a1, b1, c1, 1024, (n + 1023) // 1024)
    return (time.perf_counter() - t0) / reps
