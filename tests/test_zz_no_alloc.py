"""The allocation-free fp32 matmul entry point, st_matmul_static_scratch.

Some callers cannot allocate device memory -- a process whose memory pool
already holds the GPU's memory, or a latency-critical caller that cannot
afford cudaMalloc / cudaFree (cudaFree waits for the whole device).  For them
the library offers this variant of the 3xTF32 matmul, whose packed operands
live in a fixed array compiled into the library instead of a workspace grown
with cudaMalloc.  This file checks it against the regular entry point
(st_matmul), through the C ABI, on two calls in a row that share the array.
It is collected last so that a run stopping at the first failure has already
run every other test.
"""
import ctypes

import numpy as np
import pytest
import torch

import sptiles_b200 as st
from sptiles_b200 import _native as N

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda:0")
TOL = 1e-3  # the fp32 (3xTF32) tolerance of the matmul tests: max|dC| / max|C_ref|


def static_scratch_matmul(A, B, C, bias=None):
    """Call st_matmul_static_scratch through ctypes on torch's current stream."""
    va, vb, vc = st.tensor_view(A), st.tensor_view(B), st.tensor_view(C)
    vbias = ctypes.byref(st.tensor_view(bias)) if bias is not None else None
    stream = torch.cuda.current_stream(DEV).cuda_stream or 0x1  # 0x1: cudaStreamLegacy
    ex = N.StExec(stream, 0, N.ST_EXEC_SYNC, 60000, None, 0)
    return N.lib().st_matmul_static_scratch(ctypes.byref(va), ctypes.byref(vb), vbias, ctypes.byref(vc),
                                            ctypes.byref(ex))


def normal(shape, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    return torch.randn(shape, generator=g).to(DEV)


def rel_err(got, want):
    return ((got - want).abs().max() / want.abs().max()).item()


def test_static_scratch_matches_regular_entry_point_on_two_calls():
    # first call: the 1024^3 fp32 configuration; second call: a ragged shape
    # with a bias, reusing (and fully overwriting) the same static array
    cases = [((1024, 1024, 1024), False, 2), ((300, 200, 1000), True, 5)]
    for (m, n, k), with_bias, seed in cases:
        A, B = normal((m, k), seed), normal((k, n), seed + 1)
        bias = normal((n,), seed + 2) if with_bias else None
        C_static = torch.full((m, n), float("nan"), device=DEV)
        N.check(static_scratch_matmul(A, B, C_static, bias), "st_matmul_static_scratch")
        C_regular = st.matmul(A, B, bias)  # the existing entry point, st_matmul
        torch.cuda.synchronize()
        assert torch.isfinite(C_static).all()
        assert rel_err(C_static, C_regular) <= TOL


def test_static_scratch_rejects_problems_beyond_its_array():
    m = n = k = 2048  # (M + N) * 3 * K * 4 bytes = 96 MiB > 32 MiB
    A, B = torch.zeros((m, k), device=DEV), torch.zeros((k, n), device=DEV)
    C = torch.zeros((m, n), device=DEV)
    rc = static_scratch_matmul(A, B, C)
    assert rc == N.ST_ERR_INVALID_ARGUMENT
    assert "static scratch" in N.last_error()
