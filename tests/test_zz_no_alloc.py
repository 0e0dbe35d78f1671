"""The allocation-free fp32 matmul entry point, st_matmul_static_scratch.

Some callers cannot allocate device memory -- a process whose memory pool
already holds the GPU's memory, or a latency-critical caller that cannot
afford cudaMalloc / cudaFree (cudaFree waits for the whole device).  For them
the library offers this variant of the 3xTF32 matmul, whose packed operands
live in a fixed array compiled into the library instead of a workspace grown
with cudaMalloc.  This file checks it against the regular entry point
(st_matmul) and the oracle, through the C ABI, on calls in a row that share
the array, and checks that a call after the first one on the device leaves
the GPU's free memory unchanged.  It is collected last so that a run
stopping at the first failure has already run every other test.
"""
import ctypes

import numpy as np
import pytest
import torch

import oracle
import sptiles_b200 as st
from sptiles_b200 import _native as N

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda:0")
TOL = 1e-3  # the fp32 (3xTF32) tolerance of the matmul tests: max|dC| / max|C_ref|
TOL16 = 1e-2  # a 16-bit C is one rounding of that result


def static_scratch_matmul(A, B, C, bias=None, flags=N.ST_EXEC_SYNC):
    """Call st_matmul_static_scratch through ctypes on torch's current stream."""
    va, vb, vc = st.tensor_view(A), st.tensor_view(B), st.tensor_view(C)
    vbias = ctypes.byref(st.tensor_view(bias)) if bias is not None else None
    stream = torch.cuda.current_stream(DEV).cuda_stream or 0x1  # 0x1: cudaStreamLegacy
    ex = N.StExec(stream, 0, flags, 60000, None, 0)
    return N.lib().st_matmul_static_scratch(ctypes.byref(va), ctypes.byref(vb), vbias, ctypes.byref(vc),
                                            ctypes.byref(ex))


def normal(shape, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    return torch.randn(shape, generator=g).to(DEV)


def rel_err(got, want):
    got, want = torch.as_tensor(got).double().cpu(), torch.as_tensor(want).double().cpu()
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
        # and against the oracle (the CPU restatement of the shader arithmetic)
        rows = (0, 64) if m > 64 else (0, m)
        want = oracle.matmul(A.cpu().numpy(), B.cpu().numpy(), None if bias is None else bias.cpu().numpy(),
                             rows=rows)
        assert rel_err(C_static[rows[0]:rows[1]], want) <= TOL


@pytest.mark.parametrize("out_dtype", [torch.float16, torch.bfloat16], ids=["f16", "bf16"])
def test_static_scratch_16bit_c_matches_regular_entry_point(out_dtype):
    m, n, k = 512, 384, 700
    A, B, bias = normal((m, k), 30), normal((k, n), 31), normal((n,), 32)
    for _ in range(2):  # two calls in a row on the shared array
        C_static = torch.zeros((m, n), dtype=out_dtype, device=DEV)
        N.check(static_scratch_matmul(A, B, C_static, bias), "st_matmul_static_scratch")
        C_regular = st.matmul(A, B, bias, out_dtype=out_dtype)
        torch.cuda.synchronize()
        assert rel_err(C_static.float(), C_regular.float()) <= TOL16
        ref = A.double() @ B.double() + bias.double()
        assert rel_err(C_static.float(), ref) <= TOL16


def test_static_scratch_deterministic_flag_repeats_bit_for_bit():
    """ST_EXEC_DETERMINISTIC: split tiles fold in a fixed order (here, with no
    workspace, whole tiles), so repeated calls agree to the bit."""
    m = n = k = 1024
    A, B = normal((m, k), 40), normal((k, n), 41)
    outs = []
    for _ in range(2):
        C = torch.zeros((m, n), device=DEV)
        N.check(static_scratch_matmul(A, B, C, flags=N.ST_EXEC_SYNC | N.ST_EXEC_DETERMINISTIC),
                "st_matmul_static_scratch")
        outs.append(C)
    assert torch.equal(outs[0], outs[1])
    assert rel_err(outs[0], st.matmul(A, B)) <= TOL


def test_static_scratch_allocates_no_device_memory_after_set_up():
    """Every case once (the first call on the device is the set-up), then the
    same calls again: the device's free memory must not move."""
    shapes = [((1024, 1024, 1024), torch.float32, 0), ((300, 200, 1000), torch.float32, N.ST_EXEC_DETERMINISTIC),
              ((512, 384, 700), torch.float16, 0), ((1, 1, 0), torch.float32, 0)]
    cases = []
    for (m, n, k), dt, flags in shapes:
        A, B = normal((m, k), 50), normal((k, n), 51)
        cases.append((A, B, torch.zeros((m, n), dtype=dt, device=DEV), normal((n,), 52), flags))
    for A, B, C, bias, flags in cases:
        N.check(static_scratch_matmul(A, B, C, bias, flags=N.ST_EXEC_SYNC | flags), "st_matmul_static_scratch")
    torch.cuda.synchronize()
    free_before, _ = torch.cuda.mem_get_info(DEV)
    for A, B, C, bias, flags in cases:
        N.check(static_scratch_matmul(A, B, C, bias, flags=N.ST_EXEC_SYNC | flags), "st_matmul_static_scratch")
    torch.cuda.synchronize()
    free_after, _ = torch.cuda.mem_get_info(DEV)
    assert free_after == free_before, f"device free memory moved by {free_before - free_after} bytes"


def test_static_scratch_rejects_problems_beyond_its_array():
    m = n = k = 2048  # (M + N) * 3 * K * 4 bytes = 96 MiB > 32 MiB
    A, B = torch.zeros((m, k), device=DEV), torch.zeros((k, n), device=DEV)
    C = torch.zeros((m, n), device=DEV)
    rc = static_scratch_matmul(A, B, C)
    assert rc == N.ST_ERR_INVALID_ARGUMENT
    assert "static scratch" in N.last_error()


def test_static_scratch_size_check_cannot_wrap():
    """Extents are caller metadata: views claiming 2^31 - 1 rows, columns and
    K (whose packed size overflows 64 bits) are rejected before any device
    work, not wrapped into a small size."""
    big = 2 ** 31 - 1
    A, B, C = (torch.zeros((4, 4), device=DEV) for _ in range(3))
    va, vb, vc = st.tensor_view(A), st.tensor_view(B), st.tensor_view(C)
    va.shape[0], va.shape[1] = big, big
    vb.shape[0], vb.shape[1] = big, big
    vc.shape[0], vc.shape[1] = big, big
    ex = N.StExec(0x1, 0, N.ST_EXEC_SYNC, 1000, None, 0)
    rc = N.lib().st_matmul_static_scratch(ctypes.byref(va), ctypes.byref(vb), None, ctypes.byref(vc),
                                          ctypes.byref(ex))
    assert rc == N.ST_ERR_INVALID_ARGUMENT
    assert "static scratch" in N.last_error()
