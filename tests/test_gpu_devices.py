"""The single-box partitioner inside one process (ST_EXEC_ALL_DEVICES), on the GPU.

A context over every visible GPU splits a host-memory call: vector_add by
element ranges (or rows, for strided views), matmul by 128-row blocks of A
and C with B and the bias sent to every device.  Results must be what the
oracle computes -- bit-exact for the add and the matmul known answers,
within the matmul tolerance (max|dC| / max|C_ref| <= 1e-2 for 16-bit
inputs) on seeded normals.  With two or more GPUs, the GEMM with the
all-gather fused into its epilogue also runs inside one process: each
device stores its rows into every device's copy of C over NVLink (peer
access enabled by the multi-device context).  Runs on one GPU too (a
one-device split); the peer test needs two.
"""
import ctypes

import numpy as np
import pytest
import torch

import oracle
import sptiles_b200 as st
from sptiles_b200 import _native as N

pytestmark = pytest.mark.gpu

G = torch.cuda.device_count() if torch.cuda.is_available() else 0
ALL = tuple(range(G))
needs_two = pytest.mark.skipif(G < 2, reason="needs two GPUs")


def kat(m, n, k):
    return (oracle.kat_values(m * k, 17, 8, 0.25).reshape(m, k), oracle.kat_values(k * n, 13, 6, 0.5).reshape(k, n))


def bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.view(torch.int16).numpy().view(np.uint16)


@pytest.mark.parametrize("dtype,shape", [(torch.float16, (1000, 768, 320)), (torch.bfloat16, (130, 300, 96)),
                                         (torch.float32, (300, 200, 100))])
def test_matmul_host_split_over_all_devices_known_answer(dtype, shape):
    m, n, k = shape
    a, b = kat(m, n, k)
    A, B = torch.from_numpy(a).to(dtype), torch.from_numpy(b).to(dtype)
    C = st.matmul(A, B, out_dtype=torch.float32, devices=ALL)
    assert C.numpy().tobytes() == oracle.matmul_kat_expected(m, n, k).tobytes()


def test_matmul_host_split_bf16_with_bias():
    m, n, k = 1100, 520, 256
    rng = np.random.default_rng(4)
    a = torch.from_numpy(rng.standard_normal((m, k)) * 0.05).to(torch.bfloat16)
    b = torch.from_numpy(rng.standard_normal((k, n)) * 0.05).to(torch.bfloat16)
    bias = torch.from_numpy(rng.uniform(-1, 1, n).astype(np.float32))
    C = st.matmul(a, b, bias, out_dtype=torch.float32, devices=ALL).numpy()
    ref = oracle.matmul(bf16_bits(a), bf16_bits(b), bias.numpy(), bf16=True)
    assert np.abs(C - ref).max() / np.abs(ref).max() <= 1e-2


def test_vector_add_host_split_flat_and_strided():
    n = 1_000_003
    rng = np.random.default_rng(7)
    x = rng.uniform(-1, 1, n).astype(np.float32)
    y = rng.uniform(-1, 1, n).astype(np.float32)
    C = st.vector_add(torch.from_numpy(x), torch.from_numpy(y), devices=ALL)
    assert C.numpy().tobytes() == (x + y).tobytes()
    # row-padded host views (pitch 800, 700 columns): rows are split instead of elements
    a = rng.uniform(-1, 1, (300, 800)).astype(np.float32)
    b = rng.uniform(-1, 1, (300, 800)).astype(np.float32)
    C = st.vector_add(torch.from_numpy(a)[:, :700], torch.from_numpy(b)[:, :700], devices=ALL)
    assert C.numpy().tobytes() == np.ascontiguousarray((a + b)[:, :700]).tobytes()


def test_all_devices_runs_on_the_contexts_streams():
    a = torch.zeros(16)
    va = st.tensor_view(a)
    ctx = st.context_group(ALL)
    for stream, device in ((ctypes.c_void_p(1), -1), (None, 0)):
        ex = N.StExec(stream, device, N.ST_EXEC_ALL_DEVICES, 1000, None, 0)
        rc = N.lib().st_vector_add_host(ctx, ctypes.byref(va), ctypes.byref(va), ctypes.byref(va), ctypes.byref(ex))
        assert rc == N.ST_ERR_INVALID_ARGUMENT and "ST_EXEC_ALL_DEVICES" in N.last_error()
    with pytest.raises(ValueError, match="host tensors"):
        st.matmul(a.reshape(4, 4).cuda(), a.reshape(4, 4).cuda(), devices=ALL)


@needs_two
def test_fused_allgather_between_devices_of_one_process():
    devs = ALL[:8]
    ctx = st.context_group(devs)
    m, n, k = 3000, 1024, 512
    a, b = kat(m, n, k)
    copies, parts = [], []
    for g, d in enumerate(devs):
        r0, r1 = st.shard_range(m, len(devs), g, 128)
        dev = torch.device("cuda", d)
        A = torch.from_numpy(a[r0:r1]).to(dev, torch.bfloat16)
        B = torch.from_numpy(b).to(dev, torch.bfloat16)
        copies.append(torch.zeros((m, n), device=dev))
        parts.append((r0, A, B))
    for d in devs:
        torch.cuda.synchronize(d)  # every copy of C is allocated and zeroed before any device writes into it
    for g, d in enumerate(devs):
        r0, A, B = parts[g]
        peers = (ctypes.c_void_p * (len(devs) - 1))(*[copies[e].data_ptr() for e in range(len(devs)) if e != g])
        ex = N.StExec(None, d, N.ST_EXEC_SYNC, 60000, None, 0)
        va, vb, vc = st.tensor_view(A), st.tensor_view(B), st.tensor_view(copies[g])
        N.check(N.lib().st_matmul_allgather(ctx, ctypes.byref(va), ctypes.byref(vb), None, ctypes.byref(vc),
                                            peers, len(devs) - 1, r0, ctypes.byref(ex)), "st_matmul_allgather")
    want = oracle.matmul_kat_expected(m, n, k).tobytes()
    for C in copies:
        assert C.cpu().numpy().tobytes() == want


def test_host_buffer_launch_split_over_all_devices():
    # run_spirv_kernel's contract (host arrays, a dispatch) with the launch split over every device
    n = 1_000_003
    rng = np.random.default_rng(8)
    a = rng.uniform(-1, 1, n).astype(np.float32)
    b = rng.uniform(-1, 1, n).astype(np.float32)
    params = st.tensor_1d_descriptor(a) + st.tensor_1d_descriptor(b) + st.tensor_1d_descriptor(np.zeros(n, np.float32))
    (c,) = st.run_tile_kernel(entry_name="vector_add", parameter_arrays=params, output_indices=[6],
                              dispatch=(-(-n // 1024), 1, 1), devices=ALL)
    assert c.tobytes() == (a + b).tobytes()
    # a partial grid: only its tiles are computed, by whichever device holds them
    params = st.tensor_1d_descriptor(a) + st.tensor_1d_descriptor(b) + \
        st.tensor_1d_descriptor(np.full(n, -5.0, np.float32))
    (c,) = st.run_tile_kernel(entry_name="vector_add", parameter_arrays=params, output_indices=[6], grid=(300, 1, 1),
                              devices=ALL)
    want = np.full(n, -5.0, np.float32)
    oracle.vector_add_1d(a, b, want, 1024, 300)
    assert c.tobytes() == want.tobytes()
    # the reference's matmul_fp32 entry on its known answers
    m, k, nn = 700, 333, 500
    ka, kb = kat(m, nn, k)
    params = st.tensor_2d_descriptor(ka) + st.tensor_2d_descriptor(kb) + \
        st.tensor_2d_descriptor(np.zeros((m, nn), np.float32))
    (c,) = st.run_tile_kernel(entry_name="matmul_fp32", parameter_arrays=params, output_indices=[10],
                              grid=(-(-m // 32) * -(-nn // 32), 1, 1), devices=ALL)
    assert c.reshape(m, nn).tobytes() == oracle.matmul_kat_expected(m, nn, k).tobytes()
    # a matmul grid short of the tile count is refused, as on one device
    with pytest.raises(NotImplementedError, match="must cover"):
        st.run_tile_kernel(entry_name="matmul_fp32", parameter_arrays=params, output_indices=[10], grid=(3, 1, 1),
                           devices=ALL)
