"""fma and ftof on the GPU against the oracle, bit for bit.

The lowering's other elementwise ops (tileops.hpp:616-623 fma,
tileops.hpp:257-258 ftof) as registry entries and typed calls."""
import ctypes

import numpy as np
import pytest
import torch

import oracle
import sptiles_b200 as st
from sptiles_b200 import _native as N

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")
CODES = {torch.float32: oracle.F32, torch.float16: oracle.F16, torch.bfloat16: oracle.BF16}


def uniform(n, seed):
    return np.random.default_rng(seed).uniform(-2, 2, n).astype(np.float32)


def oracle_fma(a, b, d):
    c = np.zeros_like(a)
    oracle.vector_fma_1d(np.ascontiguousarray(a), np.ascontiguousarray(b), np.ascontiguousarray(d), c, 1024,
                         -(-a.size // 1024) or 1)
    return c


def bits(t: torch.Tensor) -> np.ndarray:
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.float32:
        return t.view(torch.int32).numpy()
    return t.view(torch.int16).numpy()


@pytest.mark.parametrize("n", [1, 3, 4, 1000, 4097, 1 << 20])
def test_fma_bit_exact(n):
    a, b = uniform(n, 1), uniform(n, 2)
    d = (-(a * b) + uniform(n, 3) * np.float32(1e-3)).astype(np.float32)  # cancellation shows the single rounding
    C = st.vector_fma(*(torch.from_numpy(x).to(DEV) for x in (a, b, d)))
    assert C.cpu().numpy().tobytes() == oracle_fma(a, b, d).tobytes()


def test_fma_strided_misaligned_and_2d():
    n = 30_011
    a, b, d = uniform(3 * n + 3, 4), uniform(3 * n + 3, 5), uniform(3 * n + 3, 6)
    A, B, D = (torch.from_numpy(x).to(DEV) for x in (a, b, d))
    C = st.vector_fma(A[1:3 * n + 1:3], B[2:3 * n + 2:3], D[0:3 * n:3])
    assert C.cpu().numpy().tobytes() == oracle_fma(a[1:3 * n + 1:3], b[2:3 * n + 2:3], d[0:3 * n:3]).tobytes()
    C2 = st.vector_fma(A[1:n + 1], B[1:n + 1], D[1:n + 1])  # 4-byte offset: scalar path
    assert C2.cpu().numpy().tobytes() == oracle_fma(a[1:n + 1], b[1:n + 1], d[1:n + 1]).tobytes()
    M = torch.from_numpy(a[:300 * 100]).to(DEV).view(300, 100)
    C3 = st.vector_fma(M.t(), M.t(), M.t())
    want = oracle_fma(a[:30000], a[:30000], a[:30000]).reshape(300, 100).T
    assert C3.cpu().numpy().tobytes() == np.ascontiguousarray(want).tobytes()


@pytest.mark.parametrize("src", [torch.float32, torch.float16, torch.bfloat16], ids=["f32", "f16", "bf16"])
@pytest.mark.parametrize("dst", [torch.float32, torch.float16, torch.bfloat16], ids=["f32", "f16", "bf16"])
def test_cast_bit_exact(src, dst):
    rng = np.random.default_rng(31)
    x = np.concatenate([rng.standard_normal(100_001) * 10.0 ** rng.integers(-9, 6, 100_001),
                        np.array([0.0, -0.0, 65504, 65519.9, 65520, 1e-8, 6e-8, 3e38, np.inf, -np.inf])]
                       ).astype(np.float32)
    A = torch.from_numpy(x).to(src).to(DEV)  # torch's own rounding makes the source
    C = st.cast(A, dst)
    assert C.dtype == dst
    a_np = A.cpu()
    a_np = a_np.view(torch.int16).numpy().view(np.uint16) if src == torch.bfloat16 else a_np.numpy()
    want = oracle.cast(a_np, CODES[dst], bf16_in=src == torch.bfloat16)
    got = bits(C)
    assert got.tobytes() == want.view(got.dtype).tobytes()
    # strided and 2D views take the element-wise kernel
    C2 = st.cast(A[: 1000 * 100].view(1000, 100).t(), dst)
    want2 = want[: 100_000].reshape(1000, 100).T
    assert bits(C2).tobytes() == np.ascontiguousarray(want2).view(got.dtype).tobytes()


def test_cast_nan_stays_nan():
    A = torch.tensor([float("nan"), -float("nan"), 1.0], device=DEV)
    for dt in (torch.float16, torch.bfloat16):
        C = st.cast(A, dt).float().cpu()
        assert torch.isnan(C[:2]).all() and C[2] == 1.0


def _launch_host(entry, arrays, grid, out_index, consts=()):
    params = []
    for a in arrays:
        params += st.tensor_1d_descriptor(a) if a.ndim == 1 else st.tensor_2d_descriptor(a)
    params += [np.array([c], np.int32) for c in consts]
    return st.run_tile_kernel(entry_name=entry, parameter_arrays=params, output_indices=[out_index], grid=grid)[0]


def test_entries_through_the_runner_with_partial_grids():
    n = 5000
    a, b, d = uniform(n, 7), uniform(n, 8), uniform(n, 9)
    c = np.full(n, 5.0, np.float32)
    got = _launch_host("vector_fma", [a, b, d, c], (3, 1, 1), 9, consts=(1024,))
    want = c.copy()
    oracle.vector_fma_1d(a, b, d, want, 1024, 3)
    assert got.tobytes() == want.tobytes()
    h = np.zeros(n, np.float16)
    got = _launch_host("cast", [a, h], (5, 1, 1), 3)
    assert got.tobytes() == oracle.cast(a, oracle.F16).tobytes()
    # 2D fma with a partial tile grid
    m2 = a[:60 * 70].reshape(60, 70)
    c2 = np.zeros((60, 70), np.float32)
    got = _launch_host("vector_fma_2d", [m2, m2, m2, c2], (1, 2, 1), 15, consts=(32, 32))
    want2 = np.zeros((60, 70), np.float32)
    want2[:32, :64] = oracle_fma(m2[:32, :64].ravel(), m2[:32, :64].ravel(), m2[:32, :64].ravel()).reshape(32, 64)
    assert got.reshape(60, 70).tobytes() == want2.tobytes()
