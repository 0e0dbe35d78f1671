"""vector_add on the GPU against the oracle: bit-exact, every path.

Sizes of the benchmark configurations (2^20 elements with 1024-element
tiles; 4096 x 4096 with 64 x 64 tiles), the reference's known answers, and
the edge cases: empty and tiny inputs, misaligned bases, mixed alignments,
strided and transposed views, partial tile grids."""
import json
from pathlib import Path

import numpy as np
import pytest
import torch

import oracle
import sptiles_b200 as st
from sptiles_b200 import _native as N

pytestmark = pytest.mark.gpu

GOLD = Path(__file__).resolve().parent / "golden"
META = json.loads((GOLD / "golden.json").read_text())
DEV = torch.device("cuda:0")


def uniform(n, seed, shape=None):
    rng = np.random.default_rng(seed)
    x = rng.uniform(-1.0, 1.0, n if shape is None else shape).astype(np.float32)
    return x


def oracle_add(a, b):
    c = np.zeros_like(a).reshape(-1)
    oracle.vector_add_1d(np.ascontiguousarray(a).reshape(-1), np.ascontiguousarray(b).reshape(-1), c, 1024,
                         -(-a.size // 1024))
    return c.reshape(a.shape)


@pytest.mark.parametrize("case", META["vector_add"], ids=lambda c: c["file"])
def test_known_answers_through_drop_in_api(case):
    f = np.load(GOLD / case["file"])
    A, B = torch.from_numpy(f["a"]), torch.from_numpy(f["b"])
    # host tensors: the reference's own calling pattern (spirv_vector_add.py:103-109)
    C = st.spirv_vector_add(A, B)
    assert C.device.type == "cpu"
    assert C.numpy().tobytes() == f["expected"].tobytes()
    # device tensors: in place on the current stream
    Cd = st.spirv_vector_add(A.to(DEV), B.to(DEV))
    assert Cd.device == A.to(DEV).device
    assert Cd.cpu().numpy().tobytes() == f["expected"].tobytes()


@pytest.mark.parametrize("case", META["vector_add"], ids=lambda c: c["file"])
def test_known_answers_through_runner(case):
    """run_tile_kernel with the reference's 9 bindings and 1024-wide dispatch."""
    f = np.load(GOLD / case["file"])
    n = case["size"]
    params = [*st.tensor_1d_descriptor(f["a"]), *st.tensor_1d_descriptor(f["b"]),
              *st.tensor_1d_descriptor(np.zeros(n, np.float32))]
    out = st.run_tile_kernel(entry_name="vector_add", parameter_arrays=params, output_indices=[6],
                             dispatch=tuple(case["dispatch"]))[0]
    assert out.tobytes() == f["expected"].tobytes()


def test_config_1d_2pow20_seed0_bit_exact():
    a, b = uniform(2 ** 20, 0), uniform(2 ** 20, 100)
    C = st.vector_add(torch.from_numpy(a).to(DEV), torch.from_numpy(b).to(DEV))
    assert C.cpu().numpy().tobytes() == oracle_add(a, b).tobytes()


def test_config_2d_4096_seed1_bit_exact():
    a, b = uniform(None, 1, (4096, 4096)), uniform(None, 101, (4096, 4096))
    C = st.vector_add(torch.from_numpy(a).to(DEV), torch.from_numpy(b).to(DEV))
    assert C.shape == (4096, 4096)
    assert C.cpu().numpy().tobytes() == oracle_add(a, b).tobytes()


@pytest.mark.parametrize("n", [0, 1, 3, 4, 17, 63, 64, 65, 1023, 1025, 4097, 100_003])
def test_ragged_sizes(n):
    a, b = uniform(n, n), uniform(n, n + 1)
    C = st.vector_add(torch.from_numpy(a).to(DEV), torch.from_numpy(b).to(DEV))
    assert C.cpu().numpy().tobytes() == oracle_add(a, b).tobytes()


@pytest.mark.parametrize("offs", [(1, 1, 1), (2, 2, 2), (3, 3, 3), (1, 2, 3), (0, 1, 0)])
def test_misaligned_and_mixed_alignment(offs):
    n = 10_007
    base = [torch.from_numpy(uniform(n + 8, 7 + i)).to(DEV) for i in range(2)]
    out = torch.zeros(n + 8, device=DEV)
    A, B = base[0][offs[0]:offs[0] + n], base[1][offs[1]:offs[1] + n]
    Cv = out[offs[2]:offs[2] + n]
    st.vector_add(A, B, out=Cv)
    want = oracle_add(A.cpu().numpy(), B.cpu().numpy())
    assert Cv.cpu().numpy().tobytes() == want.tobytes()
    # nothing outside the view was written
    assert not out[:offs[2]].any() and not out[offs[2] + n:].any()


def test_strided_1d():
    a, b = uniform(30_000, 8), uniform(30_000, 9)
    A, B = torch.from_numpy(a).to(DEV)[::3], torch.from_numpy(b).to(DEV)[::3]
    C = st.vector_add(A, B)
    assert C.cpu().numpy().tobytes() == (a[::3] + b[::3]).tobytes()


@pytest.mark.parametrize("shape", [(1, 1), (7, 5), (64, 64), (100, 70), (33, 4096), (4096, 33)])
def test_2d_shapes_and_views(shape):
    a, b = uniform(None, 12, shape), uniform(None, 13, shape)
    A, B = torch.from_numpy(a).to(DEV), torch.from_numpy(b).to(DEV)
    assert st.vector_add(A, B).cpu().numpy().tobytes() == (a + b).tobytes()
    # transposed (column-major) operands and a padded-row output
    At, Bt = A.t(), B.t()
    outbuf = torch.zeros((shape[1], shape[0] + 5), device=DEV)
    Cv = outbuf[:, : shape[0]]
    st.vector_add(At, Bt, out=Cv)
    assert Cv.cpu().numpy().tobytes() == np.ascontiguousarray((a + b).T).tobytes()
    assert not outbuf[:, shape[0]:].any()


def _launch(entry, grid, params, consts=()):
    ctx = st.context(0)
    P = (N.StParam * (len(params) + len(consts)))()
    for i, p in enumerate(params):
        if isinstance(p, torch.Tensor):
            P[i].kind, P[i].dtype, P[i].data, P[i].bytes = N.ST_PARAM_BUFFER, N.ST_F32, p.data_ptr(), \
                p.numel() * p.element_size()
        else:
            P[i].kind, P[i].value = N.ST_PARAM_I32, int(p)
    for j, c in enumerate(consts):
        P[len(params) + j].kind, P[len(params) + j].value = N.ST_PARAM_I32, int(c)
    g = N.StGrid(*grid)
    ex = N.StExec(torch.cuda.current_stream().cuda_stream, 0, N.ST_EXEC_SYNC, 60000, None, 0)
    import ctypes
    N.check(N.lib().st_launch(ctx, entry.encode(), ctypes.byref(g), P, len(P), ctypes.byref(ex)), entry)


def test_partial_tile_grid_computes_only_its_tiles():
    """Tile block b owns [b*T, (b+1)*T); a short grid leaves the rest untouched."""
    n, tile, grid = 5000, 256, 7
    a, b = uniform(n, 20), uniform(n, 21)
    A, B = torch.from_numpy(a).to(DEV), torch.from_numpy(b).to(DEV)
    C = torch.full((n,), -7.0, device=DEV)
    _launch("vector_add", (grid, 1, 1), [A, n, 1, B, n, 1, C, n, 1], consts=[tile])
    want = np.full(n, -7.0, np.float32)
    oracle.vector_add_1d(a, b, want, tile, grid)
    assert C.cpu().numpy().tobytes() == want.tobytes()


def test_vector_add_2d_entry_with_partial_grid():
    shape = (300, 200)
    a, b = uniform(None, 30, shape), uniform(None, 31, shape)
    A, B = torch.from_numpy(a).to(DEV), torch.from_numpy(b).to(DEV)
    C = torch.zeros(shape, device=DEV)
    grid = (3, 2, 1)  # rows < 192, cols < 128 with 64 x 64 tiles
    _launch("vector_add_2d", grid, [A, 300, 200, 200, 1, B, 300, 200, 200, 1, C, 300, 200, 200, 1], consts=[64, 64])
    want = np.zeros(shape, np.float32)
    oracle.vector_add_2d(a, b, want, 64, 64, grid[0], grid[1])
    assert C.cpu().numpy().tobytes() == want.tobytes()
    # full grid of the configuration's tile shape covers everything
    _launch("vector_add_2d", (5, 4, 1), [A, 300, 200, 200, 1, B, 300, 200, 200, 1, C, 300, 200, 200, 1])
    assert C.cpu().numpy().tobytes() == (a + b).tobytes()


def test_descriptor_reaching_past_buffer_is_rejected():
    A = torch.zeros(100, device=DEV)
    with pytest.raises(ValueError, match="past its buffer"):
        _launch("vector_add", (1, 1, 1), [A, 200, 1, A, 100, 1, A, 100, 1])


@pytest.mark.parametrize("pinned", [True, False])
def test_host_arrays_chunked_pipeline(pinned):
    n = 10_000_003  # three 4M-element chunks, ragged tail
    a, b = uniform(n, 50), uniform(n, 51)
    A, B = torch.from_numpy(a), torch.from_numpy(b)
    if pinned:
        A, B = A.pin_memory(), B.pin_memory()
    C = st.vector_add(A, B)
    assert C.device.type == "cpu"
    assert C.numpy().tobytes() == oracle_add(a, b).tobytes()
    # 2D host arrays flatten to the same pipeline
    C2 = st.vector_add(A[: 4000 * 2500].view(4000, 2500), B[: 4000 * 2500].view(4000, 2500))
    assert C2.numpy().tobytes() == oracle_add(a[: 10_000_000], b[: 10_000_000]).reshape(4000, 2500).tobytes()
