"""Launching cuda_tile module entries on the GPU (st_launch_module), against the oracle.

Each fixture in tests/golden is a module that cuda.tile exported from the
reference's kernels (tests/golden/make_tilebc.py).  Launched by entry with
the module's own tile sizes, the results must be what the oracle computes
for that tile grid: bit-exact for vector_add; for matmul, bit-exact on the
reference's known-answer inputs and within the matmul tolerance (max|dC| /
max|C_ref|: 1e-3 for fp32 inputs, 1e-2 for fp16 / bf16) on seeded normals.
"""
from pathlib import Path

import numpy as np
import pytest
import torch

import oracle
import sptiles_b200 as st
from sptiles_b200 import _native as N

pytestmark = pytest.mark.gpu

GOLD = Path(__file__).resolve().parent / "golden"
DEV = torch.device("cuda:0")
CODES = {torch.float32: N.ST_F32, torch.float16: N.ST_F16, torch.bfloat16: N.ST_BF16}


def launch(module: st.TileModule, entry, grid, arrays, consts=()):
    """st_launch_module with device tensors; each array binds as (data, sizes..., strides...)."""
    binds = []
    for t in arrays:
        binds.append(t)
        binds += list(t.shape) + list(t.stride())
    P = (N.StParam * (len(binds) + len(consts)))()
    for i, b in enumerate(binds):
        if isinstance(b, torch.Tensor):
            P[i].kind, P[i].dtype, P[i].data = N.ST_PARAM_BUFFER, CODES[b.dtype], b.data_ptr()
            P[i].bytes = b.untyped_storage().nbytes() - b.storage_offset() * b.element_size()
        else:
            P[i].kind, P[i].value = N.ST_PARAM_I32, int(b)
    for j, c in enumerate(consts):
        P[len(binds) + j].kind, P[len(binds) + j].value = N.ST_PARAM_I32, int(c)
    ex = N.StExec(torch.cuda.current_stream(DEV).cuda_stream or 0x1, 0, N.ST_EXEC_SYNC, 60000, None, 0)
    module.launch(st.context(0), entry, grid, P, ex)


def uniform(n, seed):
    return np.random.default_rng(seed).uniform(-1.0, 1.0, n).astype(np.float32)


def cdiv(a, b):
    return -(-a // b)


@pytest.mark.parametrize("name,tile", [("vector_add.tilebc", 16), ("vector_add2D.tilebc", 512),
                                       ("vector_add_tile1024.tilebc", 1024)])
@pytest.mark.parametrize("n", [1 << 20, 5003])
def test_vector_add_modules_bit_exact(name, tile, n):
    m = st.TileModule(GOLD / name)
    assert m.entry().constants == (tile,)
    a, b = uniform(n, 0), uniform(n, 1)
    A, B = torch.from_numpy(a).to(DEV), torch.from_numpy(b).to(DEV)
    for grid in (cdiv(n, tile), cdiv(n, tile) // 2 + 1):  # full, then partial: only the named tiles
        C = torch.full((n,), -3.0, device=DEV)
        launch(m, None, (grid, 1, 1), [A, B, C])
        want = np.full(n, -3.0, np.float32)
        oracle.vector_add_1d(a, b, want, tile, grid)
        assert C.cpu().numpy().tobytes() == want.tobytes()


def test_vector_add_module_through_the_runner_with_a_dispatch():
    # run_spirv_kernel's contract with the module in place of the SPIR-V: host arrays, 1024-wide dispatch
    n = 4112
    a, b = uniform(n, 2), uniform(n, 3)
    c = np.zeros(n, np.float32)
    params = st.tensor_1d_descriptor(a) + st.tensor_1d_descriptor(b) + st.tensor_1d_descriptor(c)
    (out,) = st.run_tile_kernel(module=GOLD / "vector_add.tilebc", parameter_arrays=params, output_indices=[6],
                                dispatch=(cdiv(n, 1024), 1, 1))
    want = np.zeros(n, np.float32)
    oracle.vector_add_1d(a, b, want, 16, cdiv(n, 16))
    assert out.tobytes() == want.tobytes()


def kat(m, n, k, dtype):
    a = oracle.kat_values(m * k, 17, 8, 0.25).reshape(m, k)
    b = oracle.kat_values(k * n, 13, 6, 0.5).reshape(k, n)
    return torch.from_numpy(a).to(DEV, dtype), torch.from_numpy(b).to(DEV, dtype)


@pytest.mark.parametrize("shape", [(256, 256, 256), (100, 70, 33), (1024, 1024, 1024)])
def test_reference_matmul_module_known_answers(shape):
    m, n, k = shape
    mod = st.TileModule(GOLD / "matmul.tilebc")
    A, B = kat(m, n, k, torch.float32)
    C = torch.full((m, n), float("nan"), device=DEV)
    launch(mod, "matmul_fp32", (cdiv(m, 32) * cdiv(n, 32), 1, 1), [A, B, C])
    assert C.cpu().numpy().tobytes() == oracle.matmul_kat_expected(m, n, k).tobytes()


def test_reference_matmul_module_seeded_normals():
    m, n, k = 300, 200, 170
    rng = np.random.default_rng(2)
    a = rng.standard_normal((m, k)).astype(np.float32)
    b = rng.standard_normal((k, n)).astype(np.float32)
    C = torch.zeros((m, n), device=DEV)
    launch(st.TileModule(GOLD / "matmul.tilebc"), None, (cdiv(m, 32) * cdiv(n, 32), 1, 1),
           [torch.from_numpy(a).to(DEV), torch.from_numpy(b).to(DEV), C])
    ref = oracle.matmul(a, b)
    assert np.abs(C.cpu().numpy() - ref).max() / np.abs(ref).max() <= 1e-3


def test_matmul_module_through_the_runner_on_host_arrays():
    m, n, k = 64, 64, 64
    a = oracle.kat_values(m * k, 17, 8, 0.25).reshape(m, k)
    b = oracle.kat_values(k * n, 13, 6, 0.5).reshape(k, n)
    c = np.zeros((m, n), np.float32)
    params = st.tensor_2d_descriptor(a) + st.tensor_2d_descriptor(b) + st.tensor_2d_descriptor(c)
    (out,) = st.run_tile_kernel(module=GOLD / "matmul.tilebc", entry_name="matmul_fp32", parameter_arrays=params,
                                output_indices=[10], dispatch=(cdiv(m * n, 1024), 1, 1))
    assert out.reshape(m, n).tobytes() == oracle.matmul_kat_expected(m, n, k).tobytes()


def test_f16_module_with_f32_output_known_answer_and_normals():
    mod = st.TileModule(GOLD / "matmul_f16_f32out.tilebc")
    assert mod.entry().constants == (128, 256, 64)
    m, n, k = 512, 768, 320
    A, B = kat(m, n, k, torch.float16)
    C = torch.zeros((m, n), device=DEV)
    launch(mod, "matmul_f16", (cdiv(m, 128) * cdiv(n, 256), 1, 1), [A, B, C])
    assert C.cpu().numpy().tobytes() == oracle.matmul_kat_expected(m, n, k).tobytes()
    rng = np.random.default_rng(3)
    a = (rng.standard_normal((m, k)) * 0.1).astype(np.float16)
    b = (rng.standard_normal((k, n)) * 0.1).astype(np.float16)
    launch(mod, "matmul_f16", (cdiv(m, 128) * cdiv(n, 256), 1, 1),
           [torch.from_numpy(a).to(DEV), torch.from_numpy(b).to(DEV), C])
    ref = oracle.matmul(a, b)
    assert np.abs(C.cpu().numpy() - ref).max() / np.abs(ref).max() <= 1e-2
    # the module declares f16 operands: f32 ones are refused before any work
    with pytest.raises(ValueError, match="declares f16 data, got f32"):
        launch(mod, "matmul_f16", (cdiv(m, 128) * cdiv(n, 256), 1, 1), [A.float(), B.float(), C])


@pytest.mark.parametrize("grid", [1, 7, 148])
def test_persistent_bf16_module_any_grid(grid):
    mod = st.TileModule(GOLD / "persistent_matmul_bf16.tilebc")
    m, n, k = 640, 512, 256
    A, B = kat(m, n, k, torch.bfloat16)
    C = torch.zeros((m, n), device=DEV, dtype=torch.bfloat16)
    launch(mod, None, (grid, 1, 1), [A, B, C])
    want = torch.from_numpy(oracle.matmul_kat_expected(m, n, k)).to(torch.bfloat16)
    assert torch.equal(C.cpu(), want)


def test_multi_entry_module_each_entry_with_its_tiles():
    mod = st.TileModule(GOLD / "matmul_multi.tilebc")
    m, n, k = 384, 320, 96
    for e, dtype in zip(mod.entries, (torch.float32, torch.float16, torch.bfloat16)):
        tm, tn, _ = e.constants
        A, B = kat(m, n, k, dtype)
        C = torch.zeros((m, n), device=DEV, dtype=dtype)
        launch(mod, e.name, (cdiv(m, tm) * cdiv(n, tn), 1, 1), [A, B, C])
        want = torch.from_numpy(oracle.matmul_kat_expected(m, n, k)).to(dtype)
        assert torch.equal(C.cpu(), want), e.name
        if cdiv(m, tm) * cdiv(n, tn) > 1:  # a grid short of the module's tile count is refused
            with pytest.raises(NotImplementedError):
                launch(mod, e.name, (cdiv(m, tm) * cdiv(n, tn) - 1, 1, 1), [A, B, C])


def test_ambiguous_module_with_the_callers_tile_sizes():
    mod = st.TileModule(GOLD / "matmul_ambiguous.tilebc")
    m, n, k = 200, 130, 64
    A, B = kat(m, n, k, torch.float32)
    C = torch.zeros((m, n), device=DEV)
    with pytest.raises(ValueError, match="unambiguously"):
        launch(mod, "matmul_fp32_large", (cdiv(m, 64) * cdiv(n, 64), 1, 1), [A, B, C])
    launch(mod, "matmul_fp32_large", (cdiv(m, 64) * cdiv(n, 64), 1, 1), [A, B, C], consts=(64, 64, 32))
    assert C.cpu().numpy().tobytes() == oracle.matmul_kat_expected(m, n, k).tobytes()


def test_module_launch_counts_native_kernels():
    before = st.kernel_launches()
    n = 4096
    A = torch.ones(n, device=DEV)
    C = torch.zeros(n, device=DEV)
    launch(st.TileModule(GOLD / "vector_add_tile1024.tilebc"), None, (4, 1, 1), [A, A, C])
    assert st.kernel_launches() > before
    assert torch.equal(C, torch.full((n,), 2.0, device=DEV))
