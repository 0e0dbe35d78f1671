"""The tensor-core matmul on the GPU against the oracle.

Tolerance (relative to the largest reference magnitude of the matrix, since
normal inputs make elementwise relative error meaningless near zero):
  fp32 inputs (3xTF32):      max|C - C_ref| / max|C_ref| <= 1e-3
  fp16 / bf16 inputs:        max|C - C_ref| / max|C_ref| <= 1e-2
The reference's known-answer inputs make every partial sum exact, so those
cases are compared bit for bit, at the benchmark configurations' full sizes
as well.
"""
import contextlib
import ctypes
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
TOL = {torch.float32: 1e-3, torch.float16: 1e-2, torch.bfloat16: 1e-2}


def rel_err(got: np.ndarray, want: np.ndarray) -> float:
    scale = float(np.max(np.abs(want))) or 1.0
    return float(np.max(np.abs(got.astype(np.float64) - want.astype(np.float64)))) / scale


def to_np(t: torch.Tensor) -> np.ndarray:
    """Host numpy copy; bf16 as uint16 bit patterns (the oracle's convention)."""
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


def as_f32(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()


def oracle_mm(A, B, bias=None, rows=None, out=oracle.F32):
    bf = A.dtype == torch.bfloat16
    return oracle.matmul(to_np(A), to_np(B), None if bias is None else to_np(bias), bf16=bf, out_dtype=out,
                         rows=rows)


@contextlib.contextmanager
def deterministic():
    """torch.use_deterministic_algorithms(True) for the block (the library then
    passes ST_EXEC_DETERMINISTIC)."""
    prev = torch.are_deterministic_algorithms_enabled()
    torch.use_deterministic_algorithms(True)
    try:
        yield
    finally:
        torch.use_deterministic_algorithms(prev)


def kat(m, n, k, dtype):
    a = oracle.kat_values(m * k, 17, 8, 0.25).reshape(m, k)
    b = oracle.kat_values(k * n, 13, 6, 0.5).reshape(k, n)
    return torch.from_numpy(a).to(DEV, dtype), torch.from_numpy(b).to(DEV, dtype)


def normal(shape, std, seed, dtype):
    g = torch.Generator(device="cpu").manual_seed(seed)
    return (torch.randn(shape, generator=g) * std).to(dtype).to(DEV)


# ------------------------------------------------------------ known answers
@pytest.mark.parametrize("case", META["matmul"], ids=lambda c: c["file"])
def test_known_answers_through_drop_in_api(case):
    f = np.load(GOLD / case["file"])
    A, B = torch.from_numpy(f["a"]), torch.from_numpy(f["b"])
    C = st.spirv_matmul(A, B)  # host tensors, as the reference's main() (spirv_matmul.py:131-137)
    assert C.device.type == "cpu" and C.dtype == torch.float32
    assert C.numpy().tobytes() == f["expected"].tobytes()
    Cp = st.cutile_matmul_spirv(A, B, persistent=True)
    assert Cp.numpy().tobytes() == f["expected"].tobytes()


@pytest.mark.parametrize("case", META["matmul"], ids=lambda c: c["file"])
def test_known_answers_through_runner(case):
    f = np.load(GOLD / case["file"])
    m, n = case["m"], case["n"]
    params = [*st.tensor_2d_descriptor(f["a"]), *st.tensor_2d_descriptor(f["b"]),
              *st.tensor_2d_descriptor(np.zeros((m, n), np.float32))]
    out = st.run_tile_kernel(entry_name="matmul_fp32", parameter_arrays=params, output_indices=[10],
                             dispatch=tuple(case["dispatch"]))[0]
    assert out.reshape(m, n).tobytes() == f["expected"].tobytes()


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("mnk", [(64, 64, 64), (256, 256, 256), (100, 70, 33), (33, 129, 200), (1, 1, 1),
                                 (129, 257, 65), (1000, 24, 520)])
def test_known_answers_all_dtypes(dtype, mnk):
    m, n, k = mnk
    A, B = kat(m, n, k, dtype)
    C = st.matmul(A, B, out_dtype=torch.float32)
    assert C.cpu().numpy().tobytes() == oracle.matmul_kat_expected(m, n, k).tobytes()


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_known_answers_full_size_8192_cube(dtype):
    """The fp16 configuration's full size, every tile checked exactly."""
    A, B = kat(8192, 8192, 8192, dtype)
    C = st.matmul(A, B, out_dtype=torch.float32)
    want = torch.from_numpy(oracle.matmul_kat_expected(8192, 8192, 8192)).to(DEV)
    assert torch.equal(C, want)


def test_known_answers_full_size_bias_config():
    """M=32768, N=K=4096 bf16 with a fused bias: one rounding of (exact sum + bias)."""
    m, n, k = 32768, 4096, 4096
    A, B = kat(m, n, k, torch.bfloat16)
    g = torch.Generator(device="cpu").manual_seed(4)
    bias = (torch.rand(n, generator=g) * 2 - 1).to(torch.bfloat16)
    exact = torch.from_numpy(oracle.matmul_kat_expected(m, n, k)).to(DEV)
    want32 = exact + bias.to(DEV).float()  # fl(acc + bias), acc exact
    C32 = st.matmul(A, B, bias.to(DEV), out_dtype=torch.float32)
    bad = (C32 != want32).sum().item()
    assert bad == 0, f"{bad} elements differ, max |diff| {(C32 - want32).abs().max().item()}"
    Cbf = st.matmul(A, B, bias.to(DEV))  # C takes A's dtype (matmul.py:245)
    assert Cbf.dtype == torch.bfloat16
    assert torch.equal(Cbf, want32.to(torch.bfloat16))


# ------------------------------------------------------------ seeded random inputs
def test_config_fp32_1024_cube_3xtf32():
    A, B = normal((1024, 1024), 1.0, 2, torch.float32), normal((1024, 1024), 1.0, 20, torch.float32)
    C = st.matmul(A, B)
    want = oracle_mm(A, B)
    err = rel_err(C.cpu().numpy(), want)
    assert err <= 1e-3
    # 1xTF32 would land near 2e-4 here; 3xTF32 measures ~1.3e-5 (the tensor
    # core's fp32 accumulator does not round every add to nearest)
    assert err <= 5e-5, f"3xTF32 should be well below 1xTF32 error, got {err}"


def _sample_rows(m, block=128):
    rows = []
    for start in sorted({0, block, m // 2, m - block}):
        rows.append((max(0, start), min(m, start + 8)))
    return rows


def test_config_fp16_8192_cube_sampled_rows():
    m = n = k = 8192
    A, B = normal((m, k), 0.1, 3, torch.float16), normal((k, n), 0.1, 30, torch.float16)
    C = st.matmul(A, B, out_dtype=torch.float32)
    for r0, r1 in _sample_rows(m):
        want = oracle_mm(A, B, rows=(r0, r1))
        assert rel_err(C[r0:r1].cpu().numpy(), want) <= 1e-2 * 0.1  # far inside the 1e-2 bound


def fp64_product(A, B, bias=None):
    """C = A @ B (+ bias) in fp64 on the GPU from the same rounded inputs: every
    row of a full-size result checked against it (the oracle's row samples
    above pin the arithmetic; this covers the rest of C)."""
    C = A.double() @ B.double()
    if bias is not None:
        C += bias.double()
    return C


def full_rel_err(C, ref):
    return ((C.double() - ref).abs().max() / ref.abs().max()).item()


def test_config_fp16_8192_cube_every_row():
    m = n = k = 8192
    A, B = normal((m, k), 0.1, 3, torch.float16), normal((k, n), 0.1, 30, torch.float16)
    C = st.matmul(A, B, out_dtype=torch.float32)
    ref = fp64_product(A, B)
    assert torch.isfinite(C).all()
    # fp32 accumulation of 8192 products: ~1e-6 of max |C|; the bound is 1e-2
    assert full_rel_err(C, ref) <= 1e-4


def test_config_bf16_bias_every_row():
    m, n, k = 32768, 4096, 4096
    A, B = normal((m, k), 0.05, 4, torch.bfloat16), normal((k, n), 0.05, 40, torch.bfloat16)
    g = torch.Generator(device="cpu").manual_seed(41)
    bias = ((torch.rand(n, generator=g) * 2 - 1).to(torch.bfloat16)).to(DEV)
    ref = fp64_product(A, B, bias)
    C32 = st.matmul(A, B, bias, out_dtype=torch.float32)
    assert full_rel_err(C32, ref) <= 1e-4
    del C32
    Cbf = st.matmul(A, B, bias)  # C takes A's dtype (matmul.py:245)
    assert Cbf.dtype == torch.bfloat16
    assert full_rel_err(Cbf, ref) <= 1e-2
    # elementwise: one bf16 rounding of a sum that is fp32-accurate, so every
    # element is within one bf16 step (2^-8 relative) of the fp64 value
    d = (Cbf.double() - ref).abs()
    assert bool((d <= ref.abs() * 2.0 ** -8 + 1e-5 * ref.abs().max()).all())


def test_config_bf16_bias_sampled_rows():
    m, n, k = 32768, 4096, 4096
    A, B = normal((m, k), 0.05, 4, torch.bfloat16), normal((k, n), 0.05, 40, torch.bfloat16)
    g = torch.Generator(device="cpu").manual_seed(41)
    bias = ((torch.rand(n, generator=g) * 2 - 1).to(torch.bfloat16)).to(DEV)
    C = st.matmul(A, B, bias, out_dtype=torch.float32)
    Cbf = st.matmul(A, B, bias)
    for r0, r1 in _sample_rows(m):
        want = oracle_mm(A, B, bias, rows=(r0, r1))
        assert rel_err(C[r0:r1].cpu().numpy(), want) <= 1e-3
        wbf = oracle_mm(A, B, bias, rows=(r0, r1), out=oracle.BF16)
        got = to_np(Cbf[r0:r1])
        assert rel_err(oracle.bf16_bits_to_f32(got), oracle.bf16_bits_to_f32(wbf)) <= 1e-2


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("mnk", [(5, 7, 3), (129, 257, 65), (300, 200, 1000), (256, 512, 128), (77, 1000, 40),
                                 (1, 4096, 4096), (4096, 1, 300)])
def test_random_ragged_shapes(dtype, mnk):
    m, n, k = mnk
    A, B = normal((m, k), 1.0, m + n, dtype), normal((k, n), 1.0, k, dtype)
    C = st.matmul(A, B, out_dtype=torch.float32)
    assert rel_err(C.cpu().numpy(), oracle_mm(A, B)) <= TOL[dtype]


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
def test_operand_layouts(dtype):
    """Transposed B (K-major path), strided A and B (repack path), padded C rows."""
    m, n, k = 200, 136, 72
    A = normal((m, k), 1.0, 1, dtype)
    B = normal((k, n), 1.0, 2, dtype)
    want = oracle_mm(A, B)
    Bt = B.t().contiguous().t()  # column-major B
    assert rel_err(st.matmul(A, Bt, out_dtype=torch.float32).cpu().numpy(), want) <= TOL[dtype]
    Abig = normal((m, 2 * k), 1.0, 3, dtype)
    Abig[:, ::2] = A
    As = Abig[:, ::2]  # column stride 2
    Bbig = torch.zeros((k, n + 3), dtype=dtype, device=DEV)
    Bbig[:, :n] = B
    Bs = Bbig[:, :n]  # row stride not a multiple of 16 bytes
    out = torch.full((m, n + 8), 5.0, device=DEV)
    st.matmul(As, Bs, out=out[:, :n])
    assert rel_err(out[:, :n].cpu().numpy(), want) <= TOL[dtype]
    assert torch.all(out[:, n:] == 5.0)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("out_dtype", [torch.float32, torch.float16, torch.bfloat16])
def test_output_dtypes_and_bias(dtype, out_dtype):
    m, n, k = 384, 640, 256
    A, B = normal((m, k), 0.5, 5, dtype), normal((k, n), 0.5, 6, dtype)
    for bias_dtype in (torch.float32, dtype):
        bias = normal((n,), 1.0, 7, bias_dtype)
        C = st.matmul(A, B, bias, out_dtype=out_dtype)
        code = {torch.float32: oracle.F32, torch.float16: oracle.F16, torch.bfloat16: oracle.BF16}[out_dtype]
        want = oracle_mm(A, B, bias, out=code)
        got = to_np(C)
        if out_dtype == torch.bfloat16:
            got, want = oracle.bf16_bits_to_f32(got), oracle.bf16_bits_to_f32(want)
        assert rel_err(np.asarray(got, np.float32), np.asarray(want, np.float32)) <= 1e-2


def test_empty_contraction_gives_bias():
    A = torch.zeros((5, 0), device=DEV, dtype=torch.float16)
    B = torch.zeros((0, 7), device=DEV, dtype=torch.float16)
    bias = torch.arange(7, device=DEV, dtype=torch.float32)
    C = st.matmul(A, B, bias, out_dtype=torch.float32)
    assert torch.equal(C, bias.expand(5, 7))
    assert st.matmul(A, B, out_dtype=torch.float32).abs().sum() == 0


def _launch_matmul(entry, grid, A, B, C, consts=()):
    P = (N.StParam * (15 + len(consts)))()
    i = 0
    for t in (A, B, C):
        P[i].kind, P[i].dtype, P[i].data, P[i].bytes = N.ST_PARAM_BUFFER, st.api.dtype_code(t.dtype), \
            t.data_ptr(), t.numel() * t.element_size()
        vals = [t.shape[0], t.shape[1], t.stride(0), t.stride(1)]
        for j, v in enumerate(vals):
            P[i + 1 + j].kind, P[i + 1 + j].value = N.ST_PARAM_I32, v
        i += 5
    for c in consts:
        P[i].kind, P[i].value = N.ST_PARAM_I32, c
        i += 1
    g = N.StGrid(*grid)
    ex = N.StExec(torch.cuda.current_stream().cuda_stream, 0, N.ST_EXEC_SYNC, 60000, None, 0)
    N.check(N.lib().st_launch(st.context(0), entry.encode(), ctypes.byref(g), P, len(P), ctypes.byref(ex)), entry)


def test_persistent_entry_any_grid_and_grid_coverage_rule():
    m, n, k = 512, 384, 256
    A, B = kat(m, n, k, torch.float16)
    want = torch.from_numpy(oracle.matmul_kat_expected(m, n, k)).to(DEV)
    for grid in (1, 7, 148):
        C = torch.zeros((m, n), device=DEV)
        _launch_matmul("persistent_matmul_f16", (grid, 1, 1), A, B, C)
        assert torch.equal(C, want)
    C = torch.zeros((m, n), device=DEV)
    tiles = (m // 128) * -(-n // 256)
    _launch_matmul("matmul_f16", (tiles, 1, 1), A, B, C, consts=(128, 256, 64))
    assert torch.equal(C, want)
    with pytest.raises(NotImplementedError, match="cover"):
        _launch_matmul("matmul_f16", (tiles - 1, 1, 1), A, B, C, consts=(128, 256, 64))


def test_entry_dtype_mismatch_is_rejected():
    A, B = kat(64, 64, 64, torch.float16)
    C = torch.zeros((64, 64), device=DEV)
    with pytest.raises(ValueError, match="dtype"):
        _launch_matmul("matmul_bf16", (4, 1, 1), A, B, C)


# ------------------------------------------------------------ both kernel families
@pytest.mark.parametrize("family", ["single", "pair"])
@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16], ids=["f32", "f16", "bf16"])
@pytest.mark.parametrize("mnk", [(64, 64, 64), (100, 70, 33), (300, 520, 200), (1000, 24, 520), (513, 777, 129),
                                 (2048, 1536, 1024)])
def test_kernel_families_known_answers(monkeypatch, family, dtype, mnk):
    """One CTA per tile and CTA pairs (cta_group::2), each pinned by the override."""
    monkeypatch.setenv("SPTILES_B200_GEMM_KERNEL", family)
    m, n, k = mnk
    A, B = kat(m, n, k, dtype)
    C = st.matmul(A, B, out_dtype=torch.float32)
    assert C.cpu().numpy().tobytes() == oracle.matmul_kat_expected(m, n, k).tobytes()
    # the same B stored column-major takes the K-major operand path
    C2 = st.matmul(A, B.t().contiguous().t(), out_dtype=torch.float32)
    assert C2.cpu().numpy().tobytes() == oracle.matmul_kat_expected(m, n, k).tobytes()


@pytest.mark.parametrize("family", ["single", "pair"])
@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16], ids=["f32", "f16", "bf16"])
def test_kernel_families_random_with_bias(monkeypatch, family, dtype):
    monkeypatch.setenv("SPTILES_B200_GEMM_KERNEL", family)
    m, n, k = 700, 900, 640
    A, B = normal((m, k), 1.0, 70, dtype), normal((k, n), 1.0, 71, dtype)
    bias = normal((n,), 1.0, 72, torch.float32)
    C = st.matmul(A, B, bias, out_dtype=torch.float32)
    assert rel_err(C.cpu().numpy(), oracle_mm(A, B, bias)) <= TOL[dtype]


# ------------------------------------------------------------ host-memory calls
@pytest.mark.parametrize("pinned", [True, False])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16], ids=["f16", "bf16"])
def test_host_tensors_chunked_pipeline(pinned, dtype):
    """16-bit host operands go through the chunked copy-in / GEMM / copy-out pipeline."""
    m, n, k = 2600, 1100, 4104  # ~16 MB row chunks of A, whole 256-row tiles -> 1792 + 808 rows
    A, B = normal((m, k), 0.3, 90, dtype).cpu(), normal((k, n), 0.3, 91, dtype).cpu()
    bias = normal((n,), 1.0, 92, torch.float32).cpu()
    if pinned:
        A, B, bias = A.pin_memory(), B.pin_memory(), bias.pin_memory()
    C = st.matmul(A, B, bias, out_dtype=torch.float32)
    assert C.device.type == "cpu"
    Cd = st.matmul(A.to(DEV), B.to(DEV), bias.to(DEV), out_dtype=torch.float32)
    # the chunks and the one-call product split the partial last wave's K
    # blocks differently (stream-K), so only the fp32 summation order differs
    assert rel_err(C.numpy(), Cd.cpu().numpy()) <= 1e-5
    for r0, r1 in ((0, 8), (1784, 1800), (m - 8, m)):  # both chunks and the seam
        want = oracle_mm(A, B, bias, rows=(r0, r1))
        assert rel_err(C[r0:r1].numpy(), want) <= TOL[dtype]
    # padded host output rows; the same bits as a first call in deterministic mode
    with deterministic():
        C = st.matmul(A, B, bias, out_dtype=torch.float32)
        out = torch.full((m, n + 3), 7.0)
        st.matmul(A, B, bias, out=out[:, :n])
    assert torch.equal(out[:, :n], C) and torch.all(out[:, n:] == 7.0)


@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16], ids=["f32_out", "bf16_out"])
def test_host_tensors_row_and_column_blocks(out_dtype):
    """K = 16380 makes ~16 MB blocks of 512 rows of A / 512 columns of B: 3 row
    and 4 column blocks, 4 steps; K and N not multiples of 8 (padded device
    pitches), a padded host C."""
    m, n, k = 1300, 1700, 16380
    dtype = torch.bfloat16
    A, B = normal((m, k), 0.2, 95, dtype).cpu().pin_memory(), normal((k, n), 0.2, 96, dtype).cpu().pin_memory()
    bias = normal((n,), 1.0, 97, torch.float32).cpu()
    out = torch.full((m, n + 5), 3.0, dtype=out_dtype)
    C = st.matmul(A, B, bias, out=out[:, :n])
    assert torch.all(out[:, n:] == 3.0)
    Cd = st.matmul(A.to(DEV), B.to(DEV), bias.to(DEV), out_dtype=out_dtype).cpu()
    assert rel_err(C.float().numpy(), Cd.float().numpy()) <= (1e-5 if out_dtype == torch.float32 else 8e-3)
    for r0, r1 in ((0, 6), (509, 515), (1021, 1027), (m - 6, m)):  # the row-block seams
        want = oracle_mm(A, B, bias, rows=(r0, r1))
        assert rel_err(C[r0:r1].float().numpy(), want) <= TOL[dtype]
    for c0, c1 in ((509, 515), (1533, 1539), (n - 6, n)):  # the column-block seams
        assert rel_err(C[:, c0:c1].float().numpy(), Cd[:, c0:c1].float().numpy()) <= 8e-3


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16], ids=["f32", "f16"])
def test_calls_replay_from_a_cuda_graph(dtype):
    """Device-tensor calls issued inside torch.cuda.graph replay correctly."""
    m, n, k = 512, 384, 320
    A, B = kat(m, n, k, dtype)
    C = torch.zeros((m, n), device=DEV)
    st.matmul(A, B, out=C.to(dtype) if dtype != torch.float32 else C)  # warm-up sizes any workspace
    torch.cuda.synchronize()
    out = torch.zeros((m, n), device=DEV)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        st.matmul(A, B, out=out)
    out.fill_(-1.0)
    g.replay()
    torch.cuda.synchronize()
    assert out.cpu().numpy().tobytes() == oracle.matmul_kat_expected(m, n, k).tobytes()


# ------------------------------------------------------------ fp32: split in the kernel vs packed operands
FP32_PATHS = ["split", "pack", "fused"]


def fp32_path(monkeypatch, path):
    """pack: [hi|hi|lo] x [hi;lo;hi] packed in global memory, then one tf32
    GEMM (the default); split: the CTA-pair kernel splits raw fp32 tiles into
    tf32 hi / lo itself (opt-in; shapes whose plan is not CTA pairs still
    pack); fused: the opt-in one-CTA kernel that splits in shared memory."""
    monkeypatch.delenv("SPTILES_B200_FP32_FUSED", raising=False)
    monkeypatch.delenv("SPTILES_B200_FP32", raising=False)
    if path == "fused":
        monkeypatch.setenv("SPTILES_B200_FP32_FUSED", "1")
    elif path == "split":
        monkeypatch.setenv("SPTILES_B200_FP32", "split")


@pytest.mark.parametrize("path", FP32_PATHS)
@pytest.mark.parametrize("mnk", [(64, 64, 64), (100, 72, 36), (300, 520, 200), (1000, 24, 520), (516, 780, 132),
                                 (1024, 1024, 1024), (100, 70, 33), (2048, 2048, 512), (1536, 1000, 700),
                                 (4096, 2048, 96)])
def test_fp32_paths_known_answers(monkeypatch, path, mnk):
    fp32_path(monkeypatch, path)
    m, n, k = mnk
    A, B = kat(m, n, k, torch.float32)
    want = oracle.matmul_kat_expected(m, n, k).tobytes()
    assert st.matmul(A, B).cpu().numpy().tobytes() == want
    assert st.matmul(A, B.t().contiguous().t()).cpu().numpy().tobytes() == want  # column-major B


@pytest.mark.parametrize("path", FP32_PATHS)
def test_fp32_paths_random_accuracy(monkeypatch, path):
    fp32_path(monkeypatch, path)
    m, n, k = 768, 640, 1000
    A, B = normal((m, k), 1.0, 80, torch.float32), normal((k, n), 1.0, 81, torch.float32)
    bias = normal((n,), 1.0, 82, torch.float32)
    want = oracle_mm(A, B, bias)
    for Bv in (B, B.t().contiguous().t()):
        C = st.matmul(A, Bv, bias)
        err = rel_err(C.cpu().numpy(), want)
        assert err <= 5e-5, f"{path}: 3xTF32 error {err}"


@pytest.mark.parametrize("fold", ["ordered", "preset", "exchange", "whole"])
@pytest.mark.parametrize("mnk", [(1024, 1024, 1024), (2048, 3000, 700), (3000, 5000, 520)],
                         ids=lambda s: "x".join(map(str, s)))
def test_fp32_split_stream_k_folds(monkeypatch, fold, mnk):
    """The in-kernel split on every fold of split tiles (1024^3: every tile
    split; the others: whole-tile waves and a split last wave), against the
    packed route and the oracle, with a bias; N-contiguous and K-major B."""
    monkeypatch.setenv("SPTILES_B200_GEMM_KERNEL", "pair")
    fp32_path(monkeypatch, "split")
    if fold == "preset":
        monkeypatch.setenv("SPTILES_B200_SK_FOLD", "preset")
    elif fold == "exchange":
        monkeypatch.setenv("SPTILES_B200_SK_FOLD", "exchange")
        monkeypatch.setenv("SPTILES_B200_STREAM_K", "2")
    elif fold == "whole":
        monkeypatch.setenv("SPTILES_B200_STREAM_K", "0")
    m, n, k = mnk
    Ak, Bk = kat(m, n, k, torch.float32)
    want = oracle.matmul_kat_expected(m, n, k).tobytes()
    assert st.matmul(Ak, Bk).cpu().numpy().tobytes() == want
    assert st.matmul(Ak, Bk.t().contiguous().t()).cpu().numpy().tobytes() == want
    A, B = normal((m, k), 1.0, 83, torch.float32), normal((k, n), 1.0, 84, torch.float32)
    bias = normal((n,), 1.0, 85, torch.float32)
    C = st.matmul(A, B, bias)
    rows = (m - 64, m)
    assert rel_err(C[rows[0]:rows[1]].cpu().numpy(), oracle_mm(A, B, bias, rows=rows)) <= 5e-5
    assert full_rel_err(C, fp64_product(A, B, bias)) <= 5e-5
    fp32_path(monkeypatch, "pack")
    Cp = st.matmul(A, B, bias)
    assert rel_err(C.cpu().numpy(), Cp.cpu().numpy()) <= 5e-5


@pytest.mark.parametrize("out_dtype", [torch.float16, torch.bfloat16], ids=["f16", "bf16"])
def test_fp32_split_16bit_out(monkeypatch, out_dtype):
    fp32_path(monkeypatch, "split")
    m, n, k = 1024, 1536, 800
    A, B = normal((m, k), 1.0, 86, torch.float32), normal((k, n), 1.0, 87, torch.float32)
    bias = normal((n,), 1.0, 88, torch.float32)
    C = st.matmul(A, B, bias, out_dtype=out_dtype)
    ref = fp64_product(A, B, bias)
    assert full_rel_err(C, ref) <= 1e-2
    d = (C.double() - ref).abs()
    step = 2.0 ** -10 if out_dtype == torch.float16 else 2.0 ** -7  # one rounding step, relative
    assert bool((d <= ref.abs() * step + 1e-4 * ref.abs().max()).all())


def test_fp32_split_config_every_row_and_graph_replay(monkeypatch):
    """The fp32 configuration (1024^3, N(0, 1)): every element against fp64,
    the oracle on row samples, deterministic mode bit for bit, and a CUDA
    graph replay of the call."""
    fp32_path(monkeypatch, "split")
    A, B = normal((1024, 1024), 1.0, 2, torch.float32), normal((1024, 1024), 1.0, 20, torch.float32)
    C = st.matmul(A, B)
    assert full_rel_err(C, fp64_product(A, B)) <= 5e-5
    for r0, r1 in _sample_rows(1024):
        assert rel_err(C[r0:r1].cpu().numpy(), oracle_mm(A, B, rows=(r0, r1))) <= 5e-5
    with deterministic():
        d0, d1 = st.matmul(A, B), st.matmul(A, B)
    assert torch.equal(d0, d1)
    assert rel_err(d0.cpu().numpy(), C.cpu().numpy()) <= 5e-5
    out = torch.empty_like(C)
    st.matmul(A, B, out=out)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        st.matmul(A, B, out=out)
    for _ in range(3):
        out.fill_(float("nan"))
        g.replay()
        torch.cuda.synchronize()
        assert rel_err(out.cpu().numpy(), C.cpu().numpy()) <= 5e-5


# ------------------------------------------------------------ stream-K tail of the CTA-pair kernel
# Shapes with fewer 256 x 256 tiles than the 74 pairs, so the tiles' K blocks
# are split over more pairs and folded by each tile's owner (from ~1.2 to 4
# pieces per tile; ragged M and N; 8 to 64 K blocks per tile).
SK_SHAPES = [(1024, 4096, 1024), (256, 2048, 4096), (1000, 3000, 2000), (512, 8192, 512), (300, 520, 2000)]


@pytest.mark.parametrize("sk", ["1", "0"], ids=["stream_k", "whole_tiles"])
@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16], ids=["f32", "f16", "bf16"])
@pytest.mark.parametrize("mnk", SK_SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_stream_k_tail_known_answers(monkeypatch, sk, dtype, mnk):
    monkeypatch.setenv("SPTILES_B200_GEMM_KERNEL", "pair")
    monkeypatch.setenv("SPTILES_B200_STREAM_K", sk)
    m, n, k = mnk
    A, B = kat(m, n, k, dtype)
    C = st.matmul(A, B, out_dtype=torch.float32)
    assert C.cpu().numpy().tobytes() == oracle.matmul_kat_expected(m, n, k).tobytes()


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16], ids=["f16", "bf16"])
@pytest.mark.parametrize("mnk", SK_SHAPES[:3], ids=lambda s: "x".join(map(str, s)))
def test_stream_k_tail_random_bias_16bit_out(monkeypatch, dtype, mnk):
    monkeypatch.setenv("SPTILES_B200_GEMM_KERNEL", "pair")
    m, n, k = mnk
    A, B = normal((m, k), 0.5, 80, dtype), normal((k, n), 0.5, 81, dtype)
    bias = normal((n,), 1.0, 82, dtype)
    rows = (max(0, m - 300), m)  # the last rows: the stream-K tiles of the raster
    C = st.matmul(A, B, bias, out_dtype=dtype)
    want = oracle_mm(A, B, bias, rows=rows, out=oracle.BF16 if dtype == torch.bfloat16 else oracle.F16)
    got = to_np(C[rows[0]:rows[1]])
    if dtype == torch.bfloat16:
        got, want = oracle.bf16_bits_to_f32(got), oracle.bf16_bits_to_f32(want)
    assert rel_err(np.asarray(got, np.float32).reshape(-1), np.asarray(want, np.float32).reshape(-1)) <= TOL[dtype]
    monkeypatch.setenv("SPTILES_B200_STREAM_K", "0")
    C0 = st.matmul(A, B, bias, out_dtype=torch.float32)
    C1 = st.matmul(A, B, bias, out_dtype=torch.float32)  # default again below
    monkeypatch.setenv("SPTILES_B200_STREAM_K", "1")
    C1 = st.matmul(A, B, bias, out_dtype=torch.float32)
    # only the summation order of the split tiles differs
    assert rel_err(C1.cpu().numpy(), C0.cpu().numpy()) <= 1e-5


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16], ids=["f32", "f16", "bf16"])
@pytest.mark.parametrize("mnk", SK_SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_stream_k_exchange_fold_known_answers(monkeypatch, dtype, mnk):
    """fp32 C takes TMA reduce-adds by default; the workspace exchange (the
    fold of 16-bit C) is forced here for the same shapes."""
    monkeypatch.setenv("SPTILES_B200_GEMM_KERNEL", "pair")
    monkeypatch.setenv("SPTILES_B200_SK_FOLD", "exchange")
    m, n, k = mnk
    A, B = kat(m, n, k, dtype)
    C = st.matmul(A, B, out_dtype=torch.float32)
    assert C.cpu().numpy().tobytes() == oracle.matmul_kat_expected(m, n, k).tobytes()


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16], ids=["f32", "f16"])
@pytest.mark.parametrize("mnk", [(1024, 1024, 1024), (300, 520, 2000), (1000, 3000, 2000)],
                         ids=lambda s: "x".join(map(str, s)))
def test_stream_k_l2add_fold_random_bias(monkeypatch, dtype, mnk):
    """Every tile split: the units add onto C preset to the bias (by the fp32
    pack, or a preset kernel); agrees with whole tiles and with the exchange
    up to summation order, and with the oracle."""
    monkeypatch.setenv("SPTILES_B200_GEMM_KERNEL", "pair")
    m, n, k = mnk
    A, B = normal((m, k), 0.5, 90, dtype), normal((k, n), 0.5, 91, dtype)
    bias = normal((n,), 1.0, 92, torch.float32)
    C = st.matmul(A, B, bias, out_dtype=torch.float32)
    rows = (max(0, m - 256), m)
    want = oracle_mm(A, B, bias, rows=rows)
    assert rel_err(C[rows[0]:rows[1]].cpu().numpy(), want) <= (5e-5 if dtype == torch.float32 else TOL[dtype])
    monkeypatch.setenv("SPTILES_B200_SK_FOLD", "exchange")
    Cx = st.matmul(A, B, bias, out_dtype=torch.float32)
    monkeypatch.setenv("SPTILES_B200_STREAM_K", "0")
    C0 = st.matmul(A, B, bias, out_dtype=torch.float32)
    # 3xTF32 itself differs from fp32 by ~1e-5, and the split regroups its terms
    order_tol = 5e-5 if dtype == torch.float32 else 1e-5
    assert rel_err(C.cpu().numpy(), C0.cpu().numpy()) <= order_tol
    assert rel_err(Cx.cpu().numpy(), C0.cpu().numpy()) <= order_tol


# Shapes with whole-tile waves and a partial last wave (tiles >= pairs, more
# than 3 % of the pairs idle in the last wave).  With fp32 C the last wave's
# tiles are split over every pair by default and their units add onto C
# preset to the bias on those tiles only; the whole tiles are stored outright.
# (1024, 8192, 8192) is one rank's share of the fp16 configuration on 8 GPUs.
WAVE_TAIL_SHAPES = [(1024, 8192, 1024), (2048, 8192, 640), (1000, 8000, 700), (3000, 5000, 520),
                    (1024, 8192, 8192)]


@pytest.mark.parametrize("sk", ["ordered", "preset", "whole"])
@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16], ids=["f32", "f16", "bf16"])
@pytest.mark.parametrize("mnk", WAVE_TAIL_SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_stream_k_wave_tail_known_answers(monkeypatch, sk, dtype, mnk):
    """ordered: a split tile's first unit stores, the others add after its
    flags (the default); preset: C preset on the split tiles, every unit adds;
    whole: no split."""
    m, n, k = mnk
    if dtype == torch.float32 and k > 2048:
        pytest.skip("fp32 packs 3 K copies: the 8192-deep case is covered by the 16-bit inputs")
    monkeypatch.setenv("SPTILES_B200_GEMM_KERNEL", "pair")
    if sk == "preset":
        monkeypatch.setenv("SPTILES_B200_SK_FOLD", "preset")
    elif sk == "whole":
        monkeypatch.setenv("SPTILES_B200_STREAM_K", "1")
    A, B = kat(m, n, k, dtype)
    C = torch.full((m, n), float("nan"), device=DEV)
    st.matmul(A, B, out=C)
    assert C.cpu().numpy().tobytes() == oracle.matmul_kat_expected(m, n, k).tobytes()


@pytest.mark.parametrize("mnk", WAVE_TAIL_SHAPES[:4], ids=lambda s: "x".join(map(str, s)))
def test_stream_k_wave_tail_random_bias(monkeypatch, mnk):
    """The tail split with a bias (C preset to the bias on the split tiles)
    against whole tiles, the exchange fold and the oracle; 16-bit C keeps
    whole tiles and must match too."""
    monkeypatch.setenv("SPTILES_B200_GEMM_KERNEL", "pair")
    m, n, k = mnk
    A, B = normal((m, k), 0.5, 70, torch.float16), normal((k, n), 0.5, 71, torch.float16)
    bias = normal((n,), 1.0, 72, torch.float32)
    C = torch.full((m, n), float("nan"), device=DEV)
    st.matmul(A, B, bias, out=C)
    for rows in ((0, 64), (m - 64, m)):
        want = oracle_mm(A, B, bias, rows=rows)
        assert rel_err(C[rows[0]:rows[1]].cpu().numpy(), want) <= TOL[torch.float16]
    ref = fp64_product(A, B, bias)
    assert full_rel_err(C, ref) <= 1e-5
    monkeypatch.setenv("SPTILES_B200_SK_FOLD", "preset")
    Cp = torch.full((m, n), float("nan"), device=DEV)
    st.matmul(A, B, bias, out=Cp)  # every unit adds onto C preset to the bias
    assert rel_err(C.cpu().numpy(), Cp.cpu().numpy()) <= 1e-5
    monkeypatch.setenv("SPTILES_B200_SK_FOLD", "exchange")
    Cx = st.matmul(A, B, bias, out_dtype=torch.float32)  # exchange: mode 1, whole tiles here
    monkeypatch.delenv("SPTILES_B200_SK_FOLD")
    monkeypatch.setenv("SPTILES_B200_STREAM_K", "2")
    monkeypatch.setenv("SPTILES_B200_SK_FOLD", "exchange")
    C2x = st.matmul(A, B, bias, out_dtype=torch.float32)  # the tail split folded by exchange
    for other in (Cx, C2x):
        assert rel_err(C.cpu().numpy(), other.cpu().numpy()) <= 1e-5
    Ch = st.matmul(A, B, bias, out_dtype=torch.float16)
    assert full_rel_err(Ch, ref) <= 1e-2


def test_stream_k_wave_tail_replays_from_a_cuda_graph(monkeypatch):
    """The tail's preset kernel and the GEMM captured once and replayed."""
    monkeypatch.setenv("SPTILES_B200_GEMM_KERNEL", "pair")
    m, n, k = 1024, 8192, 1024
    A, B = kat(m, n, k, torch.float16)
    out = torch.zeros((m, n), device=DEV)
    st.matmul(A, B, out=out)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        st.matmul(A, B, out=out)
    want = oracle.matmul_kat_expected(m, n, k).tobytes()
    for _ in range(3):
        out.fill_(float("nan"))
        g.replay()
        torch.cuda.synchronize()
        assert out.cpu().numpy().tobytes() == want


@pytest.mark.parametrize("kernel", ["pair", "single"])
def test_k_order_alternation_matches_ascending_order(monkeypatch, kernel):
    """A CTA's odd-numbered tiles load K last to first (L2 reuse between
    consecutive tiles); only the summation order changes."""
    monkeypatch.setenv("SPTILES_B200_GEMM_KERNEL", kernel)
    m, n, k = 2048, 4096, 2048  # several tiles per CTA in both kernel families
    A, B = normal((m, k), 0.5, 60, torch.float16), normal((k, n), 0.5, 61, torch.float16)
    C = st.matmul(A, B, out_dtype=torch.float32)
    monkeypatch.setenv("SPTILES_B200_K_SNAKE", "0")
    C0 = st.matmul(A, B, out_dtype=torch.float32)
    assert rel_err(C.cpu().numpy(), C0.cpu().numpy()) <= 1e-5
    assert full_rel_err(C, fp64_product(A, B)) <= 1e-5
    Ak, Bk = kat(m, n, k, torch.float16)
    monkeypatch.delenv("SPTILES_B200_K_SNAKE")
    assert st.matmul(Ak, Bk, out_dtype=torch.float32).cpu().numpy().tobytes() == \
        oracle.matmul_kat_expected(m, n, k).tobytes()


@pytest.mark.parametrize("mnk", [(1024, 1024, 1024), (300, 520, 2000)], ids=lambda s: "x".join(map(str, s)))
def test_deterministic_mode_repeats_bit_for_bit(monkeypatch, mnk):
    """Split tiles with fp32 C: L2 adds by default (last-bit differences
    between runs allowed), a fixed-order fold under deterministic mode."""
    monkeypatch.setenv("SPTILES_B200_GEMM_KERNEL", "pair")
    m, n, k = mnk
    A, B = normal((m, k), 1.0, 95, torch.float32), normal((k, n), 1.0, 96, torch.float32)
    bias = normal((n,), 1.0, 97, torch.float32)
    runs = [st.matmul(A, B, bias) for _ in range(3)]
    for r in runs[1:]:
        assert rel_err(r.cpu().numpy(), runs[0].cpu().numpy()) <= 1e-6
    with deterministic():
        det = [st.matmul(A, B, bias) for _ in range(4)]
        host = st.matmul(A.cpu(), B.cpu(), bias.cpu())
    for r in det[1:]:
        assert torch.equal(r, det[0])
    assert rel_err(host.numpy(), det[0].cpu().numpy()) <= 1e-6
    assert rel_err(det[0].cpu().numpy(), runs[0].cpu().numpy()) <= 5e-5


def test_stream_k_l2add_fold_strided_out_and_graph_replay(monkeypatch):
    """fp32 1024^3: C preset and reduced in place inside a wider buffer (only
    the [m, n] view changes), captured once and replayed."""
    monkeypatch.setenv("SPTILES_B200_GEMM_KERNEL", "pair")
    m, n, k = 1024, 1000, 1024
    A, B = kat(m, n, k, torch.float32)
    buf = torch.full((m, n + 24), 7.0, device=DEV)
    out = buf[:, :n]
    st.matmul(A, B, out=out)
    torch.cuda.synchronize()
    want = oracle.matmul_kat_expected(m, n, k)
    assert np.array_equal(out.cpu().numpy(), want) and torch.all(buf[:, n:] == 7.0)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        st.matmul(A, B, out=out)
    for _ in range(3):
        out.fill_(-1.0)
        g.replay()
        torch.cuda.synchronize()
        assert np.array_equal(out.cpu().numpy(), want) and torch.all(buf[:, n:] == 7.0)


def test_stream_k_tail_replays_from_a_cuda_graph(monkeypatch):
    monkeypatch.setenv("SPTILES_B200_GEMM_KERNEL", "pair")
    m, n, k = 1024, 8192, 1024
    A, B = kat(m, n, k, torch.float16)
    out = torch.zeros((m, n), device=DEV)
    st.matmul(A, B, out=out)  # warm-up: allocates the stream-K workspace
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        st.matmul(A, B, out=out)
    want = oracle.matmul_kat_expected(m, n, k).tobytes()
    for _ in range(3):  # the flags clear themselves between replays
        out.fill_(-1.0)
        g.replay()
        torch.cuda.synchronize()
        assert out.cpu().numpy().tobytes() == want


# ------------------------------------------------------------ bounded host waits
def test_bounded_host_wait_times_out_then_the_work_completes():
    """st_sync with a 1 ms limit on ~15 ms of queued GEMMs returns
    ST_ERR_TIMEOUT (TimeoutError) without disturbing the GPU; a later wait
    completes and the results are exact."""
    ctx = st.context(0)
    sp = ctypes.c_void_p()
    N.check(N.lib().st_stream(ctx, 0, ctypes.byref(sp)), "st_stream")
    s = torch.cuda.ExternalStream(sp.value, device=DEV)
    m, n, k = 8192, 8192, 8192
    A, B = kat(m, n, k, torch.float16)
    C = torch.zeros((m, n), device=DEV)
    torch.cuda.synchronize()
    with torch.cuda.stream(s):
        for _ in range(20):
            st.matmul(A, B, out=C)
    with pytest.raises(TimeoutError):
        st.sync(0, timeout_ms=1)
    st.sync(0, timeout_ms=60000)
    assert C.cpu().numpy().tobytes() == oracle.matmul_kat_expected(m, n, k).tobytes()
    with torch.cuda.stream(s):
        C.zero_()
        st.matmul(A, B, out=C)
    st.sync(0, timeout_ms=60000)
    assert C.cpu().numpy().tobytes() == oracle.matmul_kat_expected(m, n, k).tobytes()
