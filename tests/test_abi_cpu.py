"""C ABI checks that need no GPU: the library loads, exports every symbol
include/sptiles_b200.h declares, and its host-side policy (tile raster, tile
plan, shard ranges, dispatch conversion, argument validation) behaves.
No kernel is launched here."""
import ctypes
import json
import re
from pathlib import Path

import numpy as np
import pytest
import torch

import sptiles_b200 as st
from sptiles_b200 import _native as N

ROOT = Path(__file__).resolve().parents[1]
GOLD = ROOT / "tests" / "golden"
META = json.loads((GOLD / "golden.json").read_text())


def header_symbols():
    text = (ROOT / "include" / "sptiles_b200.h").read_text()
    return sorted(set(re.findall(r"^\s*(?:const\s+char\s*\*|int)\s*(st_\w+)\s*\(", text, re.M)))


def test_library_builds_in_tree_and_loads():
    assert N.LIB_PATH.exists(), "run python -m sptiles_b200.build"
    L = N.lib()
    assert L.st_version().decode().startswith("sptiles_b200")


def test_every_header_symbol_is_exported():
    syms = header_symbols()
    assert len(syms) >= 20
    L = N.lib()
    missing = [s for s in syms if not hasattr(L, s)]
    assert not missing, missing
    assert sorted(N.EXPORTED) == syms


def test_device_count_does_not_fail_without_gpu():
    n = st.device_count()
    assert n >= 0


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-GPU error path")
def test_init_without_gpu_reports_no_device():
    h = ctypes.c_void_p()
    rc = N.lib().st_init(None, 0, ctypes.byref(h))
    assert rc == N.ST_ERR_NO_DEVICE
    assert "device" in N.last_error()


@pytest.mark.parametrize("sw", META["swizzle"], ids=lambda s: f"{s['M']}x{s['N']}_{s['tm']}x{s['tn']}")
def test_tile_raster_matches_reference_swizzle(sw):
    """GROUP_SIZE_M=8 raster against swizzle_2d_from_bid of matmul.py:14-24."""
    M, N_, tm, tn = sw["M"], sw["N"], sw["tm"], sw["tn"]
    for bid, (bm, bn) in enumerate(zip(sw["bid_m"], sw["bid_n"])):
        assert st.tile_raster(M, N_, tm, tn, 8, bid) == (bm, bn)
    # a bijection onto the tile grid
    pairs = set(zip(sw["bid_m"], sw["bid_n"]))
    assert len(pairs) == len(sw["bid_m"]) == (-(-M // tm)) * (-(-N_ // tn))


def test_tile_raster_rejects_bad_arguments():
    with pytest.raises(ValueError):
        st.tile_raster(0, 10, 32, 32, 8, 0)
    with pytest.raises(ValueError):
        st.tile_raster(64, 64, 32, 32, 8, 4)


@pytest.mark.parametrize("dt,m,n,k", [(N.ST_F16, 8192, 8192, 8192), (N.ST_BF16, 32768, 4096, 4096),
                                      (N.ST_F32, 1024, 1024, 1024), (N.ST_F16, 1024, 8192, 8192),
                                      (N.ST_F16, 100, 70, 33), (N.ST_BF16, 4096, 4096, 4096)])
def test_matmul_plan_is_sane(dt, m, n, k):
    p = st.matmul_plan(dt, m, n, k, 148)
    assert (p["block_m"], p["block_n"]) in ((128, 64), (128, 128), (128, 256), (256, 256))
    assert p["block_k"] * (4 if dt == N.ST_F32 else 2) == 128
    tiles = -(-m // p["block_m"]) * -(-n // p["block_n"])
    if p["block_m"] == 256:  # CTA pairs: two CTAs per tile, at most 74 pairs
        kb = -(-k // 64) if dt != N.ST_F32 else 3 * -(-k // 32)  # fp32: 3 x K rounded to 32, 32-deep blocks
        dp, skp, _ = st.stream_k_split(tiles, 74, kb)
        if skp == 0:
            assert p["ctas"] == 2 * min(tiles, 74)
        else:  # a stream-K tail: all pairs, or exactly the split's pairs when no tile goes out whole
            assert p["ctas"] == 2 * (74 if dp > 0 else skp)
    else:
        assert p["ctas"] == min(tiles, 148)
    assert 2 <= p["stages"] <= 8


def test_matmul_plan_headline_shapes():
    big = st.matmul_plan(N.ST_F16, 8192, 8192, 8192)
    assert (big["block_m"], big["block_n"], big["ctas"]) == (256, 256, 148)  # CTA pairs
    # a small fp32 problem spreads over more SMs with narrower tiles
    assert st.matmul_plan(N.ST_F32, 1024, 1024, 1024)["ctas"] >= 64


def test_kernel_family_override(monkeypatch):
    monkeypatch.setenv("SPTILES_B200_GEMM_KERNEL", "single")
    assert st.matmul_plan(N.ST_F16, 8192, 8192, 8192)["block_m"] == 128
    monkeypatch.setenv("SPTILES_B200_GEMM_KERNEL", "pair")
    assert st.matmul_plan(N.ST_F32, 100, 70, 33)["block_m"] == 256


@pytest.mark.parametrize("total,count,align", [(8192, 8, 128), (8192, 3, 128), (100, 4, 4), (5, 8, 4),
                                               (32768, 8, 128), (0, 2, 1), (2 ** 20 + 3, 7, 4)])
def test_shard_ranges_partition_the_range(total, count, align):
    spans = [st.shard_range(total, count, r, align) for r in range(count)]
    assert spans[0][0] == 0 and spans[-1][1] == total
    for (b0, e0), (b1, e1) in zip(spans, spans[1:]):
        assert e0 == b1
    for b, e in spans:
        assert b <= e
        assert b % align == 0 or b == total
    sizes = [e - b for b, e in spans]
    assert max(sizes) - min(sizes) <= align


def test_shard_range_rejects_bad_rank():
    with pytest.raises(ValueError):
        st.shard_range(10, 2, 2, 1)


@pytest.mark.parametrize("case", META["vector_add"] + META["matmul"], ids=lambda c: c["file"])
def test_grid_from_reference_dispatch(case):
    if "size" in case:
        # vector_add with 1024-element tiles: one tile per workgroup
        assert st.grid_from_dispatch("vector_add", case["dispatch"], 1024) == (case["dispatch"][0], 1, 1)
        # the exported 16-element tile: 64 tiles per workgroup
        assert st.grid_from_dispatch("vector_add", case["dispatch"], 16)[0] == case["dispatch"][0] * 64
    else:
        tiles = -(-case["m"] // 32) * -(-case["n"] // 32)
        assert st.grid_from_dispatch("matmul_fp32", case["dispatch"], 32 * 32) == (tiles, 1, 1)


def test_unknown_entry_is_reported_before_any_device_work():
    g = N.StGrid(1, 1, 1)
    rc = N.lib().st_launch(None, b"no_such_kernel", ctypes.byref(g), None, 0, None)
    assert rc == N.ST_ERR_UNKNOWN_ENTRY
    assert "no_such_kernel" in N.last_error()


def test_launch_without_context_is_rejected():
    g = N.StGrid(1, 1, 1)
    rc = N.lib().st_launch(None, b"vector_add", ctypes.byref(g), None, 0, None)
    assert rc == N.ST_ERR_INVALID_ARGUMENT


def test_python_api_validation_matches_reference_messages():
    a = torch.zeros(32)
    with pytest.raises(ValueError, match="same shape"):
        st.spirv_vector_add(a, torch.zeros(16))
    with pytest.raises(ValueError, match="must be a 1D tensor"):
        st.spirv_vector_add(torch.zeros(4, 4), torch.zeros(4, 4))
    with pytest.raises(ValueError, match="f32-only"):
        st.spirv_vector_add(a.half(), a.half())
    with pytest.raises(ValueError, match="divisible by 16"):
        st.spirv_vector_add(torch.zeros(24), torch.zeros(24))
    with pytest.raises(ValueError, match="Incompatible matrices"):
        st.spirv_matmul(torch.zeros(4, 5), torch.zeros(6, 4))
    with pytest.raises(ValueError, match="f32-only"):
        st.spirv_matmul(torch.zeros(4, 4).half(), torch.zeros(4, 4).half())
    with pytest.raises(ValueError, match="CUDA device"):
        st.cutile_matmul(torch.zeros(4, 4), torch.zeros(4, 4))


def test_descriptors_match_reference_layout():
    x = np.arange(12, dtype=np.float32).reshape(3, 4)
    d2 = st.tensor_2d_descriptor(x)
    assert [int(v[0]) for v in d2[1:]] == [3, 4, 4, 1]
    d1 = st.tensor_1d_descriptor(np.arange(7, dtype=np.float32))
    assert [int(v[0]) for v in d1[1:]] == [7, 1]


def test_device_wait_check_rejects_bad_arguments_before_device_work():
    ex = N.StExec(None, 0, N.ST_EXEC_SYNC, 1000, None, 0)
    for kind, limit in ((2, 1000), (-1, 1000), (0, 0), (1, 10_000_001)):
        assert N.lib().st_check_device_wait(None, kind, limit, ctypes.byref(ex)) == N.ST_ERR_INVALID_ARGUMENT
        assert "st_check_device_wait" in N.last_error()


def test_all_devices_flag_is_refused_where_it_does_not_apply():
    ex = N.StExec(None, -1, N.ST_EXEC_ALL_DEVICES, 1000, None, 0)
    t = N.StTensor()
    g = N.StGrid(1, 1, 1)
    calls = [
        lambda: N.lib().st_vector_add(None, ctypes.byref(t), ctypes.byref(t), ctypes.byref(t), ctypes.byref(ex)),
        lambda: N.lib().st_matmul(None, ctypes.byref(t), ctypes.byref(t), None, ctypes.byref(t), ctypes.byref(ex)),
        lambda: N.lib().st_launch(None, b"vector_add", ctypes.byref(g), None, 0, ctypes.byref(ex)),
        lambda: N.lib().st_cast(None, ctypes.byref(t), ctypes.byref(t), ctypes.byref(ex)),
    ]
    for call in calls:
        assert call() == N.ST_ERR_INVALID_ARGUMENT
        assert "ST_EXEC_ALL_DEVICES applies to" in N.last_error()
