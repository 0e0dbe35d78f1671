"""The reference's host-side tests (examples.cpp: run_vector_add_test,
run_matmul_test) as a C++ program over the C ABI, with no Python in the
loop: built with g++ against include/sptiles_b200.h and the in-tree library,
run on the GPU (known answers, bit for bit; also through the entries of
cuda_tile modules) and, without one, checked to fail cleanly at st_init."""
import shutil
import subprocess
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parent.parent
SRC = ROOT / "tests" / "c_abi" / "run_compute_example.cpp"
LIB = ROOT / "sptiles_b200" / "libsptiles_b200.so"


def build(tmp_path: Path) -> Path:
    gxx = shutil.which("g++")
    if gxx is None or not LIB.exists():
        pytest.skip("needs g++ and the built library")
    exe = tmp_path / "run_compute_example"
    subprocess.run([gxx, "-std=c++17", "-O2", "-Wall", "-Werror", f"-I{ROOT / 'include'}", str(SRC),
                    f"-L{LIB.parent}", "-lsptiles_b200", f"-Wl,-rpath,{LIB.parent}", "-o", str(exe)],
                   check=True, timeout=300)
    return exe


def test_example_builds_and_fails_cleanly_without_a_gpu(tmp_path):
    exe = build(tmp_path)
    if torch.cuda.is_available():
        pytest.skip("a GPU is present; the GPU test runs the program")
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 2, r.stdout + r.stderr
    assert "no CUDA device" in r.stderr
    assert r.stdout.startswith("library ")


@pytest.mark.gpu
def test_example_runs_the_reference_tests_on_the_gpu(tmp_path):
    exe = build(tmp_path)
    modules = [str(ROOT / "tests" / "golden" / f) for f in ("vector_add.tilebc", "vector_add2D.tilebc",
                                                             "matmul.tilebc", "matmul_multi.tilebc")]
    r = subprocess.run([str(exe), *modules], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    out = r.stdout
    for line in ("vector_add n=1024 ok", "vector_add n=4112 ok", "matmul_fp32 64x64x64 ok",
                 "matmul_fp32 33x129x200 ok", "module vector_add tile=16 n=4112 ok",
                 "module vector_add tile=512 n=4112 ok", "module matmul_fp32 tiles=32x32x32 ok",
                 "entry matmul_f16: 15 bindings, 3 arrays, backend matmul_f16",
                 f"partitioner matmul_fp32 1000x700x333 on {torch.cuda.device_count()} devices ok",
                 f"partitioner vector_add n=1000003 on {torch.cuda.device_count()} devices ok", "all checks passed"):
        assert line in out, out
