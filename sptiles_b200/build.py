"""Build recipe of the native library (nvcc, sm_100a only).

    python -m sptiles_b200.build          # writes sptiles_b200/libsptiles_b200.so

The library is built in-tree so that it travels with the source tree; the
CUDA runtime is linked statically, and the driver's tensor-map encoder is
resolved at run time, so the .so needs nothing but libcuda at load time.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB = PKG / "libsptiles_b200.so"
SOURCES = ["runtime.cu", "vecadd.cu", "elementwise.cu", "gemm.cu", "pack.cu", "noalloc.cu", "module.cu", "diag.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    exe = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(exe).exists():
        raise RuntimeError("nvcc not found: the sm_100a library cannot be built")
    return exe


def command(out: Path = LIB, extra: list[str] | None = None) -> list[str]:
    return [nvcc(), *ARCH, "-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-O3",
            "-Xptxas", "-O3", "--expt-relaxed-constexpr", "-shared", "-cudart", "static",
            f"-I{ROOT / 'include'}", *(extra or []), "-o", str(out), *[str(CSRC / s) for s in SOURCES]]


def stale() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    deps = [CSRC / s for s in SOURCES] + list(CSRC.glob("*.h")) + list(CSRC.glob("*.cuh")) + \
        [ROOT / "include" / "sptiles_b200.h"]
    return any(d.stat().st_mtime > t for d in deps if d.exists())


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not stale():
        return LIB
    cmd = command()
    if verbose:
        print(" ".join(cmd), flush=True)
    tmp = LIB.with_suffix(".so.tmp")
    cmd[cmd.index("-o") + 1] = str(tmp)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
    print(f"built {LIB}")
