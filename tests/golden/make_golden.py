"""Generate the golden fixtures in this folder from the reference's own Python code.

Run in a container where the reference tree is mounted (it is read, never
written):

    python tests/golden/make_golden.py <path of the reference tree>

What is taken from the reference, unmodified, by import:
  * shaders/spirv_runtime.py: LOCAL_SIZE_X, ceil_div, tensor_1d_descriptor,
    tensor_2d_descriptor (the cutile_python_v1 argument layout).  The module
    imports the Kompute package ``kp`` at import time, which is not installed;
    a placeholder module is put in ``sys.modules`` so the import succeeds --
    none of the Kompute-backed functions is called.
  * shaders/spirv_vector_add.py: VECTOR_ADD_TILE_SIZE, _vector_add_dispatch,
    and the known-answer inputs of its main() (arange(size), arange(1000, ...)).
  * shaders/spirv_matmul.py: MATMUL_TILE_M/N, _matmul_dispatch, _demo_values.
  * shaders/matmul.py: swizzle_2d_from_bid (the GROUP_SIZE_M raster of the
    cuTile matmul kernel), evaluated on plain Python integers.

The expected outputs are what the reference's own tests compare against:
``A + B`` (spirv_vector_add.py:107-108) and ``A @ B`` (spirv_matmul.py:135-136),
computed by torch on the CPU.  For these inputs both are exact in fp32.
The fixtures are small .npz files; the GPU box never reads the reference.
"""
from __future__ import annotations

import json
import sys
import types
from pathlib import Path

import numpy as np

OUT = Path(__file__).resolve().parent


def _import_reference(ref_root: Path):
    shaders = ref_root / "shaders"
    sys.path.insert(0, str(shaders))
    if "kp" not in sys.modules:
        sys.modules["kp"] = types.ModuleType("kp")  # placeholder: never used
    import spirv_runtime  # noqa: E402
    import spirv_vector_add  # noqa: E402
    import spirv_matmul  # noqa: E402
    try:
        import matmul as cutile_matmul  # noqa: E402  (needs the cuda.tile package)
    except Exception:  # pragma: no cover - only when cuda.tile is absent
        cutile_matmul = None
    return spirv_runtime, spirv_vector_add, spirv_matmul, cutile_matmul


def main(ref_root: str) -> None:
    import torch

    rt, va, mm, ct_mm = _import_reference(Path(ref_root))
    meta = {
        "LOCAL_SIZE_X": rt.LOCAL_SIZE_X,
        "VECTOR_ADD_TILE_SIZE": va.VECTOR_ADD_TILE_SIZE,
        "MATMUL_TILE_M": mm.MATMUL_TILE_M,
        "MATMUL_TILE_N": mm.MATMUL_TILE_N,
        "vector_add_output_index": 6,
        "matmul_output_index": 10,
        "vector_add": [],
        "matmul": [],
        "swizzle": [],
    }

    # vector_add known answers: sizes of examples.cpp:707-709 (1024), the
    # README and argparse default (2048), and a multi-workgroup size.
    for size in (1024, 2048, 4096 + 16):
        A = torch.arange(size, dtype=torch.float32)
        B = torch.arange(1000, 1000 + size, dtype=torch.float32)
        expected = (A + B).numpy()
        params = [*rt.tensor_1d_descriptor(A.numpy()), *rt.tensor_1d_descriptor(B.numpy()),
                  *rt.tensor_1d_descriptor(np.zeros(size, dtype=np.float32))]
        name = f"vector_add_{size}.npz"
        np.savez_compressed(OUT / name, a=A.numpy(), b=B.numpy(), expected=expected,
                            scalars=np.array([int(p[0]) for i, p in enumerate(params) if i % 3], dtype=np.int64))
        meta["vector_add"].append({
            "file": name, "size": size,
            "dispatch": list(va._vector_add_dispatch(size)),
            "n_params": len(params),
            "param_kinds": ["buffer" if i % 3 == 0 else "i32" for i in range(len(params))],
        })

    # matmul known answers: examples.cpp:712-714 default (64^3), the README
    # size (256^3), and ragged shapes that exercise zero-padded edge tiles.
    for (m, n, k) in ((64, 64, 64), (256, 256, 256), (100, 70, 33), (33, 129, 200)):
        A = mm._demo_values(m * k, 17, 8, 0.25).reshape(m, k)
        B = mm._demo_values(k * n, 13, 6, 0.5).reshape(k, n)
        expected = (A @ B).numpy()
        params = [*rt.tensor_2d_descriptor(A.numpy()), *rt.tensor_2d_descriptor(B.numpy()),
                  *rt.tensor_2d_descriptor(np.zeros((m, n), dtype=np.float32))]
        name = f"matmul_{m}x{n}x{k}.npz"
        scalars = np.array([int(p[0]) for i, p in enumerate(params) if i % 5], dtype=np.int64)
        np.savez_compressed(OUT / name, a=A.numpy(), b=B.numpy(), expected=expected, scalars=scalars)
        meta["matmul"].append({
            "file": name, "m": m, "n": n, "k": k,
            "dispatch": list(mm._matmul_dispatch(m, n)),
            "n_params": len(params),
            "param_kinds": ["buffer" if i % 5 == 0 else "i32" for i in range(len(params))],
        })

    # GROUP_SIZE_M = 8 tile raster of matmul.py:14-24, over every tile id.
    if ct_mm is not None:
        for (M, N, tm, tn) in ((1024, 1024, 128, 256), (1000, 700, 32, 32), (8192, 8192, 128, 256),
                               (300, 5000, 128, 128), (64, 64, 32, 32)):
            tiles = -(-M // tm) * -(-N // tn)
            pairs = [ct_mm.swizzle_2d_from_bid(M, N, tm, tn, 8, bid) for bid in range(tiles)]
            meta["swizzle"].append({"M": M, "N": N, "tm": tm, "tn": tn,
                                    "bid_m": [int(p[0]) for p in pairs], "bid_n": [int(p[1]) for p in pairs]})

    (OUT / "golden.json").write_text(json.dumps(meta, indent=1) + "\n")
    print(f"wrote fixtures to {OUT}")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <path of the reference tree>")
    main(sys.argv[1])
