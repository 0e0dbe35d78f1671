"""Build the cuda_tile module fixtures (TileIR bytecode, .tilebc) in this folder
from the reference's own cuTile kernels.

Run in a container where the reference tree is mounted (it is read, never
written) and the cuda.tile package is installed (1.3.0 was used):

    python tests/golden/make_tilebc.py <path of the reference tree>

Every module is produced here, from source, by cuda.tile's bytecode export:

  * vector_add.tilebc, vector_add2D.tilebc, matmul.tilebc -- the reference's
    own ``compile_only()`` of shaders/vecadd.py, shaders/vecadd2.py and
    shaders/matmul.py, unmodified (tile 16; tile 16 x 32 loaded as 512
    contiguous elements; fp32 32 x 32 x 32, symbol matmul_fp32);
  * further modules from the same kernels and the reference's signature
    helpers (``make_matmul_signature``, ``make_contiguous_2d_constraint``):
    the configurations' tile sizes (vector_add tile 1024, matmul 128 x 256 x
    64), f16 / bf16 operands with an f32 C, the persistent kernel, several
    entries in one module, and two fp32 entries whose tile sizes cannot be
    told apart from the module alone.

The kernel files are executed under the relative names ``shaders/<file>``
so that no path of the generating machine lands in the modules' debug
information.  ``tilebc_expected.json`` records, per module, what the
script asked the exporter for -- symbols, array ranks and element types,
tile sizes, sm_100 hints -- and the backend kernel each entry maps to; the
reader under test (st_module_load) must recover exactly that.
"""
from __future__ import annotations

import json
import linecache
import os
import sys
import tempfile
import types
from pathlib import Path

OUT = Path(__file__).resolve().parent


def load_kernel_file(ref_root: Path, stem: str) -> types.ModuleType:
    """Execute shaders/<stem>.py of the reference as a module named by its relative path."""
    src = (ref_root / "shaders" / f"{stem}.py").read_text()
    rel = f"shaders/{stem}.py"
    # inspect (used by cuTile to read kernel source) accepts a file name that is in linecache
    linecache.cache[rel] = (len(src), None, src.splitlines(True), rel)
    mod = types.ModuleType(stem)
    mod.__file__ = rel
    sys.modules[stem] = mod
    # dont_inherit: this file's __future__ annotations must not turn the kernels' into strings
    exec(compile(src, rel, "exec", dont_inherit=True), mod.__dict__)
    return mod


def export(ct, ct_compilation, kernel, signatures, path: Path) -> None:
    ct_compilation.export_kernel(kernel, signatures=signatures, output_file=str(path), gpu_code="sm_100",
                                 output_format="tileir_bytecode", bytecode_version="13.1")


def vector_signature(ct, ct_compilation, tile_size: int, constants: list[int], symbol: str):
    arr = ct_compilation.ArrayConstraint(
        ct.float32, 1, index_dtype=ct.int32, stride_lower_bound_incl=0, alias_groups=[],
        may_alias_internally=False, stride_constant=(1,), shape_divisible_by=tile_size, base_addr_divisible_by=1)
    return ct_compilation.KernelSignature(parameters=[arr, arr, arr, *constants],
                                          calling_convention=ct_compilation.CallingConvention.cutile_python_v1(),
                                          symbol=symbol)


def matmul_mixed_signature(ct, ct_compilation, mm, in_dtype, out_dtype, tm, tn, tk, symbol):
    a = mm.make_contiguous_2d_constraint(in_dtype)
    c = mm.make_contiguous_2d_constraint(out_dtype)
    return ct_compilation.KernelSignature(parameters=[a, a, c, tm, tn, tk],
                                          calling_convention=ct_compilation.CallingConvention.cutile_python_v1(),
                                          symbol=symbol)


def entry(symbol, arrays, constants, backend, num_cta_in_cga=0):
    n_params = sum(1 + 2 * rank for rank, _ in arrays)
    return {"name": symbol, "n_params": n_params, "arrays": [list(a) for a in arrays],
            "constants": list(constants), "backend_entry": backend, "num_cta_in_cga": num_cta_in_cga,
            "occupancy": 0}


def main(ref_root: str) -> None:
    ref = Path(ref_root)
    import cuda.tile as ct
    import cuda.tile.compilation as ct_compilation

    vecadd = load_kernel_file(ref, "vecadd")
    vecadd2 = load_kernel_file(ref, "vecadd2")
    mm = load_kernel_file(ref, "matmul")
    f32, f16, bf16 = "f32", "f16", "bf16"
    expected = {}
    cwd = os.getcwd()
    with tempfile.TemporaryDirectory(dir=OUT) as tmp:
        os.chdir(tmp)
        try:
            # the reference's own exports, as its compile_only() functions write them
            for mod, name in ((vecadd, "vector_add.tilebc"), (vecadd2, "vector_add2D.tilebc"),
                              (mm, "matmul.tilebc")):
                mod.compile_only()
                (OUT / name).write_bytes(Path(tmp, name).read_bytes())
        finally:
            os.chdir(cwd)
    expected["vector_add.tilebc"] = [entry("vector_add", [(1, f32)] * 3, [16], "vector_add")]
    expected["vector_add2D.tilebc"] = [entry("vector_add", [(1, f32)] * 3, [16 * 32], "vector_add")]
    expected["matmul.tilebc"] = [entry("matmul_fp32", [(2, f32)] * 3, [32, 32, 32], "matmul_fp32", 2)]

    # the configurations' tile sizes
    export(ct, ct_compilation, vecadd.vector_add, [vector_signature(ct, ct_compilation, 1024, [1024], "vector_add")],
           OUT / "vector_add_tile1024.tilebc")
    expected["vector_add_tile1024.tilebc"] = [entry("vector_add", [(1, f32)] * 3, [1024], "vector_add")]

    export(ct, ct_compilation, mm.matmul_kernel,
           [matmul_mixed_signature(ct, ct_compilation, mm, ct.float16, ct.float32, 128, 256, 64, "matmul_f16")],
           OUT / "matmul_f16_f32out.tilebc")
    expected["matmul_f16_f32out.tilebc"] = [
        entry("matmul_f16", [(2, f16), (2, f16), (2, f32)], [128, 256, 64], "matmul_f16", 2)]

    export(ct, ct_compilation, mm.persistent_matmul_kernel,
           [mm.make_matmul_signature(ct.bfloat16, 128, 256, 64, "persistent_matmul_bf16")],
           OUT / "persistent_matmul_bf16.tilebc")
    expected["persistent_matmul_bf16.tilebc"] = [
        entry("persistent_matmul_bf16", [(2, bf16)] * 3, [128, 256, 64], "persistent_matmul_bf16")]

    # several entries in one module: each entry's operand types pick its tiles
    export(ct, ct_compilation, mm.matmul_kernel,
           [mm.make_matmul_signature(ct.float32, 32, 32, 32, "matmul_fp32"),
            mm.make_matmul_signature(ct.float16, 128, 256, 64, "matmul_f16"),
            mm.make_matmul_signature(ct.bfloat16, 64, 128, 32, "matmul_bf16")],
           OUT / "matmul_multi.tilebc")
    expected["matmul_multi.tilebc"] = [
        entry("matmul_fp32", [(2, f32)] * 3, [32, 32, 32], "matmul_fp32", 2),
        entry("matmul_f16", [(2, f16)] * 3, [128, 256, 64], "matmul_f16", 2),
        entry("matmul_bf16", [(2, bf16)] * 3, [64, 128, 32], "matmul_bf16", 2)]

    # two fp32 entries with different tiles: the module alone cannot say which is whose
    export(ct, ct_compilation, mm.matmul_kernel,
           [mm.make_matmul_signature(ct.float32, 32, 32, 32, "matmul_fp32_small"),
            mm.make_matmul_signature(ct.float32, 64, 64, 32, "matmul_fp32_large")],
           OUT / "matmul_ambiguous.tilebc")
    expected["matmul_ambiguous.tilebc"] = [
        entry("matmul_fp32_small", [(2, f32)] * 3, [], "matmul_fp32", 2),
        entry("matmul_fp32_large", [(2, f32)] * 3, [], "matmul_fp32", 2)]

    meta = {"cuda_tile_version": getattr(ct, "__version__", "unknown"), "bytecode_version": [13, 1, 0],
            "modules": expected}
    (OUT / "tilebc_expected.json").write_text(json.dumps(meta, indent=1) + "\n")
    for name in expected:
        print(f"wrote {name} ({(OUT / name).stat().st_size} bytes)")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_tilebc.py <reference root>")
    main(sys.argv[1])
