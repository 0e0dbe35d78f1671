"""cuda_tile modules (TileIR bytecode, .tilebc): entry discovery and launch.

The reference's translator takes a .tilebc written by cuTile's exporter
(shaders/vecadd.py:23-58, shaders/matmul.py:287-306), loads it
(src/main.cpp:75-104) and derives each entry's bindings from its parameter
types (src/lower.hpp:197-310).  ``TileModule`` does the same discovery over
the C ABI (st_module_*): which entries the module exports, their bindings in
the cutile_python_v1 layout, their tile sizes and sm_100 hints, and which
sm_100a kernel of this backend serves each one.  ``TileModule.launch`` is
st_launch_module: it checks the bindings against the module before running
the registered kernel.  The module's code itself is not decoded or run.
"""
from __future__ import annotations

import ctypes
import math
import os
from dataclasses import dataclass
from typing import Sequence

from . import _native as N

_DTYPE_NAMES = {N.ST_F32: "f32", N.ST_F16: "f16", N.ST_BF16: "bf16", N.ST_I32: "i32"}
_KIND_NAMES = {N.ST_MODULE_PARAM_BUFFER: "buffer", N.ST_MODULE_PARAM_I32: "i32", N.ST_MODULE_PARAM_OTHER: "other"}


@dataclass(frozen=True)
class ModuleEntry:
    """One cuda_tile.entry of a module, as the C ABI reports it."""

    index: int
    name: str
    params: tuple[tuple[str, str | None], ...]  # (kind, element type) per binding
    arrays: tuple[tuple[int, str | None], ...]  # (rank, element type) per array descriptor
    constants: tuple[int, ...]                   # tile sizes; empty when the module is ambiguous
    num_cta_in_cga: int
    occupancy: int
    backend_entry: str | None                    # st_launch registry entry, None = not served here

    @property
    def n_params(self) -> int:
        return len(self.params)

    @property
    def tile_elems(self) -> int | None:
        """Elements of one output tile: tile_size (1D), tile_m * tile_n (2D), tm * tn (matmul)."""
        if not self.constants:
            return None
        if self.backend_entry and "matmul" in self.backend_entry:
            return self.constants[0] * self.constants[1]
        return math.prod(self.constants)


class TileModule:
    """A parsed .tilebc module.  ``source`` is a path or the module's bytes."""

    def __init__(self, source: str | os.PathLike | bytes | bytearray | memoryview):
        self._handle = ctypes.c_void_p()
        L = N.lib()
        if isinstance(source, (bytes, bytearray, memoryview)):
            data = bytes(source)
            buf = ctypes.create_string_buffer(data, len(data))
            N.check(L.st_module_load(ctypes.cast(buf, ctypes.c_void_p), len(data), ctypes.byref(self._handle)),
                    "st_module_load")
        else:
            N.check(L.st_module_load_file(os.fsencode(source), ctypes.byref(self._handle)), "st_module_load_file")
        major, minor, tag = ctypes.c_int32(), ctypes.c_int32(), ctypes.c_int32()
        N.check(L.st_module_version(self._handle, ctypes.byref(major), ctypes.byref(minor), ctypes.byref(tag)),
                "st_module_version")
        self.version = (major.value, minor.value, tag.value)
        self.entries = self._read_entries()

    def _read_entries(self) -> list[ModuleEntry]:
        L = N.lib()
        count = ctypes.c_int32()
        N.check(L.st_module_entry_count(self._handle, ctypes.byref(count)), "st_module_entry_count")
        out = []
        for i in range(count.value):
            info = N.StModuleEntryInfo()
            N.check(L.st_module_entry(self._handle, i, ctypes.byref(info)), "st_module_entry")
            params = []
            for p in range(info.n_params):
                kind, dtype = ctypes.c_int32(), ctypes.c_int32()
                N.check(L.st_module_param(self._handle, i, p, ctypes.byref(kind), ctypes.byref(dtype)),
                        "st_module_param")
                params.append((_KIND_NAMES[kind.value], _DTYPE_NAMES.get(dtype.value)))
            out.append(ModuleEntry(
                index=i, name=info.name.decode(), params=tuple(params),
                arrays=tuple((info.array_rank[a], _DTYPE_NAMES.get(info.array_dtype[a]))
                             for a in range(info.n_arrays)),
                constants=tuple(info.constants[: info.n_constants]),
                num_cta_in_cga=info.num_cta_in_cga, occupancy=info.occupancy,
                backend_entry=info.backend_entry.decode() if info.backend_entry else None))
        return out

    def entry(self, name: str | None = None) -> ModuleEntry:
        """The entry called ``name`` (or the only one)."""
        if name is None:
            if len(self.entries) != 1:
                raise ValueError(f"the module holds {len(self.entries)} entries: name the one to launch")
            return self.entries[0]
        for e in self.entries:
            if e.name == name:
                return e
        raise ValueError(f"Entry point {name} was not found in the module.")

    @property
    def handle(self) -> int:
        if not self._handle:
            raise ValueError("the module is closed")
        return self._handle.value

    def launch(self, ctx: int, entry_name: str | None, grid: Sequence[int], params: ctypes.Array,
               exec_: N.StExec) -> None:
        """st_launch_module with prepared bindings (``params``: an array of StParam)."""
        g = N.StGrid(*[int(x) for x in grid])
        N.check(N.lib().st_launch_module(ctx, self.handle, entry_name.encode() if entry_name else None,
                                         ctypes.byref(g), params, len(params), ctypes.byref(exec_)),
                f"st_launch_module({entry_name or self.entry().name})")

    def close(self) -> None:
        if self._handle:
            N.lib().st_module_free(self._handle)
            self._handle = ctypes.c_void_p()

    def __enter__(self) -> "TileModule":
        return self

    def __exit__(self, *exc) -> None:
        self.close()

    def __del__(self) -> None:
        try:
            self.close()
        except Exception:
            pass
