"""cuda_tile module (.tilebc) discovery on the CPU, through the C ABI.

The fixtures in tests/golden were exported here by cuda.tile from the
reference's own kernels (tests/golden/make_tilebc.py); the reader must
recover what the exporter was asked for (tilebc_expected.json): each entry's
symbol, bindings, array ranks and types, tile sizes, sm_100 hints, and the
backend kernel that serves it.  Malformed input -- every truncation of every
fixture, seeded byte corruption, wrong magic, unknown versions, MLIR text --
must come back as an error status, never a crash.  st_launch_module's
binding checks run before any device work, so they are tested here too.
"""
import ctypes
import json
import random
from pathlib import Path

import pytest

import sptiles_b200 as st
from sptiles_b200 import _native as N

GOLD = Path(__file__).resolve().parent / "golden"
EXPECTED = json.loads((GOLD / "tilebc_expected.json").read_text())
FIXTURES = sorted(EXPECTED["modules"])


def load_bytes(data: bytes):
    h = ctypes.c_void_p()
    buf = ctypes.create_string_buffer(data, len(data))
    rc = N.lib().st_module_load(ctypes.cast(buf, ctypes.c_void_p), len(data), ctypes.byref(h))
    return rc, h


def entry_dict(e: st.ModuleEntry) -> dict:
    return {"name": e.name, "n_params": e.n_params, "arrays": [list(a) for a in e.arrays],
            "constants": list(e.constants), "backend_entry": e.backend_entry,
            "num_cta_in_cga": e.num_cta_in_cga, "occupancy": e.occupancy}


@pytest.mark.parametrize("name", FIXTURES)
def test_fixture_entries_match_the_export(name):
    with st.TileModule(GOLD / name) as m:
        assert m.version == tuple(EXPECTED["bytecode_version"])
        assert [entry_dict(e) for e in m.entries] == EXPECTED["modules"][name]
        for e in m.entries:
            # cutile_python_v1: per array its data, then a size and a stride per dimension
            kinds = []
            for rank, dtype in e.arrays:
                kinds += [("buffer", dtype)] + [("i32", "i32")] * (2 * rank)
            assert list(e.params) == kinds


@pytest.mark.parametrize("name", FIXTURES)
def test_bytes_and_file_agree(name):
    data = (GOLD / name).read_bytes()
    assert [entry_dict(e) for e in st.TileModule(data).entries] == \
        [entry_dict(e) for e in st.TileModule(GOLD / name).entries]


def test_reference_vector_add_modules_bind_nine_params():
    # the runner binds 9 parameters for vector_add, output at index 6 (spirv_vector_add.py:85)
    for name in ("vector_add.tilebc", "vector_add2D.tilebc"):
        e = st.TileModule(GOLD / name).entry()
        assert e.n_params == 9 and [i for i, p in enumerate(e.params) if p[0] == "buffer"] == [0, 3, 6]
    # and 15 for matmul, output at index 10 (spirv_matmul.py:90)
    e = st.TileModule(GOLD / "matmul.tilebc").entry("matmul_fp32")
    assert e.n_params == 15 and [i for i, p in enumerate(e.params) if p[0] == "buffer"] == [0, 5, 10]
    assert e.tile_elems == 32 * 32


@pytest.mark.parametrize("name", FIXTURES)
def test_every_truncation_is_an_error(name):
    data = (GOLD / name).read_bytes()
    for cut in range(len(data)):
        rc, h = load_bytes(data[:cut])
        assert rc == N.ST_ERR_INVALID_ARGUMENT, (cut, rc)
        assert not h.value
        msg = N.last_error()
        assert "malformed" in msg or "not CUDA Tile bytecode" in msg, msg


def test_corrupted_bytes_never_crash():
    rnd = random.Random(1234)
    blobs = [(GOLD / n).read_bytes() for n in FIXTURES]
    accepted = 0
    for trial in range(4000):
        data = bytearray(rnd.choice(blobs))
        for _ in range(rnd.randint(1, 4)):
            i = rnd.randrange(12, len(data))  # keep the header so parsing goes deep
            data[i] = rnd.randrange(256) if rnd.random() < 0.7 else data[i] ^ (1 << rnd.randrange(8))
        rc, h = load_bytes(bytes(data))
        assert rc in (N.ST_OK, N.ST_ERR_INVALID_ARGUMENT, N.ST_ERR_UNSUPPORTED), rc
        if rc == N.ST_OK:
            accepted += 1
            count = ctypes.c_int32()
            N.check(N.lib().st_module_entry_count(h, ctypes.byref(count)))
            info = N.StModuleEntryInfo()
            for i in range(count.value):
                N.check(N.lib().st_module_entry(h, i, ctypes.byref(info)))
                assert 0 <= info.n_arrays <= 8 and 0 <= info.n_constants <= 3
            N.lib().st_module_free(h)
    assert accepted > 0  # corruption inside function bodies is invisible to the reader


def test_not_bytecode_and_unknown_versions():
    data = (GOLD / "vector_add.tilebc").read_bytes()
    for bad in (b"", b"module {\n  cuda_tile.entry @vector_add() {}\n}\n", b"\x7fTileIR", b"\x7fTileIX\x00" + data[8:]):
        rc, _ = load_bytes(bad)
        assert rc == N.ST_ERR_INVALID_ARGUMENT
        assert "not CUDA Tile bytecode" in N.last_error()
    for major, minor in ((14, 0), (13, 0), (13, 9), (12, 8)):
        rc, _ = load_bytes(data[:8] + bytes([major, minor]) + data[10:])
        assert rc == N.ST_ERR_UNSUPPORTED
        assert f"{major}.{minor} is not supported" in N.last_error()
    with pytest.raises(ValueError, match="could not open"):
        st.TileModule(GOLD / "no_such_module.tilebc")


def test_entry_without_a_kernel_here():
    # the same module with its symbol renamed (same length, so the tables stay valid)
    data = (GOLD / "vector_add.tilebc").read_bytes()
    assert data.count(b"vector_add") == 1
    m = st.TileModule(data.replace(b"vector_add", b"vector_sub"))
    e = m.entry()
    assert e.name == "vector_sub" and e.backend_entry is None and e.constants == ()
    rc = _launch_rc(m, None, _params_for(e))
    assert rc == N.ST_ERR_UNKNOWN_ENTRY and "no sm_100a kernel" in N.last_error()


# ---------------------------------------------------------------- launch checks (before any device work)
def _params_for(e: st.ModuleEntry, *, dtype_override=None, kinds_override=None):
    P = (N.StParam * e.n_params)()
    codes = {"f32": N.ST_F32, "f16": N.ST_F16, "bf16": N.ST_BF16}
    for i, (kind, dtype) in enumerate(e.params):
        kind = (kinds_override or {}).get(i, kind)
        if kind == "buffer":
            P[i].kind, P[i].dtype, P[i].data = N.ST_PARAM_BUFFER, codes.get(dtype_override or dtype, 99), 0x1000
        else:
            P[i].kind, P[i].value = N.ST_PARAM_I32, 1
    return P


def _launch_rc(m, name, P, n=None):
    g = N.StGrid(1, 1, 1)
    ex = N.StExec(None, 0, N.ST_EXEC_SYNC, 1000, None, 0)
    return N.lib().st_launch_module(None, m.handle, name.encode() if name else None, ctypes.byref(g), P,
                                    len(P) if n is None else n, ctypes.byref(ex))


def test_launch_rejects_bindings_that_do_not_match_the_module():
    m = st.TileModule(GOLD / "matmul_multi.tilebc")
    e = m.entry("matmul_f16")
    assert _launch_rc(m, "matmul_f32", _params_for(e)) == N.ST_ERR_UNKNOWN_ENTRY
    assert "was not found in the module" in N.last_error()
    assert _launch_rc(m, None, _params_for(e)) == N.ST_ERR_INVALID_ARGUMENT
    assert "holds 3 entries" in N.last_error()
    assert _launch_rc(m, "matmul_f16", _params_for(e), n=14) == N.ST_ERR_INVALID_ARGUMENT
    assert "takes 15 bindings" in N.last_error()
    assert _launch_rc(m, "matmul_f16", _params_for(e, dtype_override="f32")) == N.ST_ERR_INVALID_ARGUMENT
    assert "declares f16 data, got f32" in N.last_error()
    assert _launch_rc(m, "matmul_f16", _params_for(e, kinds_override={1: "buffer"})) == N.ST_ERR_INVALID_ARGUMENT
    assert "i32 scalar in the module" in N.last_error()
    assert _launch_rc(m, "matmul_f16", _params_for(e, kinds_override={5: "i32"})) == N.ST_ERR_INVALID_ARGUMENT
    assert "is a buffer in the module" in N.last_error()


def test_ambiguous_tile_sizes_must_be_passed():
    m = st.TileModule(GOLD / "matmul_ambiguous.tilebc")
    e = m.entry("matmul_fp32_large")
    assert _launch_rc(m, e.name, _params_for(e)) == N.ST_ERR_INVALID_ARGUMENT
    assert "cannot be read unambiguously" in N.last_error()


# ---------------------------------------------------------------- synthetic modules
def _varint(x: int) -> bytes:
    out = bytearray()
    while True:
        b = x & 0x7F
        x >>= 7
        out.append(b | (0x80 if x else 0))
        if not x:
            return bytes(out)


def _int_list(vals, width):
    return _varint(len(vals)) + b"".join(v.to_bytes(width, "little", signed=True) for v in vals)


def _table(items, width=4):
    out = bytearray(_varint(len(items)))
    out += b"\xcb" * (-len(out) % width)
    off = 0
    for it in items:
        out += off.to_bytes(width, "little")
        off += len(it)
    return bytes(out) + b"".join(items)


def _module(version, strings, types, funcs):
    """A minimal module: header, function, type and string sections (the layout of TileIR bytecode)."""
    major, minor, tag = version
    buf = bytearray(b"\x7fTileIR\x00" + bytes([major, minor]) + tag.to_bytes(2, "little"))

    def section(sid, payload, align):
        buf.append(sid | (0x80 if align > 1 else 0))
        buf.extend(_varint(len(payload)))
        if align > 1:
            buf.extend(_varint(align))
            buf.extend(b"\xcb" * (-len(buf) % align))
        buf.extend(payload)

    fsec = bytearray(_varint(len(funcs)))
    for name_id, sig, flags, hints, body in funcs:
        fsec += _varint(name_id) + _varint(sig) + bytes([flags]) + _varint(1) + hints + _varint(len(body)) + body
    section(2, bytes(fsec), 8)
    section(5, _table(types), 4)
    section(1, _table([s.encode() for s in strings]), 4)
    buf.append(0)
    return bytes(buf)


def _types_for_vector_add(version, tile, view_dtype=0x07, index=0x03):
    pv = (_varint(0) if version >= (13, 3, 0) else b"") + _int_list([tile], 4) + _varint(6) + _int_list([0], 4)
    if version < (13, 3, 0):
        pv += b"\x00"  # no padding value (13.3 says so in the leading flags instead)
    return [b"\x00", b"\x03", b"\x07", b"\x0c\x02", b"\x0d\x03" + _int_list([], 8),
            b"\x0d" + _varint(7 if index == 0x04 else 1) + _int_list([], 8),
            b"\x0e" + _varint(2 if view_dtype == 0x07 else 8) + _int_list([-(1 << 63)], 8) + _int_list([1], 8),
            b"\x04",  # i64 (id 7)
            b"\x05",  # f16 (id 8)
            b"\x0f" + pv,  # partition view (id 9)
            b"\x10" + _varint(9) + b"".join(_varint(t) for t in [4, 5, 5] * 3) + _varint(0)]  # signature (id 10)


@pytest.mark.parametrize("version", [(13, 1, 0), (13, 2, 0), (13, 3, 0)])
def test_synthetic_module_versions_helpers_and_hints(version):
    strings = ["vector_add", "helper", "sm_100", "occupancy", "num_cta_in_cga", "sm_90"]
    types = _types_for_vector_add(version, 256)
    # hints: sm_90 {num_cta_in_cga: 4}, sm_100 {occupancy: 3, num_cta_in_cga: 1}
    def int_attr(v):
        return b"\x01" + _varint(1) + _varint(v)

    hints = (b"\x0b" + _varint(2) + _varint(5) + b"\x0a" + _varint(1) + _varint(4) + int_attr(4)
             + _varint(2) + b"\x0a" + _varint(2) + _varint(3) + int_attr(3) + _varint(4) + int_attr(1))
    funcs = [(1, 10, 0x00, b"", b"\x01\x02\x03"),  # a non-entry function: not listed
             (0, 10, 0x06, hints, b"\x00" * 40)]
    m = st.TileModule(_module(version, strings, types, funcs))
    assert m.version == version
    assert [e.name for e in m.entries] == ["vector_add"]
    e = m.entry()
    assert (e.n_params, e.arrays, e.constants) == (9, ((1, "f32"),) * 3, (256,))
    assert (e.occupancy, e.num_cta_in_cga, e.backend_entry) == (3, 1, "vector_add")


def test_synthetic_module_unsupported_parameter_types():
    version = (13, 1, 0)
    # sizes and strides of type i64: not bindable as the i32 scalars of cutile_python_v1
    types = _types_for_vector_add(version, 128, index=0x04)
    m = st.TileModule(_module(version, ["vector_add"], types, [(0, 10, 0x02, b"", b"")]))
    e = m.entry()
    assert e.params[1] == ("other", None) and e.arrays == () and e.backend_entry is None
    # a partition view over an f16 view does not give the f32 add its tile
    types = _types_for_vector_add(version, 128, view_dtype=0x05)
    e = st.TileModule(_module(version, ["vector_add"], types, [(0, 10, 0x02, b"", b"")])).entry()
    assert e.backend_entry == "vector_add" and e.constants == ()


def test_synthetic_module_structural_errors():
    version = (13, 1, 0)
    types = _types_for_vector_add(version, 64)
    good = _module(version, ["vector_add"], types, [(0, 10, 0x02, b"", b"")])
    assert st.TileModule(good).entry().constants == (64,)
    cases = {
        "function name id": [(3, 10, 0x02, b"", b"")],
        "not a function type": [(0, 4, 0x02, b"", b"")],
        "signature type id": [(0, 99, 0x02, b"", b"")],
        "entry hints": [(0, 10, 0x06, b"\x07\x00", b"")],  # dense-elements attributes are not hints
    }
    for what, funcs in cases.items():
        rc, _ = load_bytes(_module(version, ["vector_add"], types, funcs))
        assert rc == N.ST_ERR_INVALID_ARGUMENT, what
        assert "malformed" in N.last_error(), what
    # a section repeated, and a module without its end marker
    rc, _ = load_bytes(good[:-1] + b"\x01\x00" + b"\x00")
    assert rc == N.ST_ERR_INVALID_ARGUMENT and "repeated section" in N.last_error()
    rc, _ = load_bytes(good[:-1])
    assert rc == N.ST_ERR_INVALID_ARGUMENT and "end marker" in N.last_error()
    # a partition view whose view is not a tensor view
    bad_types = list(types)
    bad_types[9] = b"\x0f" + _int_list([64], 4) + _varint(2) + _int_list([0], 4) + b"\x00"
    rc, _ = load_bytes(_module(version, ["vector_add"], bad_types, [(0, 10, 0x02, b"", b"")]))
    assert rc == N.ST_ERR_INVALID_ARGUMENT and "partition view" in N.last_error()
