// module.cu -- cuda_tile modules (TileIR bytecode, ".tilebc"): entry
// discovery and launch by module entry.
//
// The reference's translator loads a .tilebc (src/main.cpp:75-104:
// isTileIRBytecode, readBytecode), turns every cuda_tile.entry into a SPIR-V
// function whose parameters become the module's bindings in order
// (src/lower.hpp:197-310: replace_entries, convert_entry_type --
// tile<ptr<f32>> becomes an f32[] storage buffer and tile<i32> an i32 --
// and attach_spirv_abi_attrs, binding i = parameter i), and its host runners
// bind arrays to those positions.  This backend runs hand-written sm_100a
// kernels instead of lowering the module's code, so it reads only what a
// launch needs from the module:
//
//   * each entry function's symbol and parameter types: the binding layout,
//     grouped into cutile_python_v1 array descriptors (data, then a size and
//     a stride per dimension);
//   * the entry's sm_100 optimisation hints (num_cta_in_cga, occupancy);
//   * the tile shapes of the module's partition views: the kernel constants
//     (tile_size, tm/tn/tk) that cuTile folds into the code and that the
//     cuda_tile grid is counted in.
//
// Function bodies are skipped by their length and never decoded.
//
// Layout read here (bytecode versions 13.1 to 13.3; the format is the one
// cuda.tile's bytecode writer produces, cuda/tile/_bytecode/writer.py and
// type.py, Apache-2.0): an 8-byte magic "\x7fTileIR\0", major, minor and a
// 16-bit tag; then sections, each a byte id (bit 7: an alignment follows), a
// varint length, the optional varint alignment and padding up to it (from
// the start of the file), and the payload; a zero byte ends the module.
// Varints are little-endian base-128.  The string and type sections are
// tables: a count, padding to the index width, one offset per item, then the
// items' bytes.  The function section holds, per function, its name
// (string id), its signature (type id), a flag byte (0x02 entry, 0x04 hints
// follow), a debug index, the hints, and the body's length and bytes.
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <new>
#include <set>
#include <string>
#include <tuple>
#include <vector>

#include "common.h"

namespace st {
namespace {

constexpr uint8_t kMagic[8] = {0x7f, 'T', 'i', 'l', 'e', 'I', 'R', 0x00};

enum Section : uint8_t { kSecEnd = 0, kSecString = 1, kSecFunc = 2, kSecType = 5 };

// Leading byte of an encoded type.
enum TypeTag : uint8_t {
    kTyI1 = 0x00, kTyI8 = 0x01, kTyI16 = 0x02, kTyI32 = 0x03, kTyI64 = 0x04, kTyF16 = 0x05, kTyBF16 = 0x06,
    kTyF32 = 0x07, kTyTF32 = 0x08, kTyF64 = 0x09, kTyF8E4M3 = 0x0a, kTyF8E5M2 = 0x0b,
    kTyPointer = 0x0c, kTyTile = 0x0d, kTyTensorView = 0x0e, kTyPartitionView = 0x0f, kTyFunc = 0x10,
    kTyToken = 0x11, kTyF8E8M0 = 0x12, kTyF4E2M1 = 0x13,
};

// Tags of the tagged attributes that entry hints may hold.
enum AttrTag : uint8_t {
    kAttrInteger = 0x01, kAttrFloat = 0x02, kAttrBool = 0x03, kAttrType = 0x04, kAttrString = 0x05,
    kAttrArray = 0x06, kAttrDivBy = 0x08, kAttrDictionary = 0x0a, kAttrOptHints = 0x0b, kAttrBounded = 0x0c,
};

constexpr int kMaxArrays = 8;

// Bounds-checked reader over one byte range; every read past the end clears ok.
struct Cursor {
    const uint8_t *p = nullptr;
    const uint8_t *end = nullptr;
    bool ok = true;

    size_t left() const { return ok ? static_cast<size_t>(end - p) : 0; }
    uint8_t byte() {
        if (!ok || p >= end) return static_cast<uint8_t>(ok = false);
        return *p++;
    }
    uint64_t varint() {
        uint64_t x = 0;
        for (int shift = 0; shift < 64; shift += 7) {
            const uint8_t c = byte();
            if (!ok) return 0;
            x |= static_cast<uint64_t>(c & 0x7f) << shift;
            if (!(c & 0x80)) return x;
        }
        ok = false;  // more than ten groups
        return 0;
    }
    int64_t svarint() {  // zig-zag
        const uint64_t u = varint();
        return static_cast<int64_t>(u >> 1) ^ -static_cast<int64_t>(u & 1);
    }
    uint64_t fixed(int width) {
        if (!ok || left() < static_cast<size_t>(width)) return ok = false, 0;
        uint64_t x = 0;
        for (int i = 0; i < width; ++i) x |= static_cast<uint64_t>(p[i]) << (8 * i);
        p += width;
        return x;
    }
    int64_t fixed_signed(int width) {
        const uint64_t u = fixed(width);
        if (width == 8) return static_cast<int64_t>(u);
        const uint64_t sign = uint64_t(1) << (8 * width - 1);
        return static_cast<int64_t>((u ^ sign) - sign);
    }
    void skip(uint64_t n) {
        if (!ok || left() < n) ok = false;
        else p += n;
    }
    // A count of items that take at least one byte each.
    uint64_t count() {
        const uint64_t n = varint();
        if (n > left()) ok = false;
        return ok ? n : 0;
    }
};

struct Type {
    uint8_t tag = 0xff;
    uint64_t elem = UINT64_MAX;   // Pointer: pointee; Tile / TensorView: element type
    std::vector<int64_t> shape;   // Tile / TensorView shape; PartitionView tile shape
    uint64_t view = UINT64_MAX;   // PartitionView: its tensor view
    std::vector<uint64_t> params; // Func
};

// One item of a table section (strings, types).
struct Table {
    std::vector<std::pair<const uint8_t *, size_t>> items;
};

bool read_table(const uint8_t *sec, size_t len, int index_width, Table *out) {
    Cursor c{sec, sec + len};
    const uint64_t n = c.count();
    const size_t head = static_cast<size_t>(c.p - sec);
    c.skip((index_width - head % index_width) % index_width);
    if (!c.ok || n > c.left() / index_width) return false;
    std::vector<uint64_t> off(n);
    for (uint64_t i = 0; i < n; ++i) off[i] = c.fixed(index_width);
    const uint8_t *data = c.p;
    const size_t data_len = c.left();
    if (!c.ok) return false;
    out->items.clear();
    for (uint64_t i = 0; i < n; ++i) {
        const uint64_t b = off[i], e = i + 1 < n ? off[i + 1] : data_len;
        if (b > e || e > data_len) return false;
        out->items.emplace_back(data + b, static_cast<size_t>(e - b));
    }
    return true;
}

bool read_int_list(Cursor &c, int width, std::vector<int64_t> *out) {
    const uint64_t n = c.varint();
    if (!c.ok || n > c.left() / width) return false;
    out->resize(n);
    for (uint64_t i = 0; i < n; ++i) (*out)[i] = c.fixed_signed(width);
    return c.ok;
}

bool parse_type(const uint8_t *b, size_t len, uint32_t version, Type *t) {
    Cursor c{b, b + len};
    t->tag = c.byte();
    if (!c.ok) return false;
    switch (t->tag) {
    case kTyPointer: t->elem = c.varint(); break;
    case kTyTile:
        t->elem = c.varint();
        if (!read_int_list(c, 8, &t->shape)) return false;
        break;
    case kTyTensorView: {
        t->elem = c.varint();
        if (!read_int_list(c, 8, &t->shape)) return false;
        std::vector<int64_t> strides;
        if (!read_int_list(c, 8, &strides)) return false;
        break;
    }
    case kTyPartitionView: {
        if (version >= 130300) c.varint();  // optional-field flags
        if (!read_int_list(c, 4, &t->shape)) return false;
        t->view = c.varint();
        break;  // dim map and padding value are not needed
    }
    case kTyFunc: {
        const uint64_t np = c.count();
        for (uint64_t i = 0; i < np && c.ok; ++i) t->params.push_back(c.varint());
        break;
    }
    default: break;  // scalar types and types this reader does not need
    }
    return c.ok;
}

int dtype_of_scalar(uint8_t tag) {
    switch (tag) {
    case kTyF32: return ST_F32;
    case kTyF16: return ST_F16;
    case kTyBF16: return ST_BF16;
    case kTyI32: return ST_I32;
    default: return -1;
    }
}

const char *dtype_name(int dtype) {
    switch (dtype) {
    case ST_F32: return "f32";
    case ST_F16: return "f16";
    case ST_BF16: return "bf16";
    case ST_I32: return "i32";
    default: return "an unsupported type";
    }
}

// Skip one tagged attribute; record integer entries of an sm_100 hint dictionary.
struct HintSink {
    int *num_cta_in_cga = nullptr;
    int *occupancy = nullptr;
};

bool skip_attr(Cursor &c, const std::vector<std::string> &strings, const std::vector<Type> &types, int depth,
               const std::string &key, const HintSink *sink);

bool skip_dict(Cursor &c, const std::vector<std::string> &strings, const std::vector<Type> &types, int depth,
               const HintSink *sink) {
    const uint64_t n = c.count();
    for (uint64_t i = 0; i < n && c.ok; ++i) {
        const uint64_t k = c.varint();
        if (!c.ok || k >= strings.size()) return false;
        if (!skip_attr(c, strings, types, depth + 1, strings[k], sink)) return false;
    }
    return c.ok;
}

bool skip_attr(Cursor &c, const std::vector<std::string> &strings, const std::vector<Type> &types, int depth,
               const std::string &key, const HintSink *sink) {
    if (depth > 16) return false;
    const uint8_t tag = c.byte();
    switch (tag) {
    case kAttrInteger: {
        c.varint();  // type
        const uint64_t v = c.varint();
        if (sink && c.ok) {
            if (key == "num_cta_in_cga" && sink->num_cta_in_cga) *sink->num_cta_in_cga = static_cast<int>(v);
            if (key == "occupancy" && sink->occupancy) *sink->occupancy = static_cast<int>(v);
        }
        break;
    }
    case kAttrFloat: {
        const uint64_t ty = c.varint();
        if (!c.ok || ty >= types.size()) return false;
        const uint8_t t = types[ty].tag;
        if (t == kTyF8E4M3 || t == kTyF8E5M2 || t == kTyF8E8M0 || t == kTyF4E2M1) c.byte();
        else c.varint();
        break;
    }
    case kAttrBool: c.byte(); break;
    case kAttrType:
    case kAttrString: c.varint(); break;
    case kAttrArray: {
        const uint64_t n = c.count();
        for (uint64_t i = 0; i < n && c.ok; ++i)
            if (!skip_attr(c, strings, types, depth + 1, std::string(), nullptr)) return false;
        break;
    }
    case kAttrDivBy: {
        c.varint();
        const uint8_t f = c.byte();
        if (f & 1) c.svarint();
        if (f & 2) c.svarint();
        break;
    }
    case kAttrBounded: {
        const uint8_t f = c.byte();
        if (f & 1) c.svarint();
        if (f & 2) c.svarint();
        break;
    }
    case kAttrDictionary: return skip_dict(c, strings, types, depth, sink);
    case kAttrOptHints: {
        // per target architecture, a dictionary of hints; keep sm_100's
        const uint64_t n = c.count();
        for (uint64_t i = 0; i < n && c.ok; ++i) {
            const uint64_t arch = c.varint();
            if (!c.ok || arch >= strings.size()) return false;
            const bool ours = strings[arch] == "sm_100" || strings[arch] == "sm_100a";
            if (!skip_attr(c, strings, types, depth + 1, std::string(), ours ? sink : nullptr)) return false;
        }
        break;
    }
    default: return false;  // dense elements and the like do not appear in entry hints
    }
    return c.ok;
}

}  // namespace
}  // namespace st

// ------------------------------------------------------------------ the module
struct st_module_entry_rec {
    std::string name;
    std::vector<int32_t> kinds;   // ST_MODULE_PARAM_*
    std::vector<int32_t> dtypes;  // element type of a buffer, ST_I32 for scalars, -1 otherwise
    int32_t n_arrays = 0;
    int32_t array_rank[8] = {};
    int32_t array_dtype[8] = {};
    bool layout_ok = false;       // parameters group into whole array descriptors
    int32_t n_constants = 0;
    int32_t constants[3] = {};
    int32_t num_cta_in_cga = 0;
    int32_t occupancy = 0;
    const char *backend = nullptr;
};

struct st_module {
    int32_t major = 0, minor = 0, tag = 0;
    std::vector<st_module_entry_rec> entries;
};

namespace st {
namespace {

// Group the flat bindings into cutile_python_v1 array descriptors: a buffer,
// then 2*rank i32 scalars (sizes, then strides).
void group_arrays(st_module_entry_rec &e) {
    e.n_arrays = 0;
    e.layout_ok = false;
    const size_t n = e.kinds.size();
    size_t i = 0;
    while (i < n) {
        if (e.kinds[i] != ST_MODULE_PARAM_BUFFER) return;
        size_t j = i + 1;
        while (j < n && e.kinds[j] == ST_MODULE_PARAM_I32) ++j;
        const size_t scalars = j - i - 1;
        if (scalars == 0 || scalars % 2 != 0 || scalars > 4 || e.n_arrays == kMaxArrays) return;
        e.array_rank[e.n_arrays] = static_cast<int32_t>(scalars / 2);
        e.array_dtype[e.n_arrays] = e.dtypes[i];
        ++e.n_arrays;
        i = j;
    }
    e.layout_ok = e.n_arrays > 0;
}

bool all_arrays(const st_module_entry_rec &e, int count, int rank, int dtype) {
    if (e.n_arrays != count) return false;
    for (int i = 0; i < count; ++i)
        if (e.array_rank[i] != rank || (dtype >= 0 && e.array_dtype[i] != dtype)) return false;
    return true;
}

// The registered kernel that serves an entry.  The symbol names the
// computation, as in st_launch's registry; the reference's exports are
// "vector_add" (rank-1 arrays; vecadd.py, vecadd2.py) and "matmul_fp32"
// (matmul.py:287-296).  A "vector_add" over rank-2 arrays is the 2D add; a
// symbol containing "matmul" is the mmaf matmul in A's dtype (with
// "persistent": the persistent kernel, matmul.py:106-178), a fourth rank-1
// array being the fused bias.
const char *pick_backend(const st_module_entry_rec &e) {
    if (!e.layout_ok) return nullptr;
    const std::string &s = e.name;
    if (s == "vector_add" || s == "vector_add_2d") {
        if (all_arrays(e, 3, 1, ST_F32)) return s == "vector_add" ? "vector_add" : nullptr;
        if (all_arrays(e, 3, 2, ST_F32)) return "vector_add_2d";
        return nullptr;
    }
    if (s == "vector_fma" || s == "vector_fma_2d") {
        if (all_arrays(e, 4, 1, ST_F32)) return s == "vector_fma" ? "vector_fma" : nullptr;
        if (all_arrays(e, 4, 2, ST_F32)) return "vector_fma_2d";
        return nullptr;
    }
    if (s == "cast" || s == "cast_2d") {
        if (all_arrays(e, 2, 1, -1)) return s == "cast" ? "cast" : nullptr;
        if (all_arrays(e, 2, 2, -1)) return "cast_2d";
        return nullptr;
    }
    if (s.find("matmul") != std::string::npos) {
        const bool bias = e.n_arrays == 4 && e.array_rank[3] == 1;
        if (!(e.n_arrays == 3 || bias)) return nullptr;
        for (int i = 0; i < 3; ++i)
            if (e.array_rank[i] != 2) return nullptr;
        const int dt = e.array_dtype[0];
        if (e.array_dtype[1] != dt) return nullptr;
        const bool persistent = s.find("persistent") != std::string::npos;
        static const char *const names[2][2][3] = {
            {{"matmul_fp32", "matmul_f16", "matmul_bf16"},
             {"matmul_fp32_bias", "matmul_f16_bias", "matmul_bf16_bias"}},
            {{"persistent_matmul_fp32", "persistent_matmul_f16", "persistent_matmul_bf16"},
             {nullptr, nullptr, nullptr}}};
        if (dt != ST_F32 && dt != ST_F16 && dt != ST_BF16) return nullptr;
        return names[persistent][bias][dt];
    }
    return nullptr;
}

struct PartitionTile {
    std::vector<int64_t> shape;  // the tile shape
    int view_dtype;              // element type of the tensor view it partitions
    size_t view_rank;
};

// The kernel constants of an entry, from the tile shapes of the module's
// partition views over tensor views of the entry's element types and ranks.
// They are set only when those views admit exactly one assignment.
void recover_constants(st_module_entry_rec &e, const std::vector<PartitionTile> &pv) {
    e.n_constants = 0;
    if (!e.backend) return;
    const std::string b = e.backend;
    std::set<std::vector<int64_t>> found;
    auto positive = [](const std::vector<int64_t> &s) {
        for (int64_t v : s)
            if (v <= 0 || v > (1 << 20)) return false;
        return true;
    };
    if (b.find("matmul") != std::string::npos) {
        const int ab = e.array_dtype[0], cd = e.array_dtype[2];
        std::set<std::pair<int64_t, int64_t>> a_tiles, c_tiles;
        for (const PartitionTile &t : pv) {
            if (t.shape.size() != 2 || t.view_rank != 2 || !positive(t.shape)) continue;
            if (t.view_dtype == ab) a_tiles.insert({t.shape[0], t.shape[1]});
            if (t.view_dtype == cd) c_tiles.insert({t.shape[0], t.shape[1]});
        }
        // A is tm x tk, B is tk x tn (same element type), C is tm x tn
        for (const auto &a : a_tiles)
            for (const auto &bt : a_tiles)
                if (bt.first == a.second && c_tiles.count({a.first, bt.second}))
                    found.insert({a.first, bt.second, a.second});
    } else {
        const int rank = e.array_rank[0];
        std::set<int> dts;
        for (int i = 0; i < e.n_arrays; ++i) dts.insert(e.array_dtype[i]);
        for (const PartitionTile &t : pv)
            if (static_cast<int>(t.shape.size()) == rank && static_cast<int>(t.view_rank) == rank &&
                dts.count(t.view_dtype) && positive(t.shape))
                found.insert(t.shape);
    }
    if (found.size() != 1) return;
    const std::vector<int64_t> &v = *found.begin();
    e.n_constants = static_cast<int32_t>(v.size());
    for (size_t i = 0; i < v.size() && i < 3; ++i) e.constants[i] = static_cast<int32_t>(v[i]);
}

int bad(const char *what) { return fail(ST_ERR_INVALID_ARGUMENT, std::string("malformed TileIR bytecode: ") + what); }

int parse_module(const uint8_t *buf, size_t size, st_module *m) {
    if (size < 12 || std::memcmp(buf, kMagic, 8) != 0)
        return fail(ST_ERR_INVALID_ARGUMENT, "input is not CUDA Tile bytecode (no TileIR magic number)");
    m->major = buf[8];
    m->minor = buf[9];
    m->tag = static_cast<int32_t>(buf[10] | (buf[11] << 8));
    const uint32_t version = static_cast<uint32_t>(m->major) * 10000 + m->minor * 100 + m->tag;
    if (m->major != 13 || m->minor < 1 || m->minor > 3)
        return fail(ST_ERR_UNSUPPORTED, "TileIR bytecode version " + std::to_string(m->major) + "." +
                                            std::to_string(m->minor) + " is not supported (13.1 to 13.3 are)");
    // sections
    const uint8_t *sec[8] = {};
    size_t sec_len[8] = {};
    Cursor c{buf + 12, buf + size};
    bool ended = false;
    while (c.ok && c.left() > 0) {
        const uint8_t id = c.byte();
        if (id == kSecEnd) {
            ended = true;
            break;
        }
        const uint64_t len = c.varint();
        if (id & 0x80) {
            const uint64_t align = c.varint();
            if (!c.ok || align == 0 || align > 4096) return bad("section alignment");
            const uint64_t pos = static_cast<uint64_t>(c.p - buf);
            c.skip((align - pos % align) % align);
        }
        if (!c.ok || len > c.left()) return bad("section length");
        const uint8_t sid = id & 0x7f;
        if (sid < 8) {
            if (sec[sid]) return bad("repeated section");
            sec[sid] = c.p;
            sec_len[sid] = static_cast<size_t>(len);
        }
        c.skip(len);
    }
    if (!c.ok || !ended) return bad("truncated (no end marker)");
    if (!sec[kSecString] || !sec[kSecType] || !sec[kSecFunc]) return bad("missing string, type or function section");

    // strings and types
    Table st_tab, ty_tab;
    if (!read_table(sec[kSecString], sec_len[kSecString], 4, &st_tab)) return bad("string table");
    if (!read_table(sec[kSecType], sec_len[kSecType], 4, &ty_tab)) return bad("type table");
    std::vector<std::string> strings;
    for (const auto &it : st_tab.items) strings.emplace_back(reinterpret_cast<const char *>(it.first), it.second);
    std::vector<Type> types(ty_tab.items.size());
    for (size_t i = 0; i < types.size(); ++i)
        if (!parse_type(ty_tab.items[i].first, ty_tab.items[i].second, version, &types[i])) return bad("type entry");
    auto type_at = [&](uint64_t id) -> const Type * { return id < types.size() ? &types[id] : nullptr; };

    // partition views and the tensor views they partition
    std::vector<PartitionTile> pv;
    for (const Type &t : types) {
        if (t.tag != kTyPartitionView) continue;
        const Type *view = type_at(t.view);
        if (!view || view->tag != kTyTensorView) return bad("partition view of a non-view type");
        const Type *el = type_at(view->elem);
        pv.push_back({t.shape, el ? dtype_of_scalar(el->tag) : -1, view->shape.size()});
    }

    // functions
    Cursor f{sec[kSecFunc], sec[kSecFunc] + sec_len[kSecFunc]};
    const uint64_t nf = f.count();
    for (uint64_t fi = 0; fi < nf && f.ok; ++fi) {
        const uint64_t name_id = f.varint();
        const uint64_t sig_id = f.varint();
        const uint8_t flags = f.byte();
        f.varint();  // debug info index
        if (!f.ok) return bad("function record");
        if (name_id >= strings.size()) return bad("function name id");
        const Type *sig = type_at(sig_id);
        if (!sig || sig->tag != kTyFunc) return bad("function signature is not a function type");
        st_module_entry_rec e;
        e.name = strings[name_id];
        if (flags & 0x04) {
            st::HintSink sink{&e.num_cta_in_cga, &e.occupancy};
            if (!skip_attr(f, strings, types, 0, std::string(), &sink)) return bad("entry hints");
        }
        const uint64_t body = f.varint();
        f.skip(body);
        if (!f.ok) return bad("function body length");
        if (!(flags & 0x02)) continue;  // only entries are launchable
        for (uint64_t p : sig->params) {
            const Type *t = type_at(p);
            if (!t) return bad("parameter type id");
            int32_t kind = ST_MODULE_PARAM_OTHER, dt = -1;
            if (t->tag == kTyTile && t->shape.empty()) {
                const Type *el = type_at(t->elem);
                if (el && el->tag == kTyPointer) {
                    const Type *pointee = type_at(el->elem);
                    kind = ST_MODULE_PARAM_BUFFER;
                    dt = pointee ? dtype_of_scalar(pointee->tag) : -1;
                    if (dt == ST_I32) dt = -1;  // integer buffers have no kernel here
                } else if (el && el->tag == kTyI32) {
                    kind = ST_MODULE_PARAM_I32;
                    dt = ST_I32;
                }
            }
            e.kinds.push_back(kind);
            e.dtypes.push_back(dt);
        }
        group_arrays(e);
        e.backend = pick_backend(e);
        recover_constants(e, pv);
        m->entries.push_back(std::move(e));
    }
    if (!f.ok) return bad("function section");
    return ST_OK;
}

const st_module_entry_rec *find_module_entry(const st_module *m, const char *name) {
    if (!name) return m->entries.size() == 1 ? &m->entries[0] : nullptr;
    for (const st_module_entry_rec &e : m->entries)
        if (e.name == name) return &e;
    return nullptr;
}

}  // namespace
}  // namespace st

using namespace st;

extern "C" int st_module_load(const void *bytes, uint64_t size, st_module **out) {
    if (!out) return fail(ST_ERR_INVALID_ARGUMENT, "st_module_load: out is null");
    *out = nullptr;
    if (!bytes && size > 0) return fail(ST_ERR_INVALID_ARGUMENT, "st_module_load: bytes is null");
    st_module *m = new (std::nothrow) st_module;
    if (!m) return fail(ST_ERR_OUT_OF_MEMORY, "st_module_load");
    int rc;
    try {
        rc = parse_module(static_cast<const uint8_t *>(bytes), static_cast<size_t>(size), m);
    } catch (const std::bad_alloc &) {
        rc = fail(ST_ERR_OUT_OF_MEMORY, "st_module_load");
    }
    if (rc != ST_OK) {
        delete m;
        return rc;
    }
    *out = m;
    return ST_OK;
}

extern "C" int st_module_load_file(const char *path, st_module **out) {
    if (!out) return fail(ST_ERR_INVALID_ARGUMENT, "st_module_load_file: out is null");
    *out = nullptr;
    if (!path) return fail(ST_ERR_INVALID_ARGUMENT, "st_module_load_file: path is null");
    FILE *fp = std::fopen(path, "rb");
    if (!fp) return fail(ST_ERR_INVALID_ARGUMENT, std::string("could not open input file '") + path + "'");
    std::vector<uint8_t> data;
    uint8_t chunk[65536];
    size_t got;
    while ((got = std::fread(chunk, 1, sizeof(chunk), fp)) > 0) {
        data.insert(data.end(), chunk, chunk + got);
        if (data.size() > (size_t(256) << 20)) {
            std::fclose(fp);
            return fail(ST_ERR_INVALID_ARGUMENT, std::string("'") + path + "' is larger than 256 MiB");
        }
    }
    const bool err = std::ferror(fp) != 0;
    std::fclose(fp);
    if (err) return fail(ST_ERR_INVALID_ARGUMENT, std::string("could not read '") + path + "'");
    return st_module_load(data.data(), data.size(), out);
}

extern "C" int st_module_free(st_module *module) {
    delete module;
    return ST_OK;
}

extern "C" int st_module_version(const st_module *module, int32_t *major, int32_t *minor, int32_t *tag) {
    if (!module) return fail(ST_ERR_INVALID_ARGUMENT, "st_module_version: module is null");
    if (major) *major = module->major;
    if (minor) *minor = module->minor;
    if (tag) *tag = module->tag;
    return ST_OK;
}

extern "C" int st_module_entry_count(const st_module *module, int32_t *count) {
    if (!module || !count) return fail(ST_ERR_INVALID_ARGUMENT, "st_module_entry_count: null argument");
    *count = static_cast<int32_t>(module->entries.size());
    return ST_OK;
}

extern "C" int st_module_entry(const st_module *module, int32_t index, st_module_entry_info *out) {
    if (!module || !out) return fail(ST_ERR_INVALID_ARGUMENT, "st_module_entry: null argument");
    if (index < 0 || static_cast<size_t>(index) >= module->entries.size())
        return fail(ST_ERR_INVALID_ARGUMENT, "st_module_entry: index out of range");
    const st_module_entry_rec &e = module->entries[index];
    std::memset(out, 0, sizeof(*out));
    out->name = e.name.c_str();
    out->n_params = static_cast<int32_t>(e.kinds.size());
    out->n_arrays = e.layout_ok ? e.n_arrays : 0;
    for (int i = 0; i < out->n_arrays; ++i) {
        out->array_rank[i] = e.array_rank[i];
        out->array_dtype[i] = e.array_dtype[i];
    }
    out->n_constants = e.n_constants;
    for (int i = 0; i < 3; ++i) out->constants[i] = e.constants[i];
    out->num_cta_in_cga = e.num_cta_in_cga;
    out->occupancy = e.occupancy;
    out->backend_entry = e.backend;
    return ST_OK;
}

extern "C" int st_module_param(const st_module *module, int32_t entry, int32_t param, int32_t *kind,
                               int32_t *dtype) {
    if (!module) return fail(ST_ERR_INVALID_ARGUMENT, "st_module_param: module is null");
    if (entry < 0 || static_cast<size_t>(entry) >= module->entries.size())
        return fail(ST_ERR_INVALID_ARGUMENT, "st_module_param: entry index out of range");
    const st_module_entry_rec &e = module->entries[entry];
    if (param < 0 || static_cast<size_t>(param) >= e.kinds.size())
        return fail(ST_ERR_INVALID_ARGUMENT, "st_module_param: parameter index out of range");
    if (kind) *kind = e.kinds[param];
    if (dtype) *dtype = e.dtypes[param];
    return ST_OK;
}

extern "C" int st_launch_module(st_ctx *ctx, const st_module *module, const char *entry_name, const st_grid *grid,
                                const st_param *params, int32_t n_params, const st_exec *exec) {
    if (!module) return fail(ST_ERR_INVALID_ARGUMENT, "st_launch_module: module is null");
    const st_module_entry_rec *e = find_module_entry(module, entry_name);
    if (!e) {
        if (!entry_name)
            return fail(ST_ERR_INVALID_ARGUMENT, "the module holds " + std::to_string(module->entries.size()) +
                                                     " entries: name the one to launch");
        return fail(ST_ERR_UNKNOWN_ENTRY, std::string("Entry point ") + entry_name + " was not found in the module.");
    }
    if (!e->backend)
        return fail(ST_ERR_UNKNOWN_ENTRY, "entry " + e->name +
                                              " of the module has no sm_100a kernel here (known: vector_add, "
                                              "vector_fma, cast and *matmul* over f32 / f16 / bf16 arrays)");
    if (!params && n_params > 0) return fail(ST_ERR_INVALID_ARGUMENT, "st_launch_module: params is null");
    const int32_t n = static_cast<int32_t>(e->kinds.size());
    if (n_params < n || n_params > n + 3)
        return fail(ST_ERR_INVALID_ARGUMENT, "entry " + e->name + " takes " + std::to_string(n) +
                                                 " bindings (and up to 3 tile-size constants), got " +
                                                 std::to_string(n_params));
    for (int32_t i = 0; i < n; ++i) {
        const st_param &p = params[i];
        if (e->kinds[i] == ST_MODULE_PARAM_BUFFER) {
            if (p.kind != ST_PARAM_BUFFER)
                return fail(ST_ERR_INVALID_ARGUMENT, "binding " + std::to_string(i) + " of " + e->name +
                                                         " is a buffer in the module");
            if (p.dtype != e->dtypes[i])
                return fail(ST_ERR_INVALID_ARGUMENT, "binding " + std::to_string(i) + " of " + e->name +
                                                         ": the module declares " + dtype_name(e->dtypes[i]) +
                                                         " data, got " + dtype_name(p.dtype));
        } else if (p.kind != ST_PARAM_I32) {
            return fail(ST_ERR_INVALID_ARGUMENT, "binding " + std::to_string(i) + " of " + e->name +
                                                     " is an i32 scalar in the module");
        }
    }
    if (n_params > n)  // the caller's own tile sizes
        return st_launch(ctx, e->backend, grid, params, n_params, exec);
    if (e->n_constants == 0)
        return fail(ST_ERR_INVALID_ARGUMENT, "the tile sizes of entry " + e->name +
                                                 " cannot be read unambiguously from this module: pass them as "
                                                 "trailing i32 constants");
    std::vector<st_param> all(params, params + n);
    for (int i = 0; i < e->n_constants; ++i) all.push_back(st_param{ST_PARAM_I32, ST_I32, nullptr, 0, e->constants[i]});
    return st_launch(ctx, e->backend, grid, all.data(), static_cast<int32_t>(all.size()), exec);
}
