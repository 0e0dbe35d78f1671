// run_compute_example.cpp -- the reference's two host-side tests
// (src/examples.cpp: run_vector_add_test, run_matmul_test) written against
// the C ABI of include/sptiles_b200.h, with no Python: device buffers in
// place of Vulkan buffers, st_launch in place of run_compute.
//
// Inputs are the reference tests' own: a[i] = i, b[i] = 1000 + i for the add
// (examples.cpp:477-480), A = ((i mod 17) - 8) / 4 and B = ((i mod 13) - 6) / 2
// for the matmul (examples.cpp:590-596).  Both products are exact in fp32,
// so results are compared bit for bit with a sequential CPU loop (and the
// reference's own |diff| <= 1e-3 holds a fortiori).
//
// It then splits host-memory calls over every visible device in one process
// (the single-box partitioner, ST_EXEC_ALL_DEVICES).
//
// Given .tilebc paths on the command line, it also does what the
// reference's translator front end does with a module (src/main.cpp:75-187):
// load it, list its entries, and run each vector_add / matmul_fp32 entry
// (st_launch_module) with the module's own tile sizes on the same inputs.
//
// Exit status: 0 all checks passed, 1 a mismatch or a library error, 2 no
// CUDA device (st_init failed).
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <vector>

#include "sptiles_b200.h"

namespace {

st_ctx *g_ctx = nullptr;

bool ok(int rc, const char *what) {
    if (rc == ST_OK) return true;
    std::fprintf(stderr, "%s failed (%d): %s\n", what, rc, st_last_error());
    return false;
}

// One device buffer holding a copy of `host`.
void *device_copy(const std::vector<float> &host) {
    void *p = nullptr;
    const uint64_t bytes = host.size() * sizeof(float);
    if (!ok(st_alloc(g_ctx, -1, bytes, &p), "st_alloc")) return nullptr;
    if (!ok(st_upload(g_ctx, -1, p, host.data(), bytes), "st_upload")) return nullptr;
    return p;
}

st_param buffer(void *p, size_t elems) { return st_param{ST_PARAM_BUFFER, ST_F32, p, elems * sizeof(float), 0}; }
st_param i32(int64_t v) { return st_param{ST_PARAM_I32, 0, nullptr, 0, v}; }

// vector_add with the runner's 9 bindings and 1024-wide dispatch.
bool vector_add_test(uint32_t n) {
    std::vector<float> a(n), b(n), c(n, 0.0f);
    for (uint32_t i = 0; i < n; ++i) {
        a[i] = static_cast<float>(i);
        b[i] = static_cast<float>(1000 + i);
    }
    void *da = device_copy(a), *db = device_copy(b), *dc = device_copy(c);
    if (!da || !db || !dc) return false;
    const st_param p[9] = {buffer(da, n), i32(n), i32(1), buffer(db, n), i32(n), i32(1),
                           buffer(dc, n), i32(n), i32(1)};
    const uint32_t dispatch[3] = {(n + 1023) / 1024, 1, 1};
    st_grid grid;
    if (!ok(st_grid_from_dispatch("vector_add", dispatch, 1024, &grid), "st_grid_from_dispatch")) return false;
    const st_exec ex = {nullptr, -1, ST_EXEC_SYNC, 60000, nullptr, 0};
    if (!ok(st_launch(g_ctx, "vector_add", &grid, p, 9, &ex), "st_launch(vector_add)")) return false;
    if (!ok(st_download(g_ctx, -1, c.data(), dc, n * sizeof(float)), "st_download")) return false;
    st_free(g_ctx, -1, da);
    st_free(g_ctx, -1, db);
    st_free(g_ctx, -1, dc);
    for (uint32_t i = 0; i < n; ++i)
        if (c[i] != a[i] + b[i] || std::fabs(c[i] - (a[i] + b[i])) > 1e-3f) {
            std::fprintf(stderr, "vector_add n=%u: c[%u] = %g, want %g\n", n, i, c[i], a[i] + b[i]);
            return false;
        }
    std::printf("vector_add n=%u ok\n", n);
    return true;
}

// matmul_fp32 with the runner's 15 bindings (data, dim0, dim1, stride0,
// stride1 for A, B, C) and one 1024-invocation workgroup per 32 x 32 tile.
bool matmul_test(int m, int n, int k) {
    std::vector<float> a(static_cast<size_t>(m) * k), b(static_cast<size_t>(k) * n), c(static_cast<size_t>(m) * n, 0.0f);
    for (size_t i = 0; i < a.size(); ++i) a[i] = static_cast<float>(static_cast<int>(i % 17) - 8) * 0.25f;
    for (size_t i = 0; i < b.size(); ++i) b[i] = static_cast<float>(static_cast<int>(i % 13) - 6) * 0.5f;
    void *da = device_copy(a), *db = device_copy(b), *dc = device_copy(c);
    if (!da || !db || !dc) return false;
    const st_param p[15] = {buffer(da, a.size()), i32(m), i32(k), i32(k), i32(1),
                            buffer(db, b.size()), i32(k), i32(n), i32(n), i32(1),
                            buffer(dc, c.size()), i32(m), i32(n), i32(n), i32(1)};
    const uint32_t tiles = static_cast<uint32_t>(((m + 31) / 32) * ((n + 31) / 32));
    const uint32_t dispatch[3] = {tiles, 1, 1};
    st_grid grid;
    if (!ok(st_grid_from_dispatch("matmul_fp32", dispatch, 32 * 32, &grid), "st_grid_from_dispatch")) return false;
    const st_exec ex = {nullptr, -1, ST_EXEC_SYNC, 60000, nullptr, 0};
    if (!ok(st_launch(g_ctx, "matmul_fp32", &grid, p, 15, &ex), "st_launch(matmul_fp32)")) return false;
    if (!ok(st_download(g_ctx, -1, c.data(), dc, c.size() * sizeof(float)), "st_download")) return false;
    st_free(g_ctx, -1, da);
    st_free(g_ctx, -1, db);
    st_free(g_ctx, -1, dc);
    for (int i = 0; i < m; ++i)
        for (int j = 0; j < n; ++j) {
            float acc = 0.0f;  // the reference test's CPU loop: k ascending, fp32
            for (int q = 0; q < k; ++q) acc += a[static_cast<size_t>(i) * k + q] * b[static_cast<size_t>(q) * n + j];
            const float got = c[static_cast<size_t>(i) * n + j];
            if (got != acc) {
                std::fprintf(stderr, "matmul %dx%dx%d: C[%d,%d] = %g, want %g\n", m, n, k, i, j, got, acc);
                return false;
            }
        }
    std::printf("matmul_fp32 %dx%dx%d ok\n", m, n, k);
    return true;
}

// Known answers through a module entry: vector_add (a = i, b = 1000 + i) and
// matmul_fp32 (the mod-17 / mod-13 values), with the module's tile grid.
bool module_entry_test(const st_module *mod, const st_module_entry_info &e) {
    const st_exec ex = {nullptr, -1, ST_EXEC_SYNC, 60000, nullptr, 0};
    if (e.backend_entry && std::strcmp(e.backend_entry, "vector_add") == 0 && e.n_constants == 1) {
        const uint32_t n = 4112, tile = static_cast<uint32_t>(e.constants[0]);
        std::vector<float> a(n), b(n), c(n, 0.0f);
        for (uint32_t i = 0; i < n; ++i) {
            a[i] = static_cast<float>(i);
            b[i] = static_cast<float>(1000 + i);
        }
        void *da = device_copy(a), *db = device_copy(b), *dc = device_copy(c);
        if (!da || !db || !dc) return false;
        const st_param p[9] = {buffer(da, n), i32(n), i32(1), buffer(db, n), i32(n), i32(1),
                               buffer(dc, n), i32(n), i32(1)};
        const st_grid grid = {(n + tile - 1) / tile, 1, 1};
        if (!ok(st_launch_module(g_ctx, mod, e.name, &grid, p, 9, &ex), "st_launch_module(vector_add)")) return false;
        if (!ok(st_download(g_ctx, -1, c.data(), dc, n * sizeof(float)), "st_download")) return false;
        st_free(g_ctx, -1, da);
        st_free(g_ctx, -1, db);
        st_free(g_ctx, -1, dc);
        for (uint32_t i = 0; i < n; ++i)
            if (c[i] != a[i] + b[i]) {
                std::fprintf(stderr, "module vector_add: c[%u] = %g, want %g\n", i, c[i], a[i] + b[i]);
                return false;
            }
        std::printf("module %s tile=%u n=%u ok\n", e.name, tile, n);
        return true;
    }
    if (e.backend_entry && std::strcmp(e.backend_entry, "matmul_fp32") == 0 && e.n_constants == 3) {
        const int m = 100, n = 70, k = 33, tm = e.constants[0], tn = e.constants[1];
        std::vector<float> a(static_cast<size_t>(m) * k), b(static_cast<size_t>(k) * n), c(static_cast<size_t>(m) * n);
        for (size_t i = 0; i < a.size(); ++i) a[i] = static_cast<float>(static_cast<int>(i % 17) - 8) * 0.25f;
        for (size_t i = 0; i < b.size(); ++i) b[i] = static_cast<float>(static_cast<int>(i % 13) - 6) * 0.5f;
        void *da = device_copy(a), *db = device_copy(b), *dc = device_copy(c);
        if (!da || !db || !dc) return false;
        const st_param p[15] = {buffer(da, a.size()), i32(m), i32(k), i32(k), i32(1),
                                buffer(db, b.size()), i32(k), i32(n), i32(n), i32(1),
                                buffer(dc, c.size()), i32(m), i32(n), i32(n), i32(1)};
        const st_grid grid = {static_cast<uint32_t>(((m + tm - 1) / tm) * ((n + tn - 1) / tn)), 1, 1};
        if (!ok(st_launch_module(g_ctx, mod, e.name, &grid, p, 15, &ex), "st_launch_module(matmul)")) return false;
        if (!ok(st_download(g_ctx, -1, c.data(), dc, c.size() * sizeof(float)), "st_download")) return false;
        st_free(g_ctx, -1, da);
        st_free(g_ctx, -1, db);
        st_free(g_ctx, -1, dc);
        for (int i = 0; i < m; ++i)
            for (int j = 0; j < n; ++j) {
                float acc = 0.0f;
                for (int q = 0; q < k; ++q) acc += a[static_cast<size_t>(i) * k + q] * b[static_cast<size_t>(q) * n + j];
                if (c[static_cast<size_t>(i) * n + j] != acc) {
                    std::fprintf(stderr, "module matmul: C[%d,%d] = %g, want %g\n", i, j,
                                 c[static_cast<size_t>(i) * n + j], acc);
                    return false;
                }
            }
        std::printf("module %s tiles=%dx%dx%d ok\n", e.name, tm, tn, e.constants[2]);
        return true;
    }
    std::printf("module %s: not run by this example\n", e.name);
    return true;
}

// The single-box partitioner in one process: a context over every visible
// device, host-memory calls split across them (ST_EXEC_ALL_DEVICES).
bool partitioner_test() {
    int32_t count = 0;
    if (!ok(st_device_count(&count), "st_device_count") || count < 1) return false;
    std::vector<int32_t> devs(count);
    for (int32_t i = 0; i < count; ++i) devs[i] = i;
    st_ctx *all = nullptr;
    if (!ok(st_init(devs.data(), count, &all), "st_init(all devices)")) return false;
    const st_exec ex = {nullptr, -1, ST_EXEC_ALL_DEVICES, 60000, nullptr, 0};
    bool good = true;
    {  // matmul_fp32 known answer, ragged: rows in 128-row blocks per device
        const int m = 1000, n = 700, k = 333;
        std::vector<float> a(static_cast<size_t>(m) * k), b(static_cast<size_t>(k) * n), c(static_cast<size_t>(m) * n);
        for (size_t i = 0; i < a.size(); ++i) a[i] = static_cast<float>(static_cast<int>(i % 17) - 8) * 0.25f;
        for (size_t i = 0; i < b.size(); ++i) b[i] = static_cast<float>(static_cast<int>(i % 13) - 6) * 0.5f;
        const st_tensor ta = {a.data(), ST_F32, 2, {m, k}, {k, 1}};
        const st_tensor tb = {b.data(), ST_F32, 2, {k, n}, {n, 1}};
        const st_tensor tc = {c.data(), ST_F32, 2, {m, n}, {n, 1}};
        good = ok(st_matmul_host(all, &ta, &tb, nullptr, &tc, &ex), "st_matmul_host(all devices)");
        for (int i = 0; good && i < m; ++i)
            for (int j = 0; good && j < n; ++j) {
                float acc = 0.0f;
                for (int q = 0; q < k; ++q) acc += a[static_cast<size_t>(i) * k + q] * b[static_cast<size_t>(q) * n + j];
                if (c[static_cast<size_t>(i) * n + j] != acc) {
                    std::fprintf(stderr, "partitioner matmul: C[%d,%d] = %g, want %g\n", i, j,
                                 c[static_cast<size_t>(i) * n + j], acc);
                    good = false;
                }
            }
        if (good) std::printf("partitioner matmul_fp32 %dx%dx%d on %d devices ok\n", m, n, k, count);
    }
    if (good) {  // vector_add by element ranges
        const int64_t n = 1000003;
        std::vector<float> a(n), b(n), c(n, 0.0f);
        for (int64_t i = 0; i < n; ++i) {
            a[i] = static_cast<float>(i);
            b[i] = static_cast<float>(1000 + i);
        }
        const st_tensor ta = {a.data(), ST_F32, 1, {n, 0}, {1, 0}};
        const st_tensor tb = {b.data(), ST_F32, 1, {n, 0}, {1, 0}};
        const st_tensor tc = {c.data(), ST_F32, 1, {n, 0}, {1, 0}};
        good = ok(st_vector_add_host(all, &ta, &tb, &tc, &ex), "st_vector_add_host(all devices)");
        for (int64_t i = 0; good && i < n; ++i)
            if (c[i] != a[i] + b[i]) {
                std::fprintf(stderr, "partitioner vector_add: c[%lld] = %g\n", static_cast<long long>(i), c[i]);
                good = false;
            }
        if (good) std::printf("partitioner vector_add n=%lld on %d devices ok\n", static_cast<long long>(n), count);
    }
    st_shutdown(all);
    return good;
}

bool module_test(const char *path) {
    st_module *mod = nullptr;
    if (!ok(st_module_load_file(path, &mod), "st_module_load_file")) return false;
    int32_t major = 0, minor = 0, count = 0;
    st_module_version(mod, &major, &minor, nullptr);
    st_module_entry_count(mod, &count);
    std::printf("loaded %s: TileIR bytecode %d.%d, %d entries\n", path, major, minor, count);
    bool all = true;
    for (int32_t i = 0; i < count; ++i) {
        st_module_entry_info e;
        if (!ok(st_module_entry(mod, i, &e), "st_module_entry")) {
            all = false;
            continue;
        }
        std::printf("  entry %s: %d bindings, %d arrays, backend %s\n", e.name, e.n_params, e.n_arrays,
                    e.backend_entry ? e.backend_entry : "(none)");
        all = module_entry_test(mod, e) && all;
    }
    st_module_free(mod);
    return all;
}

}  // namespace

int main(int argc, char **argv) {
    std::printf("library %s\n", st_version());
    if (st_init(nullptr, 0, &g_ctx) != ST_OK) {
        std::fprintf(stderr, "no CUDA device: %s\n", st_last_error());
        return 2;
    }
    bool all = true;
    for (uint32_t n : {1024u, 2048u, 4112u}) all = vector_add_test(n) && all;
    const int shapes[4][3] = {{64, 64, 64}, {256, 256, 256}, {100, 70, 33}, {33, 129, 200}};
    for (const auto &s : shapes) all = matmul_test(s[0], s[1], s[2]) && all;
    for (int i = 1; i < argc; ++i) all = module_test(argv[i]) && all;
    st_shutdown(g_ctx);
    all = partitioner_test() && all;
    std::printf(all ? "all checks passed\n" : "FAILED\n");
    return all ? 0 : 1;
}
