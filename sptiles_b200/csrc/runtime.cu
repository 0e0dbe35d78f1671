// runtime.cu -- the host runtime behind the C ABI (include/sptiles_b200.h).
//
// It replaces the reference's Vulkan host (src/examples.cpp:133-448) and the
// Kompute runner (shaders/spirv_runtime.py:153-174): instead of building a
// pipeline from SPIR-V per call, a named cuda_tile entry is looked up in a
// registry of hand-written sm_100a kernels, its cutile_python_v1 bindings are
// turned back into tensor views, the cuda_tile grid is mapped onto the
// kernels' own launch shape, and the work is queued on a CUDA stream.
// Waits are bounded (an event poll with a deadline) where the reference
// waited on a fence forever (examples.cpp:439).
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

#include "common.h"

namespace st {

static thread_local std::string g_last_error;
static std::atomic<uint64_t> g_launches{0};

void note_launch(uint64_t n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

bool pdl_enabled() {
    static const bool on = [] {
        const char *v = std::getenv("SPTILES_B200_PDL");
        return !(v != nullptr && v[0] == '0');
    }();
    return on;
}

int fail(int code, const std::string &msg) {
    g_last_error = msg;
    return code;
}

int cuda_fail(cudaError_t e, const char *what) {
    const int code = (e == cudaErrorMemoryAllocation) ? ST_ERR_OUT_OF_MEMORY
                     : (e == cudaErrorNoDevice || e == cudaErrorInsufficientDriver) ? ST_ERR_NO_DEVICE
                                                                                     : ST_ERR_CUDA;
    return fail(code, std::string(what) + ": " + cudaGetErrorName(e) + " (" + cudaGetErrorString(e) + ")");
}

namespace {

constexpr uint32_t kDefaultTimeoutMs = 60000;
// bound for every on-device barrier wait of the tensor-core kernels
constexpr uint64_t kDeviceWaitLimitNs = 4ull * 1000 * 1000 * 1000;

// A device buffer the runtime owns and grows on demand (operand packing,
// staging of host-memory calls).  `ready` orders reuse across streams.
struct Workspace {
    void *ptr = nullptr;
    size_t bytes = 0;
    cudaEvent_t ready = nullptr;
};

struct DeviceState {
    int ordinal = 0;
    int sm_count = 0;
    cudaStream_t stream = nullptr;
    int *dev_err = nullptr;
    Workspace scratch;  // packed / repacked matmul operands
    Workspace stage;    // device copies of host-memory arguments
    Workspace sk;       // stream-K partials and flags of the CTA-pair GEMM (fixed size, flags zeroed)
    // host-memory calls: copies in and out run on their own streams so that
    // both PCIe directions overlap the kernels
    cudaStream_t copy_in = nullptr;
    cudaStream_t copy_out = nullptr;
    std::vector<cudaEvent_t> events;  // reusable ordering events
};

class DeviceGuard {
  public:
    explicit DeviceGuard(int dev) {
        cudaGetDevice(&prev_);
        cudaSetDevice(dev);
    }
    ~DeviceGuard() { cudaSetDevice(prev_); }

  private:
    int prev_ = 0;
};

}  // namespace
}  // namespace st

struct st_ctx {
    std::vector<st::DeviceState> devs;
};

namespace st {
namespace {

DeviceState *find_dev(st_ctx *ctx, int device) {
    if (!ctx || ctx->devs.empty()) return nullptr;
    if (device < 0) return &ctx->devs[0];
    for (auto &d : ctx->devs)
        if (d.ordinal == device) return &d;
    return nullptr;
}

int get_dev(st_ctx *ctx, int device, DeviceState **out) {
    if (!ctx) return fail(ST_ERR_INVALID_ARGUMENT, "null context");
    DeviceState *d = find_dev(ctx, device);
    if (!d) return fail(ST_ERR_INVALID_ARGUMENT, "device " + std::to_string(device) + " is not part of the context");
    *out = d;
    return ST_OK;
}

bool capturing(cudaStream_t stream) {
    cudaStreamCaptureStatus st = cudaStreamCaptureStatusNone;
    return cudaStreamIsCapturing(stream, &st) == cudaSuccess && st != cudaStreamCaptureStatusNone;
}

// Grow `ws` to at least `need` bytes for use on `stream`.  While `stream` is
// being captured into a CUDA graph the buffer must already be large enough
// (a warm-up call sizes it) and stream order alone sequences its users.
int ws_acquire(Workspace &ws, size_t need, cudaStream_t stream, void **out) {
    if (capturing(stream)) {
        if (need > ws.bytes)
            return fail(ST_ERR_UNSUPPORTED, "the workspace must be sized by an uncaptured call before graph capture");
        *out = ws.ptr;
        return ST_OK;
    }
    if (ws.ready == nullptr) ST_CUDA_TRY(cudaEventCreateWithFlags(&ws.ready, cudaEventDisableTiming));
    // a previous user on another stream must be done with the buffer
    ST_CUDA_TRY(cudaStreamWaitEvent(stream, ws.ready, 0));
    if (need > ws.bytes) {
        if (ws.ptr) {
            ST_CUDA_TRY(cudaStreamSynchronize(stream));
            ST_CUDA_TRY(cudaFree(ws.ptr));
            ws.ptr = nullptr;
            ws.bytes = 0;
        }
        const size_t rounded = (need + (size_t(2) << 20) - 1) & ~((size_t(2) << 20) - 1);
        ST_CUDA_TRY(cudaMalloc(&ws.ptr, rounded));
        ws.bytes = rounded;
    }
    *out = ws.ptr;
    return ST_OK;
}

int ws_release(Workspace &ws, cudaStream_t stream) {
    if (capturing(stream)) return ST_OK;
    ST_CUDA_TRY(cudaEventRecord(ws.ready, stream));
    return ST_OK;
}

void ws_free(Workspace &ws) {
    if (ws.ptr) cudaFree(ws.ptr);
    if (ws.ready) cudaEventDestroy(ws.ready);
    ws = Workspace{};
}

// The stream-K workspace: allocated with its flags zeroed by the first
// uncaptured matmul on the device (a capture before that runs whole tiles
// only), then ordered across streams like the other workspaces.
int sk_acquire(DeviceState *d, cudaStream_t stream, GemmArgs &g) {
    if (!d->sk.ptr) {
        if (capturing(stream)) return ST_OK;
        const size_t bytes = stream_k_workspace_bytes(d->sm_count);
        ST_CUDA_TRY(cudaMalloc(&d->sk.ptr, bytes));
        d->sk.bytes = bytes;
        ST_CUDA_TRY(cudaMemsetAsync(d->sk.ptr, 0, bytes, stream));
    }
    void *base = nullptr;
    ST_TRY(ws_acquire(d->sk, d->sk.bytes, stream, &base));
    g.sk_ws = static_cast<float *>(base);
    g.sk_flags = reinterpret_cast<int *>(static_cast<uint8_t *>(base) + stream_k_flag_offset(d->sm_count));
    return ST_OK;
}

// After an abort a split tile's flags may still be raised: clear them.
void sk_reset(DeviceState *d) {
    if (!d->sk.ptr) return;
    DeviceGuard guard(d->ordinal);
    const size_t off = stream_k_flag_offset(d->sm_count);
    cudaMemset(static_cast<uint8_t *>(d->sk.ptr) + off, 0, d->sk.bytes - off);
    cudaDeviceSynchronize();
}

// Bounded wait for `stream`, then collect a kernel abort from the error word.
int bounded_sync(DeviceState *d, cudaStream_t stream, uint32_t timeout_ms) {
    if (timeout_ms == 0) timeout_ms = kDefaultTimeoutMs;
    cudaEvent_t ev;
    ST_CUDA_TRY(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
    cudaError_t e = cudaEventRecord(ev, stream);
    if (e != cudaSuccess) {
        cudaEventDestroy(ev);
        return cuda_fail(e, "cudaEventRecord");
    }
    const auto deadline = std::chrono::steady_clock::now() + std::chrono::milliseconds(timeout_ms);
    int sleep_us = 2;
    while ((e = cudaEventQuery(ev)) == cudaErrorNotReady) {
        if (std::chrono::steady_clock::now() > deadline) {
            cudaEventDestroy(ev);
            return fail(ST_ERR_TIMEOUT, "work did not finish within " + std::to_string(timeout_ms) + " ms");
        }
        std::this_thread::sleep_for(std::chrono::microseconds(sleep_us));
        if (sleep_us < 200) sleep_us *= 2;
    }
    cudaEventDestroy(ev);
    if (e != cudaSuccess) return cuda_fail(e, "kernel execution");
    int code = 0;
    ST_CUDA_TRY(cudaMemcpy(&code, d->dev_err, sizeof(int), cudaMemcpyDeviceToHost));
    if (code != 0) {
        ST_CUDA_TRY(cudaMemset(d->dev_err, 0, sizeof(int)));
        sk_reset(d);
        return fail(ST_ERR_DEVICE_ABORT, "a kernel gave up a bounded wait (code " + std::to_string(code) + ")");
    }
    return ST_OK;
}

struct ExecCtx {
    DeviceState *dev = nullptr;
    cudaStream_t stream = nullptr;
    uint32_t timeout_ms = kDefaultTimeoutMs;
    int flags = 0;
};

constexpr const char *kAllDevicesScope =
    "ST_EXEC_ALL_DEVICES applies to st_vector_add_host, st_matmul_host and st_launch with ST_EXEC_HOST_BUFFERS only";

// `split_ok`: the call implements ST_EXEC_ALL_DEVICES (the host-memory
// vector_add and matmul); every other entry point refuses the flag rather
// than running on one device only.
int resolve_exec(st_ctx *ctx, const st_exec *exec, ExecCtx *out, bool split_ok = false) {
    if (exec && (exec->flags & ST_EXEC_ALL_DEVICES) && !split_ok) return fail(ST_ERR_INVALID_ARGUMENT, kAllDevicesScope);
    const int device = exec ? exec->device : -1;
    ST_TRY(get_dev(ctx, device, &out->dev));
    out->stream = (exec && exec->stream) ? static_cast<cudaStream_t>(exec->stream) : out->dev->stream;
    out->timeout_ms = (exec && exec->timeout_ms) ? exec->timeout_ms : kDefaultTimeoutMs;
    out->flags = exec ? exec->flags : 0;
    return ST_OK;
}

// ------------------------------------------------------------ tensor checks
int check_view(const st_tensor *t, const char *name, int rank) {
    if (!t) return fail(ST_ERR_INVALID_ARGUMENT, std::string(name) + " is null");
    if (t->rank != rank)
        return fail(ST_ERR_INVALID_ARGUMENT,
                    std::string(name) + " must be rank " + std::to_string(rank) + ", got " + std::to_string(t->rank));
    if (dtype_size(t->dtype) == 0) return fail(ST_ERR_INVALID_ARGUMENT, std::string(name) + " has an unknown dtype");
    for (int i = 0; i < rank; ++i) {
        if (t->shape[i] < 0) return fail(ST_ERR_INVALID_ARGUMENT, std::string(name) + " has a negative extent");
        if (t->strides[i] < 0) return fail(ST_ERR_INVALID_ARGUMENT, std::string(name) + " has a negative stride");
    }
    bool empty = false;
    for (int i = 0; i < rank; ++i) empty |= t->shape[i] == 0;
    if (!empty && !t->data) return fail(ST_ERR_INVALID_ARGUMENT, std::string(name) + " has a null data pointer");
    return ST_OK;
}

int64_t view_span(const st_tensor &t) {  // elements from base to last element + 1
    int64_t span = 1;
    for (int i = 0; i < t.rank; ++i) {
        if (t.shape[i] == 0) return 0;
        span += (t.shape[i] - 1) * t.strides[i];
    }
    return span;
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ------------------------------------------------------------ vector add
int vector_add_views(const ExecCtx &x, const st_tensor &a, const st_tensor &b, const st_tensor &c, int64_t rows,
                     int64_t cols) {
    if (c.rank == 1)
        return launch_vector_add_1d(static_cast<const float *>(a.data), a.strides[0],
                                    static_cast<const float *>(b.data), b.strides[0], static_cast<float *>(c.data),
                                    c.strides[0], cols, x.dev->sm_count, x.stream);
    return launch_vector_add_2d(static_cast<const float *>(a.data), a.strides, static_cast<const float *>(b.data),
                                b.strides, static_cast<float *>(c.data), c.strides, rows, cols, x.dev->sm_count,
                                x.stream);
}

int check_vector_add(const st_tensor *a, const st_tensor *b, const st_tensor *c) {
    if (!a || !b || !c) return fail(ST_ERR_INVALID_ARGUMENT, "vector_add: null tensor");
    const int rank = c->rank;
    if (rank != 1 && rank != 2) return fail(ST_ERR_INVALID_ARGUMENT, "vector_add: tensors must be rank 1 or 2");
    ST_TRY(check_view(a, "A", rank));
    ST_TRY(check_view(b, "B", rank));
    ST_TRY(check_view(c, "C", rank));
    for (const st_tensor *t : {a, b, c})
        if (t->dtype != ST_F32)
            return fail(ST_ERR_INVALID_ARGUMENT, "vector_add: the lowering is f32-only; tensors must be ST_F32");
    for (int i = 0; i < rank; ++i)
        if (a->shape[i] != c->shape[i] || b->shape[i] != c->shape[i])
            return fail(ST_ERR_INVALID_ARGUMENT, "vector_add: A, B and C must have the same shape");
    return ST_OK;
}

// ------------------------------------------------------------ matmul
int check_matmul(const st_tensor *a, const st_tensor *b, const st_tensor *bias, const st_tensor *c) {
    ST_TRY(check_view(a, "A", 2));
    ST_TRY(check_view(b, "B", 2));
    ST_TRY(check_view(c, "C", 2));
    if (a->shape[1] != b->shape[0])
        return fail(ST_ERR_INVALID_ARGUMENT, "Incompatible matrices: K dimension of A (" + std::to_string(a->shape[1]) +
                                                 ") must match K dimension of B (" + std::to_string(b->shape[0]) + ")");
    if (c->shape[0] != a->shape[0] || c->shape[1] != b->shape[1])
        return fail(ST_ERR_INVALID_ARGUMENT, "C must be [M, N] = [" + std::to_string(a->shape[0]) + ", " +
                                                 std::to_string(b->shape[1]) + "]");
    if (a->dtype != b->dtype) return fail(ST_ERR_INVALID_ARGUMENT, "A and B must have the same dtype");
    if (a->dtype != ST_F32 && a->dtype != ST_F16 && a->dtype != ST_BF16)
        return fail(ST_ERR_INVALID_ARGUMENT, "A and B must be ST_F32, ST_F16 or ST_BF16");
    if (c->dtype != ST_F32 && c->dtype != ST_F16 && c->dtype != ST_BF16)
        return fail(ST_ERR_INVALID_ARGUMENT, "C must be ST_F32, ST_F16 or ST_BF16");
    if (c->shape[0] > 0 && c->shape[1] > 1 && c->strides[1] != 1)
        return fail(ST_ERR_UNSUPPORTED, "C must have unit column stride");
    if (a->shape[0] > INT32_MAX || b->shape[1] > INT32_MAX || a->shape[1] > INT32_MAX)
        return fail(ST_ERR_UNSUPPORTED, "matmul extents must fit in int32 (cuda_tile index type)");
    if (bias) {
        ST_TRY(check_view(bias, "bias", 1));
        if (bias->shape[0] != b->shape[1]) return fail(ST_ERR_INVALID_ARGUMENT, "bias must have N elements");
        if (bias->dtype != ST_F32 && bias->dtype != a->dtype)
            return fail(ST_ERR_INVALID_ARGUMENT, "bias must be ST_F32 or the input dtype");
        if (bias->shape[0] > 1 && bias->strides[0] != 1)
            return fail(ST_ERR_UNSUPPORTED, "bias must be contiguous");
    }
    return ST_OK;
}

__global__ void fill_rows_kernel(void *c, int64_t ldc, int c_dtype, const void *bias, int bias_dtype, int64_t m,
                                 int64_t n) {
    pdl_wait();
    const int64_t total = m * n;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t r = i / n, q = i - r * n;
        float v = 0.0f;
        if (bias) {
            if (bias_dtype == ST_F32) v = static_cast<const float *>(bias)[q];
            else if (bias_dtype == ST_F16) v = __half2float(static_cast<const __half *>(bias)[q]);
            else v = __bfloat162float(static_cast<const __nv_bfloat16 *>(bias)[q]);
            v = 0.0f + v;
        }
        if (c_dtype == ST_F32) static_cast<float *>(c)[r * ldc + q] = v;
        else if (c_dtype == ST_F16) static_cast<__half *>(c)[r * ldc + q] = __float2half_rn(v);
        else static_cast<__nv_bfloat16 *>(c)[r * ldc + q] = __float2bfloat16_rn(v);
    }
    pdl_trigger();
}

int matmul_device(const ExecCtx &x, const st_tensor &a, const st_tensor &b, const st_tensor *bias,
                  const st_tensor &c, const PeerOutputs *peers = nullptr) {
    const int64_t M = a.shape[0], K = a.shape[1], N = b.shape[1];
    if (M == 0 || N == 0) return ST_OK;
    const void *bias_ptr = bias ? bias->data : nullptr;
    const int bias_dtype = bias ? bias->dtype : ST_F32;
    if (K == 0) {  // empty contraction: C = 0 (+ bias)
        if (peers && peers->n > 0) return fail(ST_ERR_UNSUPPORTED, "K = 0 with peer outputs");
        ST_CUDA_TRY(launch_kernel(fill_rows_kernel, 148, 256, 0, x.stream, c.data, c.strides[0], c.dtype, bias_ptr,
                                  bias_dtype, M, N));
        note_launch();
        const cudaError_t e = cudaPeekAtLastError();
        return e == cudaSuccess ? ST_OK : cuda_fail(cudaGetLastError(), "fill_rows_kernel");
    }
    GemmArgs g{};
    if (peers) g.peers = *peers;
    g.deterministic = (x.flags & ST_EXEC_DETERMINISTIC) != 0;
    g.c = c.data;
    g.ldc = c.strides[0];
    g.c_dtype = c.dtype;
    g.bias = bias_ptr;
    g.bias_dtype = bias_dtype;
    g.m = M;
    g.n = N;
    Workspace &ws = x.dev->scratch;
    if (a.dtype == ST_F32) {
        // Opt-in (SPTILES_B200_FP32_FUSED=1): split into tf32 hi/lo inside the
        // GEMM.  Its 128 x 64 tiles are bound by shared-memory bandwidth, so the
        // packed route below -- which can use the 256 x 256 CTA-pair kernel --
        // is faster from 2048^3 up (218 vs 61 TFLOP/s at 4096^3) and ties at 1024^3.
        const bool a_ok = (a.strides[1] == 1 || K == 1) && (a.strides[0] * 4) % 16 == 0 && aligned16(a.data);
        const bool b_rows_ok = (b.strides[1] == 1 || N == 1) && (b.strides[0] * 4) % 16 == 0 && aligned16(b.data);
        const bool b_cols_ok = (b.strides[0] == 1 || K == 1) && (b.strides[1] * 4) % 16 == 0 && aligned16(b.data);
        const char *fused = std::getenv("SPTILES_B200_FP32_FUSED");
        if (fused && fused[0] == '1' && a_ok && (b_rows_ok || b_cols_ok)) {
            g.ab_dtype = ST_F32;
            g.a = a.data;
            g.lda = a.strides[0];
            g.b = b.data;
            g.b_k_major = !b_rows_ok;
            g.ldb = b_rows_ok ? b.strides[0] : b.strides[1];
            g.k = K;
            return launch_gemm_3xtf32(g, x.dev->sm_count, x.dev->dev_err, kDeviceWaitLimitNs, x.stream);
        }
        // Opt-in (SPTILES_B200_FP32=split): operands TMA can address in place, on
        // a CTA-pair plan, are split into tf32 hi / lo by the pair kernel itself,
        // with no packing pass.  Its converter traffic makes it shared-memory
        // bound (~70 % of the MMA rate): it ties with packing at 1024^3 and
        // loses from 2048^3 up (750 vs 578 us at 4096^3), so packing is the default.
        const char *route = std::getenv("SPTILES_B200_FP32");
        if (route && std::strcmp(route, "split") == 0 && a_ok && (b_rows_ok || b_cols_ok)) {
            GemmArgs gs = g;
            gs.ab_dtype = ST_F32;
            gs.a = a.data;
            gs.lda = a.strides[0];
            gs.b = b.data;
            gs.b_k_major = !b_rows_ok;
            gs.ldb = b_rows_ok ? b.strides[0] : b.strides[1];
            gs.k = K;
            gs.split_fp32 = true;
            if (gemm_split_fp32_fits(gs, x.dev->sm_count)) {
                if (gemm_uses_stream_k(gs, x.dev->sm_count)) ST_TRY(sk_acquire(x.dev, x.stream, gs));
                ST_TRY(launch_gemm(gs, x.dev->sm_count, x.dev->dev_err, kDeviceWaitLimitNs, x.stream));
                if (gs.sk_ws) ST_TRY(ws_release(x.dev->sk, x.stream));
                return ST_OK;
            }
        }
        // otherwise pack [hi|hi|lo] x [hi;lo;hi] into scratch and run one tf32 GEMM
        const int64_t kp = tf32_packed_k(K);
        const size_t need = static_cast<size_t>(M + N) * 3 * kp * sizeof(float);
        void *base = nullptr;
        ST_TRY(ws_acquire(ws, need, x.stream, &base));
        float *ap = static_cast<float *>(base);
        float *bp = ap + M * 3 * kp;
        g.ab_dtype = ST_F32;
        g.a = ap;
        g.lda = 3 * kp;
        g.b = bp;
        g.ldb = 3 * kp;
        g.b_k_major = true;
        g.k = 3 * kp;
        // split tiles that fold in L2 onto a preset C start from C = bias,
        // which the pack writes; the ordered fold and the exchange use the
        // stream-K workspace (an ordered launch captured before the workspace
        // exists presets C by its own kernel instead)
        if (gemm_uses_stream_k(g, x.dev->sm_count)) ST_TRY(sk_acquire(x.dev, x.stream, g));
        CPreset preset;
        if (stream_k_l2add_mode(g, x.dev->sm_count) == 1) {
            preset.c = static_cast<float *>(c.data);
            preset.ldc = c.strides[0];
            preset.bias = bias_ptr;
            preset.bias_dtype = bias_dtype;
            preset.m = static_cast<int>(M);
            preset.n = static_cast<int>(N);
            g.c_preset = true;
        }
        ST_TRY(launch_pack_ab_tf32(static_cast<const float *>(a.data), a.strides[0], a.strides[1], M,
                                   static_cast<const float *>(b.data), b.strides[0], b.strides[1], N, K, ap, bp, kp,
                                   g.c_preset ? &preset : nullptr, x.stream));
        ST_TRY(launch_gemm(g, x.dev->sm_count, x.dev->dev_err, kDeviceWaitLimitNs, x.stream));
        if (g.sk_ws) ST_TRY(ws_release(x.dev->sk, x.stream));
        return ws_release(ws, x.stream);
    }
    // 16-bit operands: use them in place when TMA can address them
    g.ab_dtype = a.dtype;
    g.k = K;
    const bool a_ok = (a.strides[1] == 1 || K == 1) && (a.strides[0] * 2) % 16 == 0 && aligned16(a.data);
    const bool b_rows_ok = (b.strides[1] == 1 || N == 1) && (b.strides[0] * 2) % 16 == 0 && aligned16(b.data);
    const bool b_cols_ok = (b.strides[0] == 1 || K == 1) && (b.strides[1] * 2) % 16 == 0 && aligned16(b.data);
    size_t need = 0;
    const int64_t lda_p = cdiv(K, 8) * 8, ldb_p = cdiv(N, 8) * 8;
    if (!a_ok) need += static_cast<size_t>(M) * lda_p * 2;
    if (!b_rows_ok && !b_cols_ok) need += static_cast<size_t>(K) * ldb_p * 2;
    void *base = nullptr;
    if (need) ST_TRY(ws_acquire(ws, need + 32, x.stream, &base));
    uint8_t *cursor = static_cast<uint8_t *>(base);
    if (a_ok) {
        g.a = a.data;
        g.lda = a.strides[0];
    } else {
        uint16_t *ap = reinterpret_cast<uint16_t *>(cursor);
        ST_TRY(launch_repack_16(static_cast<const uint16_t *>(a.data), a.strides[0], a.strides[1], M, K, ap, lda_p,
                                x.stream));
        cursor += (static_cast<size_t>(M) * lda_p * 2 + 15) & ~size_t(15);
        g.a = ap;
        g.lda = lda_p;
    }
    if (b_rows_ok) {
        g.b = b.data;
        g.ldb = b.strides[0];
        g.b_k_major = false;
    } else if (b_cols_ok) {  // B stored column-major, i.e. as B^T [N, K] with K contiguous
        g.b = b.data;
        g.ldb = b.strides[1];
        g.b_k_major = true;
    } else {
        uint16_t *bpk = reinterpret_cast<uint16_t *>(cursor);
        ST_TRY(launch_repack_16(static_cast<const uint16_t *>(b.data), b.strides[0], b.strides[1], K, N, bpk, ldb_p,
                                x.stream));
        g.b = bpk;
        g.ldb = ldb_p;
        g.b_k_major = false;
    }
    if (gemm_uses_stream_k(g, x.dev->sm_count)) ST_TRY(sk_acquire(x.dev, x.stream, g));
    ST_TRY(launch_gemm(g, x.dev->sm_count, x.dev->dev_err, kDeviceWaitLimitNs, x.stream));
    if (g.sk_ws) ST_TRY(ws_release(x.dev->sk, x.stream));
    if (need) return ws_release(ws, x.stream);
    return ST_OK;
}

int finish(const ExecCtx &x) {
    if (x.flags & ST_EXEC_SYNC) return bounded_sync(x.dev, x.stream, x.timeout_ms);
    return ST_OK;
}

// ------------------------------------------------------------ host staging
// Copy a host tensor into a dense device tensor carved from `cursor`.
int stage_in(const ExecCtx &x, const st_tensor &h, uint8_t *&cursor, st_tensor *d) {
    *d = h;
    const size_t es = dtype_size(h.dtype);
    d->data = cursor;
    if (h.rank == 1) {
        d->strides[0] = 1;
        const size_t bytes = static_cast<size_t>(h.shape[0]) * es;
        if (h.shape[0] > 1 && h.strides[0] != 1) return fail(ST_ERR_UNSUPPORTED, "host tensors must be contiguous");
        if (bytes) ST_CUDA_TRY(cudaMemcpyAsync(cursor, h.data, bytes, cudaMemcpyHostToDevice, x.stream));
        cursor += (bytes + 255) & ~size_t(255);
        return ST_OK;
    }
    const int64_t rows = h.shape[0], cols = h.shape[1];
    d->strides[0] = cols;
    d->strides[1] = 1;
    if (rows && cols) {
        if (cols > 1 && h.strides[1] != 1) return fail(ST_ERR_UNSUPPORTED, "host tensors must have unit column stride");
        const int64_t hs0 = rows > 1 ? h.strides[0] : cols;
        ST_CUDA_TRY(cudaMemcpy2DAsync(cursor, cols * es, h.data, hs0 * es, cols * es, rows, cudaMemcpyHostToDevice,
                                      x.stream));
    }
    cursor += (static_cast<size_t>(rows * cols) * es + 255) & ~size_t(255);
    return ST_OK;
}

int stage_out(const ExecCtx &x, const st_tensor &d, const st_tensor &h) {
    const size_t es = dtype_size(h.dtype);
    if (h.rank == 1) {
        if (h.shape[0] > 1 && h.strides[0] != 1) return fail(ST_ERR_UNSUPPORTED, "host tensors must be contiguous");
        if (h.shape[0])
            ST_CUDA_TRY(cudaMemcpyAsync(h.data, d.data, h.shape[0] * es, cudaMemcpyDeviceToHost, x.stream));
        return ST_OK;
    }
    const int64_t rows = h.shape[0], cols = h.shape[1];
    if (!rows || !cols) return ST_OK;
    if (cols > 1 && h.strides[1] != 1) return fail(ST_ERR_UNSUPPORTED, "host tensors must have unit column stride");
    const int64_t hs0 = rows > 1 ? h.strides[0] : cols;
    ST_CUDA_TRY(cudaMemcpy2DAsync(h.data, hs0 * es, d.data, d.strides[0] * es, cols * es, rows,
                                  cudaMemcpyDeviceToHost, x.stream));
    return ST_OK;
}

size_t staged_bytes(const st_tensor &t) {
    size_t n = dtype_size(t.dtype);
    for (int i = 0; i < t.rank; ++i) n *= static_cast<size_t>(t.shape[i]);
    return (n + 255) & ~size_t(255);
}

// ------------------------------------------------------------ pipelined host calls
// Event `i` of the device's pool (created on first use, reused afterwards).
int pool_event(DeviceState *d, size_t i, cudaEvent_t *out) {
    while (d->events.size() <= i) {
        cudaEvent_t e;
        ST_CUDA_TRY(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
        d->events.push_back(e);
    }
    *out = d->events[i];
    return ST_OK;
}

int ensure_copy_streams(DeviceState *d) {
    if (!d->copy_in) ST_CUDA_TRY(cudaStreamCreateWithFlags(&d->copy_in, cudaStreamNonBlocking));
    if (!d->copy_out) ST_CUDA_TRY(cudaStreamCreateWithFlags(&d->copy_out, cudaStreamNonBlocking));
    return ST_OK;
}

// `waiter` waits for everything issued so far on `signaller`.
int stream_after(DeviceState *d, size_t &ev_i, cudaStream_t waiter, cudaStream_t signaller) {
    cudaEvent_t e;
    ST_TRY(pool_event(d, ev_i++, &e));
    ST_CUDA_TRY(cudaEventRecord(e, signaller));
    ST_CUDA_TRY(cudaStreamWaitEvent(waiter, e, 0));
    return ST_OK;
}

bool host_rows_dense(const st_tensor &t) {  // unit column stride (rows may be padded)
    if (t.rank == 1) return t.shape[0] <= 1 || t.strides[0] == 1;
    return t.shape[1] <= 1 || t.strides[1] == 1;
}

// Block [r0, r1) x [c0, c1) of a rank-2 host tensor <-> the same block of a
// device matrix with row pitch `ld` elements.
int copy_block_in(cudaStream_t s, void *dev, int64_t ld, const st_tensor &h, int64_t r0, int64_t r1, int64_t c0,
                  int64_t c1) {
    const size_t es = dtype_size(h.dtype);
    if (r1 <= r0 || c1 <= c0) return ST_OK;
    const int64_t hs0 = h.shape[0] > 1 ? h.strides[0] : h.shape[1];
    const uint8_t *src = static_cast<const uint8_t *>(h.data) + static_cast<size_t>(r0 * hs0 + c0) * es;
    uint8_t *dst = static_cast<uint8_t *>(dev) + static_cast<size_t>(r0 * ld + c0) * es;
    ST_CUDA_TRY(cudaMemcpy2DAsync(dst, ld * es, src, hs0 * es, (c1 - c0) * es, r1 - r0, cudaMemcpyHostToDevice, s));
    return ST_OK;
}

int copy_block_out(cudaStream_t s, const st_tensor &h, const void *dev, int64_t ld, int64_t r0, int64_t r1,
                   int64_t c0, int64_t c1) {
    const size_t es = dtype_size(h.dtype);
    if (r1 <= r0 || c1 <= c0) return ST_OK;
    const int64_t hs0 = h.shape[0] > 1 ? h.strides[0] : h.shape[1];
    uint8_t *dst = static_cast<uint8_t *>(h.data) + static_cast<size_t>(r0 * hs0 + c0) * es;
    const uint8_t *src = static_cast<const uint8_t *>(dev) + static_cast<size_t>(r0 * ld + c0) * es;
    ST_CUDA_TRY(cudaMemcpy2DAsync(dst, hs0 * es, src, ld * es, (c1 - c0) * es, r1 - r0, cudaMemcpyDeviceToHost, s));
    return ST_OK;
}

// C = A @ B (+ bias) on host tensors with 16-bit A and B.  C[i, j] needs row
// i of A and column j of B, so the received rows of A and columns of B grow
// together: step s brings row block s of A and column block s of B (~16 MB
// each) on copy_in, then computes on the caller's stream
//   C[new rows, all columns so far]  and  C[earlier rows, new columns]
// and sends those blocks of C back on copy_out.  With A and B arriving in
// step, C comes out from the first ~2 blocks on and both PCIe directions
// stay busy (with B first, nothing leaves until all of B is in).  Device
// copies use row pitches rounded up to 8 elements, so every block view is a
// 16-byte-aligned TMA operand.
int matmul_host_pipelined(const ExecCtx &x, const st_tensor &a, const st_tensor &b, const st_tensor *bias,
                          const st_tensor &c, bool wait) {
    DeviceState *d = x.dev;
    ST_TRY(ensure_copy_streams(d));
    const int64_t M = a.shape[0], K = a.shape[1], N = b.shape[1];
    const size_t ein = dtype_size(a.dtype), eout = dtype_size(c.dtype);
    const int64_t lda = cdiv(K, 8) * 8, ldb = cdiv(N, 8) * 8, ldc = cdiv(N, 8) * 8;
    const size_t a_bytes = static_cast<size_t>(M * lda) * ein, b_bytes = static_cast<size_t>(K * ldb) * ein;
    const size_t c_bytes = static_cast<size_t>(M * ldc) * eout;
    const size_t bias_bytes = bias ? static_cast<size_t>(N) * dtype_size(bias->dtype) : 0;
    auto up = [](size_t v) { return (v + 255) & ~size_t(255); };
    void *base = nullptr;
    ST_TRY(ws_acquire(d->stage, up(a_bytes) + up(b_bytes) + up(c_bytes) + up(bias_bytes), x.stream, &base));
    uint8_t *da = static_cast<uint8_t *>(base);
    uint8_t *db = da + up(a_bytes);
    uint8_t *dc = db + up(b_bytes);
    uint8_t *dbias = dc + up(c_bytes);
    size_t ev = 0;
    // the copies start after earlier work on the caller's stream (workspace reuse)
    ST_TRY(stream_after(d, ev, d->copy_in, x.stream));
    ST_TRY(stream_after(d, ev, d->copy_out, x.stream));
    if (bias) ST_CUDA_TRY(cudaMemcpyAsync(dbias, bias->data, bias_bytes, cudaMemcpyHostToDevice, d->copy_in));
    // ~16 MB blocks in whole 256-row / 256-column tiles (measured on B200 at
    // 8192^3: wider column blocks or taller row blocks were 2-4 % slower)
    const int64_t per = static_cast<int64_t>((size_t(16) << 20) / std::max<size_t>(1, static_cast<size_t>(K) * ein));
    const int64_t rows = std::max<int64_t>(256, (per / 256) * 256), cols = rows;
    const int64_t steps = std::max(cdiv(M, rows), cdiv(N, cols));
    auto view = [](const st_tensor &like, void *data, int64_t r, int64_t q, int64_t ld) {
        st_tensor v = like;
        v.data = data;
        v.rank = 2;
        v.shape[0] = r;
        v.shape[1] = q;
        v.strides[0] = ld;
        v.strides[1] = 1;
        return v;
    };
    auto gemm = [&](int64_t r0, int64_t r1, int64_t c0, int64_t c1) -> int {
        if (r1 <= r0 || c1 <= c0) return ST_OK;
        const st_tensor va = view(a, da + static_cast<size_t>(r0 * lda) * ein, r1 - r0, K, lda);
        const st_tensor vb = view(b, db + static_cast<size_t>(c0) * ein, K, c1 - c0, ldb);
        const st_tensor vc = view(c, dc + static_cast<size_t>(r0 * ldc + c0) * eout, r1 - r0, c1 - c0, ldc);
        st_tensor vbias;
        if (bias) {
            vbias = *bias;
            vbias.data = dbias + static_cast<size_t>(c0) * dtype_size(bias->dtype);
            vbias.shape[0] = c1 - c0;
            vbias.strides[0] = 1;
        }
        return matmul_device(x, va, vb, bias ? &vbias : nullptr, vc);
    };
    for (int64_t st = 0; st < steps; ++st) {
        const int64_t r0 = std::min(M, st * rows), r1 = std::min(M, (st + 1) * rows);
        const int64_t c0 = std::min(N, st * cols), c1 = std::min(N, (st + 1) * cols);
        ST_TRY(copy_block_in(d->copy_in, da, lda, a, r0, r1, 0, K));
        ST_TRY(copy_block_in(d->copy_in, db, ldb, b, 0, K, c0, c1));
        ST_TRY(stream_after(d, ev, x.stream, d->copy_in));
        ST_TRY(gemm(r0, r1, 0, c1));  // new rows x every column so far
        ST_TRY(gemm(0, r0, c0, c1));  // earlier rows x the new columns
        ST_TRY(stream_after(d, ev, d->copy_out, x.stream));
        ST_TRY(copy_block_out(d->copy_out, c, dc, ldc, r0, r1, 0, c1));
        ST_TRY(copy_block_out(d->copy_out, c, dc, ldc, 0, r0, c0, c1));
    }
    ST_TRY(stream_after(d, ev, x.stream, d->copy_out));
    ST_TRY(ws_release(d->stage, x.stream));
    return wait ? bounded_sync(d, x.stream, x.timeout_ms) : ST_OK;
}

// C = A + B on dense host arrays, in element chunks over the three streams.
int vector_add_host_pipelined(const ExecCtx &x, const st_tensor &a, const st_tensor &b, const st_tensor &c,
                              int64_t n, bool wait) {
    DeviceState *d = x.dev;
    ST_TRY(ensure_copy_streams(d));
    const size_t bytes = static_cast<size_t>(n) * 4;
    auto up = [](size_t v) { return (v + 255) & ~size_t(255); };
    void *base = nullptr;
    ST_TRY(ws_acquire(d->stage, 3 * up(bytes), x.stream, &base));
    float *da = static_cast<float *>(base);
    float *db = reinterpret_cast<float *>(static_cast<uint8_t *>(base) + up(bytes));
    float *dc = reinterpret_cast<float *>(static_cast<uint8_t *>(base) + 2 * up(bytes));
    const float *ha = static_cast<const float *>(a.data), *hb = static_cast<const float *>(b.data);
    float *hc = static_cast<float *>(c.data);
    size_t ev = 0;
    ST_TRY(stream_after(d, ev, d->copy_in, x.stream));
    ST_TRY(stream_after(d, ev, d->copy_out, x.stream));
    const int64_t chunk = int64_t(4) << 20;  // 16 MB of each array per chunk
    for (int64_t e0 = 0; e0 < n; e0 += chunk) {
        const int64_t len = std::min(chunk, n - e0);
        ST_CUDA_TRY(cudaMemcpyAsync(da + e0, ha + e0, len * 4, cudaMemcpyHostToDevice, d->copy_in));
        ST_CUDA_TRY(cudaMemcpyAsync(db + e0, hb + e0, len * 4, cudaMemcpyHostToDevice, d->copy_in));
        ST_TRY(stream_after(d, ev, x.stream, d->copy_in));
        ST_TRY(launch_vector_add_1d(da + e0, 1, db + e0, 1, dc + e0, 1, len, d->sm_count, x.stream));
        ST_TRY(stream_after(d, ev, d->copy_out, x.stream));
        ST_CUDA_TRY(cudaMemcpyAsync(hc + e0, dc + e0, len * 4, cudaMemcpyDeviceToHost, d->copy_out));
    }
    ST_TRY(stream_after(d, ev, x.stream, d->copy_out));
    ST_TRY(ws_release(d->stage, x.stream));
    return wait ? bounded_sync(d, x.stream, x.timeout_ms) : ST_OK;
}

// ------------------------------------------------------------ host-memory calls on one device
// Dense arrays of one layout: the add runs over one flat range.
bool vector_add_host_flat(const st_tensor &a, const st_tensor &b, const st_tensor &c) {
    bool flat = true;
    for (const st_tensor *t : {&a, &b, &c}) {
        if (t->rank == 1) flat &= t->shape[0] <= 1 || t->strides[0] == 1;
        else flat &= (t->shape[1] <= 1 || t->strides[1] == 1) && (t->shape[0] <= 1 || t->strides[0] == t->shape[1]);
    }
    return flat;
}

// C = A + B on host memory through the device of `x`; waits (bounded) when `wait`.
int vector_add_host_one(const ExecCtx &x, const st_tensor &a, const st_tensor &b, const st_tensor &c, bool wait) {
    int64_t n = 1;
    for (int i = 0; i < c.rank; ++i) n *= c.shape[i];
    if (vector_add_host_flat(a, b, c) && n > 0) return vector_add_host_pipelined(x, a, b, c, n, wait);
    void *base = nullptr;
    ST_TRY(ws_acquire(x.dev->stage, staged_bytes(a) + staged_bytes(b) + staged_bytes(c), x.stream, &base));
    uint8_t *cursor = static_cast<uint8_t *>(base);
    st_tensor da, db, dc;
    ST_TRY(stage_in(x, a, cursor, &da));
    ST_TRY(stage_in(x, b, cursor, &db));
    dc = c;
    dc.data = cursor;
    if (c.rank == 1) dc.strides[0] = 1;
    else {
        dc.strides[0] = c.shape[1];
        dc.strides[1] = 1;
    }
    const int64_t rows = c.rank == 2 ? c.shape[0] : 1;
    const int64_t cols = c.rank == 2 ? c.shape[1] : c.shape[0];
    ST_TRY(vector_add_views(x, da, db, dc, rows, cols));
    ST_TRY(stage_out(x, dc, c));
    ST_TRY(ws_release(x.dev->stage, x.stream));
    return wait ? bounded_sync(x.dev, x.stream, x.timeout_ms) : ST_OK;
}

// C = A @ B (+ bias) on host memory through the device of `x`; waits (bounded) when `wait`.
int matmul_host_one(const ExecCtx &x, const st_tensor &a, const st_tensor &b, const st_tensor *bias,
                    const st_tensor &c, bool wait) {
    // 16-bit operands with unit column strides: chunked and overlapped (the
    // fp32 path packs B once per call, so it stays unchunked)
    if (a.dtype != ST_F32 && a.shape[0] > 0 && b.shape[1] > 0 && a.shape[1] > 0 && host_rows_dense(a) &&
        host_rows_dense(b) && host_rows_dense(c))
        return matmul_host_pipelined(x, a, b, bias, c, wait);
    size_t need = staged_bytes(a) + staged_bytes(b) + staged_bytes(c) + (bias ? staged_bytes(*bias) : 0);
    void *base = nullptr;
    ST_TRY(ws_acquire(x.dev->stage, need, x.stream, &base));
    uint8_t *cursor = static_cast<uint8_t *>(base);
    st_tensor da, db, dbias, dc;
    ST_TRY(stage_in(x, a, cursor, &da));
    ST_TRY(stage_in(x, b, cursor, &db));
    if (bias) ST_TRY(stage_in(x, *bias, cursor, &dbias));
    dc = c;
    dc.data = cursor;
    dc.strides[0] = c.shape[1];
    dc.strides[1] = 1;
    ST_TRY(matmul_device(x, da, db, bias ? &dbias : nullptr, dc));
    ST_TRY(stage_out(x, dc, c));
    ST_TRY(ws_release(x.dev->stage, x.stream));
    return wait ? bounded_sync(x.dev, x.stream, x.timeout_ms) : ST_OK;
}

// ------------------------------------------------------------ single-box partitioner (one process)
// ST_EXEC_ALL_DEVICES: each device runs on its own stream of the context.
int check_all_devices(const st_exec *exec) {
    if (exec->stream != nullptr)
        return fail(ST_ERR_INVALID_ARGUMENT,
                    "ST_EXEC_ALL_DEVICES runs every device on the context's own stream: exec->stream must be NULL");
    if (exec->device >= 0)
        return fail(ST_ERR_INVALID_ARGUMENT, "ST_EXEC_ALL_DEVICES uses every device: exec->device must be -1");
    return ST_OK;
}

// Rows [r0, r1) of a host view (elements, for rank 1).
st_tensor host_rows(const st_tensor &t, int64_t r0, int64_t r1) {
    st_tensor v = t;
    v.data = static_cast<uint8_t *>(t.data) + static_cast<size_t>(r0 * t.strides[0]) * dtype_size(t.dtype);
    v.shape[0] = r1 - r0;
    return v;
}

// Elements [e0, e1) of a dense host array, as a rank-1 view.
st_tensor flat_range(const st_tensor &t, int64_t e0, int64_t e1) {
    st_tensor v = t;
    v.data = static_cast<uint8_t *>(t.data) + static_cast<size_t>(e0) * dtype_size(t.dtype);
    v.rank = 1;
    v.shape[0] = e1 - e0;
    v.strides[0] = 1;
    v.shape[1] = 0;
    v.strides[1] = 0;
    return v;
}

// Split [0, total) into one contiguous range per device of the context
// (boundaries on multiples of `align`, as st_shard_range), enqueue each
// range's work on its device, then wait (bounded) for every device that got
// work -- also after a failure, so that nothing is left in flight.
template <typename Enqueue>
int for_each_device_shard(st_ctx *ctx, const ExecCtx &x0, int64_t total, int64_t align, Enqueue enqueue) {
    const int g_count = static_cast<int>(ctx->devs.size());
    const int64_t units = cdiv(total, align);
    std::vector<ExecCtx> busy;
    int rc = ST_OK;
    for (int g = 0; g < g_count && rc == ST_OK; ++g) {
        const int64_t b = std::min(units * g / g_count * align, total);
        const int64_t e = std::min(units * (g + 1) / g_count * align, total);
        if (e <= b) continue;
        ExecCtx xg = x0;
        xg.dev = &ctx->devs[g];
        xg.stream = xg.dev->stream;
        DeviceGuard guard(xg.dev->ordinal);
        rc = enqueue(xg, b, e);
        busy.push_back(xg);
    }
    for (const ExecCtx &xg : busy) {
        DeviceGuard guard(xg.dev->ordinal);
        const int r = bounded_sync(xg.dev, xg.stream, xg.timeout_ms);
        if (rc == ST_OK) rc = r;
    }
    return rc;
}

// C = A + B on host memory over every device of the context: element
// ranges on 16-byte boundaries for dense arrays, rows otherwise.
int vector_add_host_split(st_ctx *ctx, const ExecCtx &x, const st_tensor &a, const st_tensor &b,
                          const st_tensor &c) {
    if (vector_add_host_flat(a, b, c)) {
        int64_t n = 1;
        for (int i = 0; i < c.rank; ++i) n *= c.shape[i];
        return for_each_device_shard(ctx, x, n, 4, [&](const ExecCtx &xg, int64_t e0, int64_t e1) {
            return vector_add_host_one(xg, flat_range(a, e0, e1), flat_range(b, e0, e1), flat_range(c, e0, e1),
                                       false);
        });
    }
    return for_each_device_shard(ctx, x, c.shape[0], 1, [&](const ExecCtx &xg, int64_t r0, int64_t r1) {
        return vector_add_host_one(xg, host_rows(a, r0, r1), host_rows(b, r0, r1), host_rows(c, r0, r1), false);
    });
}

// C = A @ B (+ bias) on host memory over every device of the context: 128-row
// blocks of A and C per device, all of B and the bias to each.
int matmul_host_split(st_ctx *ctx, const ExecCtx &x, const st_tensor &a, const st_tensor &b, const st_tensor *bias,
                      const st_tensor &c) {
    return for_each_device_shard(ctx, x, a.shape[0], 128, [&](const ExecCtx &xg, int64_t r0, int64_t r1) {
        return matmul_host_one(xg, host_rows(a, r0, r1), b, bias, host_rows(c, r0, r1), false);
    });
}

// ------------------------------------------------------------ entry registry
enum class Kind { VectorAdd1D, VectorAdd2D, Matmul, Fma1D, Fma2D, Cast1D, Cast2D };

struct Entry {
    const char *name;
    Kind kind;
    int in_dtype;
    bool bias;
    bool persistent;
    int n_constants;
    int defaults[3];
};

// cuda_tile symbols this backend serves (vecadd.py:39-48 exports
// "vector_add"; matmul.py:287-296 exports "matmul_fp32").
const Entry kEntries[] = {
    {"vector_add", Kind::VectorAdd1D, ST_F32, false, false, 1, {1024, 0, 0}},
    {"vector_add_2d", Kind::VectorAdd2D, ST_F32, false, false, 2, {64, 64, 0}},
    {"matmul_fp32", Kind::Matmul, ST_F32, false, false, 3, {32, 32, 32}},
    {"matmul_f16", Kind::Matmul, ST_F16, false, false, 3, {128, 256, 64}},
    {"matmul_bf16", Kind::Matmul, ST_BF16, false, false, 3, {128, 256, 64}},
    {"matmul_fp32_bias", Kind::Matmul, ST_F32, true, false, 3, {32, 32, 32}},
    {"matmul_f16_bias", Kind::Matmul, ST_F16, true, false, 3, {128, 256, 64}},
    {"matmul_bf16_bias", Kind::Matmul, ST_BF16, true, false, 3, {128, 256, 64}},
    {"persistent_matmul_fp32", Kind::Matmul, ST_F32, false, true, 3, {32, 32, 32}},
    {"persistent_matmul_f16", Kind::Matmul, ST_F16, false, true, 3, {128, 256, 64}},
    {"persistent_matmul_bf16", Kind::Matmul, ST_BF16, false, true, 3, {128, 256, 64}},
    // the other elementwise ops the lowering materialises (tileops.hpp:616-623, 257-258)
    {"vector_fma", Kind::Fma1D, ST_F32, false, false, 1, {1024, 0, 0}},
    {"vector_fma_2d", Kind::Fma2D, ST_F32, false, false, 2, {64, 64, 0}},
    {"cast", Kind::Cast1D, ST_F32, false, false, 1, {1024, 0, 0}},
    {"cast_2d", Kind::Cast2D, ST_F32, false, false, 2, {64, 64, 0}},
};

const Entry *find_entry(const char *name) {
    if (!name) return nullptr;
    for (const Entry &e : kEntries)
        if (std::strcmp(e.name, name) == 0) return &e;
    return nullptr;
}

// Rebuild tensor views from the flattened cutile_python_v1 bindings:
// rank 1 = (data, size, stride); rank 2 = (data, dim0, dim1, stride0, stride1).
int parse_params(const Entry &e, const st_param *params, int n_params, std::vector<st_tensor> *views,
                 std::vector<int> *buffer_index, int consts[3]) {
    std::vector<int> ranks;
    switch (e.kind) {
    case Kind::VectorAdd1D: ranks = {1, 1, 1}; break;
    case Kind::VectorAdd2D: ranks = {2, 2, 2}; break;
    case Kind::Fma1D: ranks = {1, 1, 1, 1}; break;   // A, B, D, C
    case Kind::Fma2D: ranks = {2, 2, 2, 2}; break;
    case Kind::Cast1D: ranks = {1, 1}; break;         // A, C
    case Kind::Cast2D: ranks = {2, 2}; break;
    case Kind::Matmul: ranks = e.bias ? std::vector<int>{2, 2, 2, 1} : std::vector<int>{2, 2, 2}; break;
    }
    const int n_arrays = static_cast<int>(ranks.size());
    int pos = 0;
    for (int i = 0; i < n_arrays; ++i) {
        const int r = ranks[i];
        const int need = 1 + 2 * r;
        if (pos + need > n_params)
            return fail(ST_ERR_INVALID_ARGUMENT, std::string(e.name) + " expects " +
                                                     std::to_string(n_arrays) + " array descriptors (got " +
                                                     std::to_string(n_params) + " params)");
        const st_param &buf = params[pos];
        if (buf.kind != ST_PARAM_BUFFER)
            return fail(ST_ERR_INVALID_ARGUMENT, "param " + std::to_string(pos) + " must be a buffer");
        for (int j = 1; j < need; ++j)
            if (params[pos + j].kind != ST_PARAM_I32)
                return fail(ST_ERR_INVALID_ARGUMENT, "param " + std::to_string(pos + j) + " must be an i32 scalar");
        st_tensor t{};
        t.data = buf.data;
        t.dtype = buf.dtype;
        t.rank = r;
        for (int d = 0; d < r; ++d) {
            t.shape[d] = params[pos + 1 + d].value;
            t.strides[d] = params[pos + 1 + r + d].value;
        }
        ST_TRY(check_view(&t, "array", r));
        if (buf.bytes) {
            const int64_t span = view_span(t);
            if (static_cast<uint64_t>(span) * dtype_size(t.dtype) > buf.bytes)
                return fail(ST_ERR_INVALID_ARGUMENT, "array " + std::to_string(i) + " descriptor reaches past its buffer");
        }
        views->push_back(t);
        buffer_index->push_back(pos);
        pos += need;
    }
    const int extra = n_params - pos;
    if (extra > e.n_constants)
        return fail(ST_ERR_INVALID_ARGUMENT, std::string(e.name) + " takes at most " + std::to_string(e.n_constants) +
                                                 " trailing constants");
    for (int i = 0; i < 3; ++i) consts[i] = e.defaults[i];
    for (int i = 0; i < extra; ++i) {
        if (params[pos + i].kind != ST_PARAM_I32 || params[pos + i].value <= 0 || params[pos + i].value > (1 << 20))
            return fail(ST_ERR_INVALID_ARGUMENT, "kernel constants must be positive i32 tile sizes");
        consts[i] = static_cast<int>(params[pos + i].value);
    }
    return ST_OK;
}

int run_entry(const ExecCtx &x, const Entry &e, const st_grid &grid, std::vector<st_tensor> &v, const int consts[3]) {
    const int64_t blocks = static_cast<int64_t>(grid.x) * grid.y * grid.z;
    if (e.kind == Kind::VectorAdd1D) {
        for (int i = 0; i < 3; ++i)
            if (v[i].dtype != ST_F32) return fail(ST_ERR_INVALID_ARGUMENT, "vector_add is f32-only");
        const int64_t tile = consts[0];
        int64_t n = blocks * tile;
        if (n > v[2].shape[0]) n = v[2].shape[0];
        if (n > v[0].shape[0] || n > v[1].shape[0])
            return fail(ST_ERR_INVALID_ARGUMENT, "vector_add: A and B must cover every stored element");
        return launch_vector_add_1d(static_cast<const float *>(v[0].data), v[0].strides[0],
                                    static_cast<const float *>(v[1].data), v[1].strides[0],
                                    static_cast<float *>(v[2].data), v[2].strides[0], n, x.dev->sm_count, x.stream);
    }
    if (e.kind == Kind::VectorAdd2D) {
        for (int i = 0; i < 3; ++i)
            if (v[i].dtype != ST_F32) return fail(ST_ERR_INVALID_ARGUMENT, "vector_add_2d is f32-only");
        int64_t rows = static_cast<int64_t>(grid.x) * consts[0], cols = static_cast<int64_t>(grid.y) * consts[1];
        if (grid.z == 0) rows = 0;
        rows = std::min(rows, v[2].shape[0]);
        cols = std::min(cols, v[2].shape[1]);
        for (int i = 0; i < 2; ++i)
            if (rows > v[i].shape[0] || cols > v[i].shape[1])
                return fail(ST_ERR_INVALID_ARGUMENT, "vector_add_2d: A and B must cover every stored element");
        return launch_vector_add_2d(static_cast<const float *>(v[0].data), v[0].strides,
                                    static_cast<const float *>(v[1].data), v[1].strides,
                                    static_cast<float *>(v[2].data), v[2].strides, rows, cols, x.dev->sm_count,
                                    x.stream);
    }
    if (e.kind == Kind::Fma1D || e.kind == Kind::Cast1D || e.kind == Kind::Fma2D || e.kind == Kind::Cast2D) {
        const bool fma = e.kind == Kind::Fma1D || e.kind == Kind::Fma2D;
        const size_t n_in = fma ? 3 : 1;
        st_tensor &out = v[n_in];
        if (fma)
            for (size_t i = 0; i <= n_in; ++i)
                if (v[i].dtype != ST_F32) return fail(ST_ERR_INVALID_ARGUMENT, std::string(e.name) + " is f32-only");
        int64_t rows, cols;
        if (out.rank == 1) {
            rows = 1;
            cols = std::min<int64_t>(blocks * consts[0], out.shape[0]);
            for (size_t i = 0; i < n_in; ++i)
                if (cols > v[i].shape[0])
                    return fail(ST_ERR_INVALID_ARGUMENT, std::string(e.name) + ": inputs must cover every stored element");
        } else {
            rows = std::min<int64_t>(static_cast<int64_t>(grid.x) * consts[0], out.shape[0]);
            cols = std::min<int64_t>(static_cast<int64_t>(grid.y) * consts[1], out.shape[1]);
            if (grid.z == 0) rows = 0;
            for (size_t i = 0; i < n_in; ++i)
                if (rows > v[i].shape[0] || cols > v[i].shape[1])
                    return fail(ST_ERR_INVALID_ARGUMENT, std::string(e.name) + ": inputs must cover every stored element");
        }
        int64_t s[4][2];
        for (size_t i = 0; i <= n_in; ++i) {
            s[i][0] = v[i].rank == 1 ? cols : v[i].strides[0];
            s[i][1] = v[i].rank == 1 ? v[i].strides[0] : v[i].strides[1];
        }
        if (fma)
            return launch_vector_fma(static_cast<const float *>(v[0].data), s[0], static_cast<const float *>(v[1].data),
                                     s[1], static_cast<const float *>(v[2].data), s[2], static_cast<float *>(v[3].data),
                                     s[3], rows, cols, x.dev->sm_count, x.stream);
        return launch_cast(v[0].data, v[0].dtype, s[0], v[1].data, v[1].dtype, s[1], rows, cols, x.dev->sm_count,
                           x.stream);
    }
    const st_tensor *bias = e.bias ? &v[3] : nullptr;
    ST_TRY(check_matmul(&v[0], &v[1], bias, &v[2]));
    if (v[0].dtype != e.in_dtype)
        return fail(ST_ERR_INVALID_ARGUMENT, std::string(e.name) + ": A/B dtype does not match the entry");
    const int64_t tiles = cdiv(v[0].shape[0], consts[0]) * cdiv(v[1].shape[1], consts[1]);
    if (blocks < 1) return fail(ST_ERR_INVALID_ARGUMENT, "empty grid");
    if (!e.persistent && blocks < tiles)
        return fail(ST_ERR_UNSUPPORTED, std::string(e.name) + ": the grid must cover all " + std::to_string(tiles) +
                                            " output tiles (the runtime picks its own tile shape)");
    return matmul_device(x, v[0], v[1], bias, v[2]);
}

// A host-buffer launch split over every device of the context
// (ST_EXEC_ALL_DEVICES): the region the tile grid covers, by the same rules
// as run_entry, goes to the split host calls, which write C in place.
int run_entry_split(st_ctx *ctx, const ExecCtx &x, const Entry &e, const st_grid &grid, std::vector<st_tensor> &v,
                    const int consts[3]) {
    const int64_t blocks = static_cast<int64_t>(grid.x) * grid.y * grid.z;
    if (e.kind == Kind::VectorAdd1D) {
        for (int i = 0; i < 3; ++i)
            if (v[i].dtype != ST_F32) return fail(ST_ERR_INVALID_ARGUMENT, "vector_add is f32-only");
        const int64_t n = std::min<int64_t>(blocks * consts[0], v[2].shape[0]);
        if (n > v[0].shape[0] || n > v[1].shape[0])
            return fail(ST_ERR_INVALID_ARGUMENT, "vector_add: A and B must cover every stored element");
        for (int i = 0; i < 3; ++i) v[i].shape[0] = n;
        return vector_add_host_split(ctx, x, v[0], v[1], v[2]);
    }
    if (e.kind == Kind::VectorAdd2D) {
        for (int i = 0; i < 3; ++i)
            if (v[i].dtype != ST_F32) return fail(ST_ERR_INVALID_ARGUMENT, "vector_add_2d is f32-only");
        int64_t rows = grid.z == 0 ? 0 : std::min<int64_t>(static_cast<int64_t>(grid.x) * consts[0], v[2].shape[0]);
        const int64_t cols = std::min<int64_t>(static_cast<int64_t>(grid.y) * consts[1], v[2].shape[1]);
        for (int i = 0; i < 2; ++i)
            if (rows > v[i].shape[0] || cols > v[i].shape[1])
                return fail(ST_ERR_INVALID_ARGUMENT, "vector_add_2d: A and B must cover every stored element");
        for (int i = 0; i < 3; ++i) {
            v[i].shape[0] = rows;
            v[i].shape[1] = cols;
        }
        return vector_add_host_split(ctx, x, v[0], v[1], v[2]);
    }
    if (e.kind != Kind::Matmul)
        return fail(ST_ERR_UNSUPPORTED, std::string(e.name) +
                                            ": ST_EXEC_ALL_DEVICES splits vector_add, vector_add_2d and matmul entries");
    const st_tensor *bias = e.bias ? &v[3] : nullptr;
    ST_TRY(check_matmul(&v[0], &v[1], bias, &v[2]));
    if (v[0].dtype != e.in_dtype)
        return fail(ST_ERR_INVALID_ARGUMENT, std::string(e.name) + ": A/B dtype does not match the entry");
    const int64_t tiles = cdiv(v[0].shape[0], consts[0]) * cdiv(v[1].shape[1], consts[1]);
    if (blocks < 1) return fail(ST_ERR_INVALID_ARGUMENT, "empty grid");
    if (!e.persistent && blocks < tiles)
        return fail(ST_ERR_UNSUPPORTED, std::string(e.name) + ": the grid must cover all " + std::to_string(tiles) +
                                            " output tiles (the runtime picks its own tile shape)");
    return matmul_host_split(ctx, x, v[0], v[1], bias, v[2]);
}

}  // namespace
}  // namespace st

// ============================================================ C ABI
using namespace st;

extern "C" {

const char *st_version(void) { return "sptiles_b200 0.1.0 (sm_100a)"; }

const char *st_last_error(void) { return g_last_error.c_str(); }

int st_device_count(int32_t *count) {
    if (!count) return fail(ST_ERR_INVALID_ARGUMENT, "count is null");
    int n = 0;
    const cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess) {
        cudaGetLastError();
        *count = 0;
        g_last_error = std::string("cudaGetDeviceCount: ") + cudaGetErrorString(e);
        return ST_OK;
    }
    *count = n;
    return ST_OK;
}

int st_kernel_launches(uint64_t *count) {
    if (!count) return fail(ST_ERR_INVALID_ARGUMENT, "count is null");
    *count = g_launches.load(std::memory_order_relaxed);
    return ST_OK;
}

int st_init(const int32_t *devices, int32_t n_devices, st_ctx **out) {
    if (!out) return fail(ST_ERR_INVALID_ARGUMENT, "out is null");
    *out = nullptr;
    if (n_devices < 0 || (n_devices > 0 && !devices))
        return fail(ST_ERR_INVALID_ARGUMENT, "bad device list");
    int count = 0;
    cudaError_t e = cudaGetDeviceCount(&count);
    if (e != cudaSuccess || count == 0) {
        cudaGetLastError();
        return fail(ST_ERR_NO_DEVICE, "no CUDA device is visible");
    }
    std::vector<int> ords;
    if (n_devices == 0) ords.push_back(0);
    for (int i = 0; i < n_devices; ++i) ords.push_back(devices[i]);
    auto *ctx = new st_ctx();
    for (int ord : ords) {
        if (ord < 0 || ord >= count) {
            st_shutdown(ctx);
            return fail(ST_ERR_INVALID_ARGUMENT, "device ordinal " + std::to_string(ord) + " out of range");
        }
        DeviceGuard guard(ord);
        cudaDeviceProp prop;
        e = cudaGetDeviceProperties(&prop, ord);
        if (e != cudaSuccess) {
            st_shutdown(ctx);
            return cuda_fail(e, "cudaGetDeviceProperties");
        }
        if (prop.major != 10) {
            st_shutdown(ctx);
            return fail(ST_ERR_NO_DEVICE, std::string("device ") + std::to_string(ord) + " (" + prop.name +
                                              ") is not sm_100; these kernels are built for sm_100a only");
        }
        DeviceState d;
        d.ordinal = ord;
        d.sm_count = prop.multiProcessorCount;
        if ((e = cudaStreamCreateWithFlags(&d.stream, cudaStreamNonBlocking)) != cudaSuccess ||
            (e = cudaMalloc(&d.dev_err, sizeof(int))) != cudaSuccess ||
            (e = cudaMemset(d.dev_err, 0, sizeof(int))) != cudaSuccess) {
            ctx->devs.push_back(d);
            st_shutdown(ctx);
            return cuda_fail(e, "device set-up");
        }
        ctx->devs.push_back(d);
    }
    // peer access between the context's devices (NVLink), for peer copies and
    // for GEMM epilogues that store into another device's copy of C
    for (int i : ords)
        for (int j : ords) {
            int can = 0;
            if (i == j || cudaDeviceCanAccessPeer(&can, i, j) != cudaSuccess || !can) {
                cudaGetLastError();
                continue;
            }
            DeviceGuard guard(i);
            if (cudaDeviceEnablePeerAccess(j, 0) != cudaSuccess) cudaGetLastError();  // already enabled is fine
        }
    *out = ctx;
    return ST_OK;
}

int st_shutdown(st_ctx *ctx) {
    if (!ctx) return ST_OK;
    for (auto &d : ctx->devs) {
        DeviceGuard guard(d.ordinal);
        if (d.stream) cudaStreamSynchronize(d.stream);
        if (d.copy_in) cudaStreamSynchronize(d.copy_in);
        if (d.copy_out) cudaStreamSynchronize(d.copy_out);
        ws_free(d.scratch);
        ws_free(d.stage);
        ws_free(d.sk);
        for (cudaEvent_t e : d.events) cudaEventDestroy(e);
        if (d.copy_in) cudaStreamDestroy(d.copy_in);
        if (d.copy_out) cudaStreamDestroy(d.copy_out);
        if (d.dev_err) cudaFree(d.dev_err);
        if (d.stream) cudaStreamDestroy(d.stream);
    }
    delete ctx;
    return ST_OK;
}

int st_sync(st_ctx *ctx, int32_t device, uint32_t timeout_ms) {
    DeviceState *d;
    ST_TRY(get_dev(ctx, device, &d));
    DeviceGuard guard(d->ordinal);
    return bounded_sync(d, d->stream, timeout_ms);
}

int st_stream(st_ctx *ctx, int32_t device, void **stream) {
    DeviceState *d;
    ST_TRY(get_dev(ctx, device, &d));
    if (!stream) return fail(ST_ERR_INVALID_ARGUMENT, "stream is null");
    *stream = d->stream;
    return ST_OK;
}

int st_alloc(st_ctx *ctx, int32_t device, uint64_t bytes, void **out) {
    DeviceState *d;
    ST_TRY(get_dev(ctx, device, &d));
    if (!out) return fail(ST_ERR_INVALID_ARGUMENT, "out is null");
    DeviceGuard guard(d->ordinal);
    *out = nullptr;
    if (bytes == 0) return ST_OK;
    ST_CUDA_TRY(cudaMalloc(out, bytes));
    return ST_OK;
}

int st_free(st_ctx *ctx, int32_t device, void *ptr) {
    DeviceState *d;
    ST_TRY(get_dev(ctx, device, &d));
    DeviceGuard guard(d->ordinal);
    if (ptr) ST_CUDA_TRY(cudaFree(ptr));
    return ST_OK;
}

int st_upload(st_ctx *ctx, int32_t device, void *dst, const void *src, uint64_t bytes) {
    DeviceState *d;
    ST_TRY(get_dev(ctx, device, &d));
    if (bytes && (!dst || !src)) return fail(ST_ERR_INVALID_ARGUMENT, "null pointer");
    DeviceGuard guard(d->ordinal);
    if (bytes) ST_CUDA_TRY(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, d->stream));
    return bounded_sync(d, d->stream, 0);
}

int st_download(st_ctx *ctx, int32_t device, void *dst, const void *src, uint64_t bytes) {
    DeviceState *d;
    ST_TRY(get_dev(ctx, device, &d));
    if (bytes && (!dst || !src)) return fail(ST_ERR_INVALID_ARGUMENT, "null pointer");
    DeviceGuard guard(d->ordinal);
    if (bytes) ST_CUDA_TRY(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, d->stream));
    return bounded_sync(d, d->stream, 0);
}

int st_grid_from_dispatch(const char *entry_name, const uint32_t dispatch[3], int64_t tile_elems, st_grid *out) {
    const Entry *e = find_entry(entry_name);
    if (!e) return fail(ST_ERR_UNKNOWN_ENTRY, std::string("unknown entry '") + (entry_name ? entry_name : "") + "'");
    if (!dispatch || !out || tile_elems <= 0) return fail(ST_ERR_INVALID_ARGUMENT, "bad dispatch conversion arguments");
    if (e->kind == Kind::VectorAdd2D)
        return fail(ST_ERR_UNSUPPORTED, "a 2D tile grid cannot be recovered from a linear dispatch");
    const int64_t inv = static_cast<int64_t>(dispatch[0]) * dispatch[1] * dispatch[2] * 1024;
    const int64_t tiles = cdiv(inv, tile_elems);
    if (tiles > UINT32_MAX) return fail(ST_ERR_INVALID_ARGUMENT, "dispatch too large");
    *out = st_grid{static_cast<uint32_t>(tiles), 1, 1};
    return ST_OK;
}

int st_launch(st_ctx *ctx, const char *entry_name, const st_grid *grid, const st_param *params, int32_t n_params,
              const st_exec *exec) {
    const Entry *e = find_entry(entry_name);
    if (!e) return fail(ST_ERR_UNKNOWN_ENTRY, std::string("Entry point ") + (entry_name ? entry_name : "(null)") +
                                                  " was not found in the kernel registry.");
    if (!grid || (!params && n_params > 0) || n_params < 0)
        return fail(ST_ERR_INVALID_ARGUMENT, "grid and params are required");
    const bool split = exec && (exec->flags & ST_EXEC_ALL_DEVICES);
    if (split && !(exec->flags & ST_EXEC_HOST_BUFFERS))
        return fail(ST_ERR_INVALID_ARGUMENT, kAllDevicesScope);
    ExecCtx x;
    ST_TRY(resolve_exec(ctx, exec, &x, true));
    std::vector<st_tensor> views;
    std::vector<int> bufpos;
    int consts[3];
    ST_TRY(parse_params(*e, params, n_params, &views, &bufpos, consts));
    if (split) {  // host buffers split over every device: C is written in place
        ST_TRY(check_all_devices(exec));
        return run_entry_split(ctx, x, *e, *grid, views, consts);
    }
    DeviceGuard guard(x.dev->ordinal);
    if (!(x.flags & ST_EXEC_HOST_BUFFERS)) {
        ST_TRY(run_entry(x, *e, *grid, views, consts));
        return finish(x);
    }
    // host buffers: stage every array, run, copy the requested outputs back
    // (the run_spirv_kernel contract, spirv_runtime.py:153-174)
    for (size_t i = 0; i < views.size(); ++i)
        if (params[bufpos[i]].bytes == 0)
            return fail(ST_ERR_INVALID_ARGUMENT, "host-buffer launches need the size of every buffer");
    size_t total = 0;
    for (size_t i = 0; i < views.size(); ++i) total += (params[bufpos[i]].bytes + 255) & ~uint64_t(255);
    void *base = nullptr;
    ST_TRY(ws_acquire(x.dev->stage, total, x.stream, &base));
    uint8_t *cursor = static_cast<uint8_t *>(base);
    std::vector<st_tensor> dev_views = views;
    std::vector<uint8_t *> dev_bufs;
    for (size_t i = 0; i < views.size(); ++i) {
        const st_param &p = params[bufpos[i]];
        ST_CUDA_TRY(cudaMemcpyAsync(cursor, p.data, p.bytes, cudaMemcpyHostToDevice, x.stream));
        dev_views[i].data = cursor;
        dev_bufs.push_back(cursor);
        cursor += (p.bytes + 255) & ~uint64_t(255);
    }
    ST_TRY(run_entry(x, *e, *grid, dev_views, consts));
    // default output: C, the third array of the add/matmul signatures, the last one otherwise
    const int32_t default_out[1] = {(e->kind == Kind::VectorAdd1D || e->kind == Kind::VectorAdd2D ||
                                     e->kind == Kind::Matmul)
                                        ? bufpos[2]
                                        : bufpos.back()};
    const int32_t *outs = exec && exec->n_outputs > 0 ? exec->output_indices : default_out;
    const int n_outs = exec && exec->n_outputs > 0 ? exec->n_outputs : 1;
    for (int i = 0; i < n_outs; ++i) {
        const int idx = outs[i];
        size_t which = views.size();
        for (size_t j = 0; j < bufpos.size(); ++j)
            if (bufpos[j] == idx) which = j;
        if (which == views.size()) return fail(ST_ERR_INVALID_ARGUMENT, "output index must name a buffer param");
        ST_CUDA_TRY(cudaMemcpyAsync(params[idx].data, dev_bufs[which], params[idx].bytes, cudaMemcpyDeviceToHost,
                                    x.stream));
    }
    ST_TRY(ws_release(x.dev->stage, x.stream));
    return bounded_sync(x.dev, x.stream, x.timeout_ms);
}

int st_vector_add(st_ctx *ctx, const st_tensor *a, const st_tensor *b, const st_tensor *c, const st_exec *exec) {
    ExecCtx x;
    ST_TRY(resolve_exec(ctx, exec, &x));
    ST_TRY(check_vector_add(a, b, c));
    DeviceGuard guard(x.dev->ordinal);
    const int64_t rows = c->rank == 2 ? c->shape[0] : 1;
    const int64_t cols = c->rank == 2 ? c->shape[1] : c->shape[0];
    ST_TRY(vector_add_views(x, *a, *b, *c, rows, cols));
    return finish(x);
}

int st_matmul(st_ctx *ctx, const st_tensor *a, const st_tensor *b, const st_tensor *bias, const st_tensor *c,
              const st_exec *exec) {
    ExecCtx x;
    ST_TRY(resolve_exec(ctx, exec, &x));
    ST_TRY(check_matmul(a, b, bias, c));
    DeviceGuard guard(x.dev->ordinal);
    ST_TRY(matmul_device(x, *a, *b, bias, *c));
    return finish(x);
}

int st_vector_fma(st_ctx *ctx, const st_tensor *a, const st_tensor *b, const st_tensor *d, const st_tensor *c,
                  const st_exec *exec) {
    ExecCtx x;
    ST_TRY(resolve_exec(ctx, exec, &x));
    ST_TRY(check_vector_add(a, b, c));
    ST_TRY(check_vector_add(a, d, c));
    DeviceGuard guard(x.dev->ordinal);
    const int64_t rows = c->rank == 2 ? c->shape[0] : 1;
    const int64_t cols = c->rank == 2 ? c->shape[1] : c->shape[0];
    int64_t s[4][2];
    const st_tensor *t[4] = {a, b, d, c};
    for (int i = 0; i < 4; ++i) {
        s[i][0] = t[i]->rank == 1 ? cols : t[i]->strides[0];
        s[i][1] = t[i]->rank == 1 ? t[i]->strides[0] : t[i]->strides[1];
    }
    ST_TRY(launch_vector_fma(static_cast<const float *>(a->data), s[0], static_cast<const float *>(b->data), s[1],
                             static_cast<const float *>(d->data), s[2], static_cast<float *>(c->data), s[3], rows, cols,
                             x.dev->sm_count, x.stream));
    return finish(x);
}

int st_check_device_wait(st_ctx *ctx, int32_t kind, uint32_t limit_us, const st_exec *exec) {
    if (kind != 0 && kind != 1)
        return fail(ST_ERR_INVALID_ARGUMENT, "st_check_device_wait: kind must be 0 (mbarrier) or 1 (flag)");
    if (limit_us == 0 || limit_us > 10u * 1000 * 1000)
        return fail(ST_ERR_INVALID_ARGUMENT, "st_check_device_wait: limit_us must be in [1, 10^7]");
    ExecCtx x;
    ST_TRY(resolve_exec(ctx, exec, &x));
    DeviceGuard guard(x.dev->ordinal);
    ST_TRY(launch_wait_check(kind, static_cast<uint64_t>(limit_us) * 1000, x.dev->dev_err, x.stream));
    return finish(x);
}

int st_cast(st_ctx *ctx, const st_tensor *a, const st_tensor *c, const st_exec *exec) {
    ExecCtx x;
    ST_TRY(resolve_exec(ctx, exec, &x));
    if (!a || !c) return fail(ST_ERR_INVALID_ARGUMENT, "cast: null tensor");
    if (c->rank != 1 && c->rank != 2) return fail(ST_ERR_INVALID_ARGUMENT, "cast: tensors must be rank 1 or 2");
    ST_TRY(check_view(a, "A", c->rank));
    ST_TRY(check_view(c, "C", c->rank));
    for (const st_tensor *t : {a, c})
        if (t->dtype != ST_F32 && t->dtype != ST_F16 && t->dtype != ST_BF16)
            return fail(ST_ERR_INVALID_ARGUMENT, "cast: tensors must be ST_F32, ST_F16 or ST_BF16");
    for (int i = 0; i < c->rank; ++i)
        if (a->shape[i] != c->shape[i]) return fail(ST_ERR_INVALID_ARGUMENT, "cast: A and C must have the same shape");
    DeviceGuard guard(x.dev->ordinal);
    const int64_t rows = c->rank == 2 ? c->shape[0] : 1;
    const int64_t cols = c->rank == 2 ? c->shape[1] : c->shape[0];
    const int64_t sa[2] = {a->rank == 1 ? cols : a->strides[0], a->rank == 1 ? a->strides[0] : a->strides[1]};
    const int64_t sc[2] = {c->rank == 1 ? cols : c->strides[0], c->rank == 1 ? c->strides[0] : c->strides[1]};
    ST_TRY(launch_cast(a->data, a->dtype, sa, c->data, c->dtype, sc, rows, cols, x.dev->sm_count, x.stream));
    return finish(x);
}

int st_vector_add_host(st_ctx *ctx, const st_tensor *a, const st_tensor *b, const st_tensor *c, const st_exec *exec) {
    ExecCtx x;
    ST_TRY(resolve_exec(ctx, exec, &x, true));
    ST_TRY(check_vector_add(a, b, c));
    if (x.flags & ST_EXEC_ALL_DEVICES) {
        ST_TRY(check_all_devices(exec));
        return vector_add_host_split(ctx, x, *a, *b, *c);
    }
    DeviceGuard guard(x.dev->ordinal);
    return vector_add_host_one(x, *a, *b, *c, true);
}

int st_matmul_host(st_ctx *ctx, const st_tensor *a, const st_tensor *b, const st_tensor *bias, const st_tensor *c,
                   const st_exec *exec) {
    ExecCtx x;
    ST_TRY(resolve_exec(ctx, exec, &x, true));
    ST_TRY(check_matmul(a, b, bias, c));
    if (x.flags & ST_EXEC_ALL_DEVICES) {
        ST_TRY(check_all_devices(exec));
        return matmul_host_split(ctx, x, *a, *b, bias, *c);
    }
    DeviceGuard guard(x.dev->ordinal);
    return matmul_host_one(x, *a, *b, bias, *c, true);
}

int st_ipc_handle(st_ctx *ctx, int32_t device, void *ptr, uint8_t handle[64]) {
    DeviceState *d;
    ST_TRY(get_dev(ctx, device, &d));
    if (!ptr || !handle) return fail(ST_ERR_INVALID_ARGUMENT, "st_ipc_handle: null pointer");
    static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
    DeviceGuard guard(d->ordinal);
    cudaIpcMemHandle_t h;
    ST_CUDA_TRY(cudaIpcGetMemHandle(&h, ptr));
    std::memcpy(handle, &h, 64);
    return ST_OK;
}

int st_ipc_open(st_ctx *ctx, int32_t device, const uint8_t handle[64], void **out) {
    DeviceState *d;
    ST_TRY(get_dev(ctx, device, &d));
    if (!handle || !out) return fail(ST_ERR_INVALID_ARGUMENT, "st_ipc_open: null pointer");
    DeviceGuard guard(d->ordinal);
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, 64);
    ST_CUDA_TRY(cudaIpcOpenMemHandle(out, h, cudaIpcMemLazyEnablePeerAccess));
    return ST_OK;
}

int st_ipc_close(st_ctx *ctx, int32_t device, void *ptr) {
    DeviceState *d;
    ST_TRY(get_dev(ctx, device, &d));
    DeviceGuard guard(d->ordinal);
    if (ptr) ST_CUDA_TRY(cudaIpcCloseMemHandle(ptr));
    return ST_OK;
}

int st_matmul_allgather(st_ctx *ctx, const st_tensor *a, const st_tensor *b, const st_tensor *bias,
                        const st_tensor *c_full, void *const *peer_c_full, int32_t n_peers, int64_t row_offset,
                        const st_exec *exec) {
    ExecCtx x;
    ST_TRY(resolve_exec(ctx, exec, &x));
    if (!a || !c_full) return fail(ST_ERR_INVALID_ARGUMENT, "st_matmul_allgather: null tensor");
    ST_TRY(check_view(c_full, "C", 2));
    if (n_peers < 0 || n_peers > kMaxPeers || (n_peers > 0 && !peer_c_full))
        return fail(ST_ERR_INVALID_ARGUMENT, "st_matmul_allgather: between 0 and 7 peer copies of C");
    if (row_offset < 0 || a->rank != 2 || row_offset + a->shape[0] > c_full->shape[0])
        return fail(ST_ERR_INVALID_ARGUMENT, "st_matmul_allgather: A's rows must fall inside C at row_offset");
    // this rank's rows of C, and the same rows in each peer's copy
    const size_t es = dtype_size(c_full->dtype);
    const size_t byte_off = static_cast<size_t>(row_offset) * static_cast<size_t>(c_full->strides[0]) * es;
    st_tensor c_rows = *c_full;
    c_rows.shape[0] = a->shape[0];
    c_rows.data = static_cast<uint8_t *>(c_full->data) + byte_off;
    ST_TRY(check_matmul(a, b, bias, &c_rows));
    PeerOutputs peers;
    peers.n = n_peers;
    for (int i = 0; i < n_peers; ++i) {
        if (!peer_c_full[i]) return fail(ST_ERR_INVALID_ARGUMENT, "st_matmul_allgather: null peer pointer");
        peers.base[i] = static_cast<uint8_t *>(peer_c_full[i]) + byte_off;
    }
    DeviceGuard guard(x.dev->ordinal);
    ST_TRY(matmul_device(x, *a, *b, bias, c_rows, &peers));
    return finish(x);
}

int st_shard_range(int64_t total, int32_t count, int32_t rank, int64_t align, int64_t *begin, int64_t *end) {
    if (total < 0 || count < 1 || rank < 0 || rank >= count || align < 1 || !begin || !end)
        return fail(ST_ERR_INVALID_ARGUMENT, "st_shard_range: need total >= 0, 0 <= rank < count, align >= 1");
    const int64_t units = cdiv(total, align);
    const int64_t b = units * rank / count, e = units * (rank + 1) / count;
    *begin = std::min(b * align, total);
    *end = std::min(e * align, total);
    return ST_OK;
}

}  // extern "C"
