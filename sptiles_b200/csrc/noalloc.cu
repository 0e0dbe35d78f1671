// noalloc.cu -- the fp32 (3xTF32) matmul for callers that cannot allocate
// device memory.
//
// Who needs it: a process whose memory pool already owns the GPU's memory
// (a cudaMalloc issued by a library would then fail or fragment that pool),
// and callers on a latency-critical path that cannot pay for allocation --
// cudaFree, for one, waits for the whole device to go idle.  The regular
// st_matmul keeps its packed operands in a workspace it grows with
// cudaMalloc; this entry point instead packs them into one fixed array that
// is part of the library image, so a call allocates nothing.
//
// The array is a file-scope __device__ object: once this file's module is
// on a GPU, that GPU holds its 32 MiB until the process exits.  CUDA loads a
// library's modules lazily by default (on first use), so the array, like
// the code of the kernels this entry point launches, takes its device memory
// during the first call on each device: that set-up call, made with the
// device current, resolves the array's device address with
// cudaGetSymbolAddress (host code cannot use the symbol `g_static_scratch`
// as an address: on the host it names a host-side stand-in) and loads the
// packing and GEMM kernels up front.  Later calls allocate nothing.  So a
// caller whose memory pool takes the GPU's memory makes one call per device
// before that (a 1 x 1 x 1 product will do), and, like every set-up, before
// any stream capture.
//
// All calls share the one array, which keeps whatever the last call wrote.
// The packing kernels overwrite every byte the GEMM then reads (padding
// included).  Two calls whose work overlaps on the GPU (different streams,
// or different host threads) race on the array: serialise them.
//
// A kernel that gives up a bounded wait records a code in this file's abort
// word and leaves C incomplete.  The word keeps that code until a call made
// with ST_EXEC_SYNC reads it: that call returns ST_ERR_DEVICE_ABORT (for its
// own work or for an earlier asynchronous call's) and clears the word.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <chrono>
#include <cstdint>
#include <mutex>
#include <string>
#include <thread>

#include "common.h"

namespace st {
namespace {

constexpr size_t kStaticScratchBytes = size_t(ST_STATIC_SCRATCH_BYTES);
constexpr uint64_t kWaitLimitNs = 4ull * 1000 * 1000 * 1000;

static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];
static __device__ int g_static_abort;

struct StaticDevice {
    bool ready = false;
    unsigned char *scratch = nullptr;  // device address of g_static_scratch
    int *abort_word = nullptr;         // device address of g_static_abort
    int sm_count = 0;
};

constexpr int kMaxDevices = 64;
StaticDevice g_devices[kMaxDevices];
std::mutex g_setup_mutex;

// C = bias (or 0) when K == 0.
__global__ void static_fill_kernel(void *c, int64_t ldc, int c_dtype, const void *bias, int bias_dtype, int64_t m,
                                   int64_t n) {
    const int64_t total = m * n;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t r = i / n, q = i - r * n;
        const float v = bias ? static_cast<const float *>(bias)[q] : 0.0f;
        if (c_dtype == ST_F32) static_cast<float *>(c)[r * ldc + q] = v;
        else if (c_dtype == ST_F16) static_cast<__half *>(c)[r * ldc + q] = __float2half_rn(v);
        else static_cast<__nv_bfloat16 *>(c)[r * ldc + q] = __float2bfloat16_rn(v);
    }
}

// Once per device, with that device current: resolve the symbols' device addresses.
int static_device(int dev, StaticDevice **out) {
    if (dev < 0 || dev >= kMaxDevices) return fail(ST_ERR_INVALID_ARGUMENT, "device ordinal out of range");
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    StaticDevice &d = g_devices[dev];
    if (!d.ready) {
        int major = 0, sms = 0;
        ST_CUDA_TRY(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev));
        if (major != 10) return fail(ST_ERR_NO_DEVICE, "the static-scratch matmul runs on sm_100 devices only");
        ST_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
        void *scratch = nullptr, *word = nullptr;
        ST_CUDA_TRY(cudaGetSymbolAddress(&scratch, g_static_scratch));
        ST_CUDA_TRY(cudaGetSymbolAddress(&word, g_static_abort));
        // the kernels later calls launch: their code is placed now, not on first launch
        cudaFuncAttributes attr;
        ST_CUDA_TRY(cudaFuncGetAttributes(&attr, static_fill_kernel));
        ST_TRY(preload_pack_tf32_kernels());
        ST_TRY(preload_gemm_tf32_kernels());
        d.scratch = static_cast<unsigned char *>(scratch);
        d.abort_word = static_cast<int *>(word);
        d.sm_count = sms;
        d.ready = true;
    }
    *out = &d;
    return ST_OK;
}

int check_operand(const st_tensor *t, const char *name, int rank) {
    if (!t) return fail(ST_ERR_INVALID_ARGUMENT, std::string(name) + " is null");
    if (t->rank != rank) return fail(ST_ERR_INVALID_ARGUMENT, std::string(name) + " has the wrong rank");
    for (int i = 0; i < rank; ++i)
        if (t->shape[i] < 0 || t->strides[i] < 0)
            return fail(ST_ERR_INVALID_ARGUMENT, std::string(name) + " has a negative extent or stride");
    bool empty = false;
    for (int i = 0; i < rank; ++i) empty |= t->shape[i] == 0;
    if (!empty && !t->data) return fail(ST_ERR_INVALID_ARGUMENT, std::string(name) + " has a null data pointer");
    return ST_OK;
}

// Bounded wait on the stream without creating any CUDA object.
int wait_stream(cudaStream_t stream, uint32_t timeout_ms) {
    const auto deadline = std::chrono::steady_clock::now() + std::chrono::milliseconds(timeout_ms ? timeout_ms : 60000);
    cudaError_t e;
    while ((e = cudaStreamQuery(stream)) == cudaErrorNotReady) {
        if (std::chrono::steady_clock::now() > deadline)
            return fail(ST_ERR_TIMEOUT, "the static-scratch matmul did not finish in time");
        std::this_thread::sleep_for(std::chrono::microseconds(20));
    }
    if (e != cudaSuccess) return cuda_fail(e, "static-scratch matmul execution");
    return ST_OK;
}

class CurrentDevice {
  public:
    explicit CurrentDevice(int dev) {
        cudaGetDevice(&prev_);
        cudaSetDevice(dev);
    }
    ~CurrentDevice() { cudaSetDevice(prev_); }

  private:
    int prev_ = 0;
};

}  // namespace
}  // namespace st

using namespace st;

extern "C" int st_matmul_static_scratch(const st_tensor *a, const st_tensor *b, const st_tensor *bias,
                                        const st_tensor *c, const st_exec *exec) {
    ST_TRY(check_operand(a, "A", 2));
    ST_TRY(check_operand(b, "B", 2));
    ST_TRY(check_operand(c, "C", 2));
    if (a->dtype != ST_F32 || b->dtype != ST_F32)
        return fail(ST_ERR_UNSUPPORTED, "st_matmul_static_scratch takes f32 A and B (the 3xTF32 path)");
    if (c->dtype != ST_F32 && c->dtype != ST_F16 && c->dtype != ST_BF16)
        return fail(ST_ERR_INVALID_ARGUMENT, "C must be ST_F32, ST_F16 or ST_BF16");
    const int64_t M = a->shape[0], K = a->shape[1], N = b->shape[1];
    if (b->shape[0] != K)
        return fail(ST_ERR_INVALID_ARGUMENT, "Incompatible matrices: K dimension of A (" + std::to_string(K) +
                                                 ") must match K dimension of B (" + std::to_string(b->shape[0]) +
                                                 ")");
    if (c->shape[0] != M || c->shape[1] != N) return fail(ST_ERR_INVALID_ARGUMENT, "C must be [M, N]");
    if (M > 0 && N > 1 && c->strides[1] != 1) return fail(ST_ERR_UNSUPPORTED, "C must have unit column stride");
    if (M > INT32_MAX || N > INT32_MAX || K > INT32_MAX)
        return fail(ST_ERR_UNSUPPORTED, "matmul extents must fit in int32");
    if (bias) {
        ST_TRY(check_operand(bias, "bias", 1));
        if (bias->shape[0] != N || bias->dtype != ST_F32 || (N > 1 && bias->strides[0] != 1))
            return fail(ST_ERR_INVALID_ARGUMENT, "bias must be a contiguous f32 vector of N elements");
    }
    // (M + N) * 3 * kp * 4 bytes must fit; compared by division, so that no
    // product of caller-supplied extents can wrap around
    const int64_t kp = tf32_packed_k(K);
    const uint64_t rows = static_cast<uint64_t>(M) + static_cast<uint64_t>(N);
    const uint64_t row_bytes = 3 * static_cast<uint64_t>(kp) * sizeof(float);
    if (row_bytes != 0 && rows > kStaticScratchBytes / row_bytes) {
        const std::string need = rows <= UINT64_MAX / row_bytes ? std::to_string(rows * row_bytes) + " bytes"
                                                                 : "more than 2^64 bytes";
        return fail(ST_ERR_INVALID_ARGUMENT,
                    "st_matmul_static_scratch: this problem needs " + need +
                        " of packed operands, the static scratch holds " + std::to_string(kStaticScratchBytes) +
                        " bytes ((M + N) * 3 * roundup(K, 32) * 4 must fit)");
    }
    int dev = 0;
    if (exec && exec->device >= 0) dev = exec->device;
    else ST_CUDA_TRY(cudaGetDevice(&dev));
    // NULL names the legacy default stream here: this entry point has no context
    cudaStream_t stream = exec ? static_cast<cudaStream_t>(exec->stream) : nullptr;
    if (stream != nullptr && stream != cudaStreamLegacy && stream != cudaStreamPerThread) {
        int stream_dev = -1;
        ST_CUDA_TRY(cudaStreamGetDevice(stream, &stream_dev));
        if (stream_dev != dev)
            return fail(ST_ERR_INVALID_ARGUMENT, "st_matmul_static_scratch: exec->stream belongs to device " +
                                                     std::to_string(stream_dev) + ", the call runs on device " +
                                                     std::to_string(dev));
    }
    CurrentDevice guard(dev);
    StaticDevice *sd = nullptr;
    ST_TRY(static_device(dev, &sd));
    if (M == 0 || N == 0) return ST_OK;
    if (K == 0) {
        static_fill_kernel<<<148, 256, 0, stream>>>(c->data, c->strides[0], c->dtype, bias ? bias->data : nullptr,
                                                    ST_F32, M, N);
        note_launch();
        ST_CUDA_TRY(cudaPeekAtLastError());
    } else {
        float *ap = reinterpret_cast<float *>(sd->scratch);
        float *bp = ap + M * 3 * kp;
        ST_TRY(launch_pack_a_tf32(static_cast<const float *>(a->data), a->strides[0], a->strides[1], M, K, ap, kp,
                                  stream));
        ST_TRY(launch_pack_b_tf32(static_cast<const float *>(b->data), b->strides[0], b->strides[1], K, N, bp, kp,
                                  stream));
        GemmArgs g{};
        g.ab_dtype = ST_F32;
        g.a = ap;
        g.lda = 3 * kp;
        g.b = bp;
        g.ldb = 3 * kp;
        g.b_k_major = true;
        g.c = c->data;
        g.ldc = c->strides[0];
        g.c_dtype = c->dtype;
        g.bias = bias ? bias->data : nullptr;
        g.bias_dtype = ST_F32;
        g.m = M;
        g.n = N;
        g.k = 3 * kp;
        g.deterministic = exec != nullptr && (exec->flags & ST_EXEC_DETERMINISTIC) != 0;
        ST_TRY(launch_gemm(g, sd->sm_count, sd->abort_word, kWaitLimitNs, stream));
    }
    if (exec && (exec->flags & ST_EXEC_SYNC)) {
        ST_TRY(wait_stream(stream, exec->timeout_ms));
        // this call's code, or one an earlier asynchronous call left behind
        int code = 0;
        ST_CUDA_TRY(cudaMemcpy(&code, sd->abort_word, sizeof(int), cudaMemcpyDeviceToHost));
        if (code != 0) {
            ST_CUDA_TRY(cudaMemset(sd->abort_word, 0, sizeof(int)));
            return fail(ST_ERR_DEVICE_ABORT, "a kernel gave up a bounded wait (code " + std::to_string(code) + ")");
        }
    }
    return ST_OK;
}
