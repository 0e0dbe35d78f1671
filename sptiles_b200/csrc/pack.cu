// pack.cu -- operand preparation for the tensor-core matmul.
//
// fp32 inputs: the reference computes the fp32 matmul at full precision
// (its astype(tfloat32) lowers to identity, tileops.hpp:257-258).  The
// tensor cores take tf32 (10 explicit mantissa bits), so each fp32 value is
// split x = hi + lo with hi = tf32(x) and lo = tf32(x - hi), and the product
// uses the three largest terms hi*hi + hi*lo + lo*hi -- the published
// 3xTF32 method (CUTLASS's 3xTF32 GEMM; Ootomo & Yokota, "Recovering single
// precision accuracy from Tensor Cores while surpassing the FP32 theoretical
// peak performance", IJHPCA 2022).  Both halves are rounded to tf32 here, so
// the tensor core's own handling of the discarded mantissa bits is moot.
//
// The three terms become ONE tf32 GEMM over a tripled K:
//   Ap = [hi(A) | hi(A) | lo(A)]            [M, 3*kp], K contiguous
//   Bp = [hi(B) ; lo(B) ; hi(B)]^T           [N, 3*kp], K contiguous
// with kp = K rounded up to the 32-element stage depth (zero padded).
//
// 16-bit inputs whose strides TMA cannot address are copied into a dense
// row-major scratch matrix first (repack_16).
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "common.h"

namespace st {
namespace {

constexpr int kThreads = 256;

// Round to tf32 (10 explicit mantissa bits), nearest-even; inf/nan unchanged.
__device__ __forceinline__ float tf32_round(float x) {
    uint32_t u = __float_as_uint(x);
    if ((u & 0x7f800000u) == 0x7f800000u) return x;
    u += 0x0fffu + ((u >> 13) & 1u);
    return __uint_as_float(u & 0xffffe000u);
}

__global__ void __launch_bounds__(kThreads) pack_a_kernel(const float *__restrict__ a, int64_t sa0, int64_t sa1,
                                                          int64_t m, int64_t k, float *__restrict__ ap,
                                                          int64_t kp) {
    pdl_wait();
    // one thread per 4 consecutive k of one row
    const int64_t groups = kp / 4;
    const int64_t total = m * groups;
    const int64_t step = static_cast<int64_t>(gridDim.x) * kThreads;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x; i < total; i += step) {
        const int64_t r = i / groups;
        const int64_t k0 = (i - r * groups) * 4;
        float hi[4], lo[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float x = (k0 + j < k) ? a[r * sa0 + (k0 + j) * sa1] : 0.0f;
            hi[j] = tf32_round(x);
            lo[j] = tf32_round(x - hi[j]);
        }
        float4 *row = reinterpret_cast<float4 *>(ap + r * 3 * kp);
        const float4 h = make_float4(hi[0], hi[1], hi[2], hi[3]);
        row[k0 / 4] = h;
        row[(kp + k0) / 4] = h;
        row[(2 * kp + k0) / 4] = make_float4(lo[0], lo[1], lo[2], lo[3]);
    }
    pdl_trigger();
}

// B [K, N] -> Bp [N, 3*kp]: 32 x 32 tiles transposed through shared memory.
__global__ void __launch_bounds__(kThreads) pack_b_kernel(const float *__restrict__ b, int64_t sb0, int64_t sb1,
                                                          int64_t k, int64_t n, float *__restrict__ bp,
                                                          int64_t kp) {
    pdl_wait();
    __shared__ float hi_t[32][33];
    __shared__ float lo_t[32][33];
    const int64_t k0 = static_cast<int64_t>(blockIdx.x) * 32;
    const int64_t n0 = static_cast<int64_t>(blockIdx.y) * 32;
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 8
    for (int r = ty; r < 32; r += 8) {
        const int64_t kk = k0 + r, nn = n0 + tx;
        const float x = (kk < k && nn < n) ? b[kk * sb0 + nn * sb1] : 0.0f;
        const float h = tf32_round(x);
        hi_t[r][tx] = h;
        lo_t[r][tx] = tf32_round(x - h);
    }
    __syncthreads();
    for (int r = ty; r < 32; r += 8) {
        const int64_t nn = n0 + r, kk = k0 + tx;
        if (nn < n && kk < kp) {
            float *row = bp + nn * 3 * kp;
            const float h = hi_t[tx][r];
            row[kk] = h;
            row[kp + kk] = lo_t[tx][r];
            row[2 * kp + kk] = h;
        }
    }
    pdl_trigger();
}

__device__ __forceinline__ float preset_bias(const CPreset &p, int q) {
    if (p.bias == nullptr) return 0.0f;
    float v;
    if (p.bias_dtype == ST_F32) v = static_cast<const float *>(p.bias)[q];
    else if (p.bias_dtype == ST_F16) v = __half2float(static_cast<const __half *>(p.bias)[q]);
    else v = __bfloat162float(static_cast<const __nv_bfloat16 *>(p.bias)[q]);
    return 0.0f + v;  // -0 becomes +0, as an accumulator that starts at +0 would give
}

// Both operands in one launch: blocks [0, tiles_b) transpose B's 32 x 32
// tiles (as pack_b_kernel), the rest split A's rows (as pack_a_kernel) and
// then, when preset.c is set, write C's starting value (one 16-byte store
// per four columns; rows are 16-byte aligned).
__global__ void __launch_bounds__(kThreads) pack_ab_kernel(const float *__restrict__ a, int64_t sa0, int64_t sa1,
                                                           int64_t m, const float *__restrict__ b, int64_t sb0,
                                                           int64_t sb1, int64_t n, int64_t k, int64_t kp,
                                                           float *__restrict__ ap, float *__restrict__ bp,
                                                           int tiles_k, int tiles_b, const CPreset preset) {
    pdl_wait();
    __shared__ float hi_t[32][33];
    __shared__ float lo_t[32][33];
    if (static_cast<int>(blockIdx.x) < tiles_b) {
        const int64_t k0 = static_cast<int64_t>(blockIdx.x % tiles_k) * 32;
        const int64_t n0 = static_cast<int64_t>(blockIdx.x / tiles_k) * 32;
        const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 8
        // 16-byte path: thread (r, c) = (tid / 8, tid % 8) loads B[k0 + r][n0 + 4c ..
        // + 3]; the [k][n] tiles (row pitch 33) stay free of bank conflicts
        const int vr = threadIdx.x >> 3, vc = threadIdx.x & 7;
        const bool full_n = n0 + 32 <= n;
        if (full_n && k0 + 32 <= k && sb1 == 1 && sb0 % 4 == 0 && reinterpret_cast<uintptr_t>(b) % 16 == 0) {
            const float4 v = *reinterpret_cast<const float4 *>(b + (k0 + vr) * sb0 + n0 + 4 * vc);
            const float x[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int t = 0; t < 4; ++t) {
                const float h = tf32_round(x[t]);
                hi_t[vr][4 * vc + t] = h;
                lo_t[vr][4 * vc + t] = tf32_round(x[t] - h);
            }
        } else {
            for (int r = ty; r < 32; r += 8) {
                const int64_t kk = k0 + r, nn = n0 + tx;
                const float x = (kk < k && nn < n) ? b[kk * sb0 + nn * sb1] : 0.0f;
                const float h = tf32_round(x);
                hi_t[r][tx] = h;
                lo_t[r][tx] = tf32_round(x - h);
            }
        }
        __syncthreads();
        if (full_n) {  // row n0 + vr of Bp, K elements k0 + 4c .. + 3 of each segment (k0 + 32 <= kp)
            const int kq = 4 * vc;
            const float4 h = make_float4(hi_t[kq][vr], hi_t[kq + 1][vr], hi_t[kq + 2][vr], hi_t[kq + 3][vr]);
            const float4 l = make_float4(lo_t[kq][vr], lo_t[kq + 1][vr], lo_t[kq + 2][vr], lo_t[kq + 3][vr]);
            float *row = bp + (n0 + vr) * 3 * kp + k0 + kq;
            *reinterpret_cast<float4 *>(row) = h;
            *reinterpret_cast<float4 *>(row + kp) = l;
            *reinterpret_cast<float4 *>(row + 2 * kp) = h;
        } else {
            for (int r = ty; r < 32; r += 8) {
                const int64_t nn = n0 + r, kk = k0 + tx;
                if (nn < n && kk < kp) {
                    float *row = bp + nn * 3 * kp;
                    const float h = hi_t[tx][r];
                    row[kk] = h;
                    row[kp + kk] = lo_t[tx][r];
                    row[2 * kp + kk] = h;
                }
            }
        }
        return;
    }
    // A's rows, then C's preset rows: block j of the rest handles rows j,
    // j + blocks, ... (no index division), one 4-element group per thread
    // and pass; 16-byte loads when A's rows are dense and aligned
    const int64_t blocks = static_cast<int64_t>(gridDim.x) - tiles_b;
    const int64_t j0 = static_cast<int64_t>(blockIdx.x) - tiles_b;
    const int groups = static_cast<int>(kp / 4);
    const bool a_vec = sa1 == 1 && sa0 % 4 == 0 && reinterpret_cast<uintptr_t>(a) % 16 == 0;
    for (int64_t r = j0; r < m; r += blocks) {
        const float *arow = a + r * sa0;
        float4 *prow = reinterpret_cast<float4 *>(ap + r * 3 * kp);
        for (int q = threadIdx.x; q < groups; q += kThreads) {
            const int64_t k0 = 4 * static_cast<int64_t>(q);
            float x[4];
            if (a_vec && k0 + 4 <= k) {
                const float4 v = *reinterpret_cast<const float4 *>(arow + k0);
                x[0] = v.x;
                x[1] = v.y;
                x[2] = v.z;
                x[3] = v.w;
            } else {
#pragma unroll
                for (int t = 0; t < 4; ++t) x[t] = k0 + t < k ? arow[(k0 + t) * sa1] : 0.0f;
            }
            float hi[4], lo[4];
#pragma unroll
            for (int t = 0; t < 4; ++t) {
                hi[t] = tf32_round(x[t]);
                lo[t] = tf32_round(x[t] - hi[t]);
            }
            const float4 h = make_float4(hi[0], hi[1], hi[2], hi[3]);
            prow[q] = h;
            prow[groups + q] = h;
            prow[2 * groups + q] = make_float4(lo[0], lo[1], lo[2], lo[3]);
        }
    }
    if (preset.c != nullptr) {
        const int quads = (preset.n + 3) / 4;
        for (int64_t r = j0; r < preset.m; r += blocks) {
            float *row = preset.c + r * preset.ldc;
            for (int q = threadIdx.x; q < quads; q += kThreads) {
                const int q0 = 4 * q;
                if (q0 + 4 <= preset.n) {
                    reinterpret_cast<float4 *>(row)[q] =
                        make_float4(preset_bias(preset, q0), preset_bias(preset, q0 + 1),
                                    preset_bias(preset, q0 + 2), preset_bias(preset, q0 + 3));
                } else {
                    for (int c = q0; c < preset.n; ++c) row[c] = preset_bias(preset, c);
                }
            }
        }
    }
    pdl_trigger();
}

__global__ void __launch_bounds__(kThreads) repack_16_kernel(const uint16_t *__restrict__ src, int64_t s0,
                                                             int64_t s1, int64_t rows, int64_t cols,
                                                             uint16_t *__restrict__ dst, int64_t ld) {
    pdl_wait();
    const int64_t total = rows * ld;
    const int64_t step = static_cast<int64_t>(gridDim.x) * kThreads;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x; i < total; i += step) {
        const int64_t r = i / ld, c = i - r * ld;
        dst[i] = c < cols ? src[r * s0 + c * s1] : static_cast<uint16_t>(0);
    }
    pdl_trigger();
}

int grid_1d(int64_t items) {
    int64_t g = cdiv(items, kThreads);
    if (g > 148 * 16) g = 148 * 16;
    return static_cast<int>(g > 0 ? g : 1);
}

}  // namespace

int64_t tf32_packed_k(int64_t k) { return cdiv(k, 32) * 32; }

int preload_pack_tf32_kernels() {
    cudaFuncAttributes attr;
    ST_CUDA_TRY(cudaFuncGetAttributes(&attr, pack_a_kernel));
    ST_CUDA_TRY(cudaFuncGetAttributes(&attr, pack_b_kernel));
    return ST_OK;
}

int launch_pack_a_tf32(const float *a, int64_t sa0, int64_t sa1, int64_t m, int64_t k, float *ap, int64_t kp,
                       cudaStream_t stream) {
    if (m <= 0 || kp <= 0) return ST_OK;
    ST_CUDA_TRY(launch_kernel(pack_a_kernel, grid_1d(m * (kp / 4)), kThreads, 0, stream, a, sa0, sa1, m, k, ap, kp));
    note_launch();
    const cudaError_t e = cudaPeekAtLastError();
    return e == cudaSuccess ? ST_OK : cuda_fail(cudaGetLastError(), "pack_a_kernel");
}

int launch_pack_b_tf32(const float *b, int64_t sb0, int64_t sb1, int64_t k, int64_t n, float *bp, int64_t kp,
                       cudaStream_t stream) {
    if (n <= 0 || kp <= 0) return ST_OK;
    dim3 grid(static_cast<unsigned>(cdiv(kp, 32)), static_cast<unsigned>(cdiv(n, 32)));
    ST_CUDA_TRY(launch_kernel(pack_b_kernel, grid, kThreads, 0, stream, b, sb0, sb1, k, n, bp, kp));
    note_launch();
    const cudaError_t e = cudaPeekAtLastError();
    return e == cudaSuccess ? ST_OK : cuda_fail(cudaGetLastError(), "pack_b_kernel");
}

int launch_pack_ab_tf32(const float *a, int64_t sa0, int64_t sa1, int64_t m, const float *b, int64_t sb0,
                        int64_t sb1, int64_t n, int64_t k, float *ap, float *bp, int64_t kp, const CPreset *preset,
                        cudaStream_t stream) {
    if (kp <= 0 || (m <= 0 && n <= 0)) return ST_OK;
    const CPreset cp = preset != nullptr && preset->m > 0 && preset->n > 0 ? *preset : CPreset{};
    if (cp.c != nullptr && (reinterpret_cast<uintptr_t>(cp.c) % 16 != 0 || cp.ldc % 4 != 0))
        return fail(ST_ERR_INVALID_ARGUMENT, "C preset needs 16-byte aligned rows");
    const int64_t tiles_k = cdiv(kp, 32);
    const int64_t tiles_b = n > 0 ? tiles_k * cdiv(n, 32) : 0;
    // one block per row of A (or of C's preset), at most 148 x 16
    const int64_t rows = m > cp.m ? m : cp.m;
    const int64_t blocks_a = rows > 0 ? (rows < 148 * 16 ? rows : 148 * 16) : 0;
    if (kp / 4 > (int64_t(1) << 30)) return fail(ST_ERR_UNSUPPORTED, "fp32 K too large for one pack launch");
    if (tiles_b + blocks_a > (int64_t(1) << 31) - 1)
        return fail(ST_ERR_UNSUPPORTED, "fp32 operands too large for one pack launch");
    ST_CUDA_TRY(launch_kernel(pack_ab_kernel, static_cast<unsigned>(tiles_b + blocks_a), kThreads, 0, stream, a, sa0,
                              sa1, m > 0 ? m : 0, b, sb0, sb1, n, k, kp, ap, bp, static_cast<int>(tiles_k),
                              static_cast<int>(tiles_b), cp));
    note_launch();
    const cudaError_t e = cudaPeekAtLastError();
    return e == cudaSuccess ? ST_OK : cuda_fail(cudaGetLastError(), "pack_ab_kernel");
}

int launch_repack_16(const uint16_t *src, int64_t s0, int64_t s1, int64_t rows, int64_t cols, uint16_t *dst,
                     int64_t ld, cudaStream_t stream) {
    if (rows <= 0 || ld <= 0) return ST_OK;
    ST_CUDA_TRY(
        launch_kernel(repack_16_kernel, grid_1d(rows * ld), kThreads, 0, stream, src, s0, s1, rows, cols, dst, ld));
    note_launch();
    const cudaError_t e = cudaPeekAtLastError();
    return e == cudaSuccess ? ST_OK : cuda_fail(cudaGetLastError(), "repack_16_kernel");
}

}  // namespace st
