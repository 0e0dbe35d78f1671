// vecadd.cu -- the elementwise tile add (cuda_tile `vector_add`, 1D and 2D).
//
// Semantics follow the reference lowering: each stored element is one
// IEEE binary32 add of the two loaded elements (tileops.hpp:610-614), so any
// correct add is bit-exact.  The tile structure only decides WHICH elements
// are produced; the runtime turns a tile grid into an element range (or a
// row/column rectangle) and these kernels stream over it.
//
// Design: HBM-bound (8 bytes read + 4 written per element).  The contiguous
// path moves 16-byte vectors with streaming cache hints, keeps several
// vectors per thread in flight, and runs a grid of (SM count x resident
// CTAs) threads that stride over the range.  Misaligned heads/tails and
// non-unit strides fall back to scalar (still coalesced) loops.
#include <cuda_runtime.h>

#include <cstdint>

#include "common.h"

namespace st {
namespace {

constexpr int kThreads = 256;
#ifndef ST_VADD_UNROLL
#define ST_VADD_UNROLL 2
#endif
constexpr int kUnroll = ST_VADD_UNROLL;  // 16-byte vectors per thread per iteration
constexpr int kCtasPerSm = 8;     // 2048 resident threads per SM

__device__ __forceinline__ float4 load_stream(const float4 *p) {
    float4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "l"(p));
    return v;
}

__device__ __forceinline__ void store_stream(float4 *p, float4 v) {
    asm volatile("st.global.L1::no_allocate.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(v.x), "f"(v.y), "f"(v.z),
                 "f"(v.w)
                 : "memory");
}

// Contiguous, 16-byte aligned: n4 float4 vectors.
__global__ void __launch_bounds__(kThreads) vadd_vec4_kernel(const float4 *__restrict__ a,
                                                             const float4 *__restrict__ b, float4 *__restrict__ c,
                                                             int64_t n4) {
    pdl_wait();
    const int64_t step = static_cast<int64_t>(gridDim.x) * kThreads * kUnroll;
    int64_t base = static_cast<int64_t>(blockIdx.x) * kThreads * kUnroll + threadIdx.x;
    // full iterations: every unrolled slot is in range
    for (; base + (kUnroll - 1) * kThreads < n4; base += step) {
        float4 va[kUnroll], vb[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            va[u] = load_stream(a + base + u * kThreads);
            vb[u] = load_stream(b + base + u * kThreads);
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            float4 r;
            r.x = va[u].x + vb[u].x;
            r.y = va[u].y + vb[u].y;
            r.z = va[u].z + vb[u].z;
            r.w = va[u].w + vb[u].w;
            store_stream(c + base + u * kThreads, r);
        }
    }
    // ragged last iteration
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
        const int64_t i = base + u * kThreads;
        if (i < n4) {
            const float4 x = load_stream(a + i), y = load_stream(b + i);
            float4 r;
            r.x = x.x + y.x;
            r.y = x.y + y.y;
            r.z = x.z + y.z;
            r.w = x.w + y.w;
            store_stream(c + i, r);
        }
    }
    pdl_trigger();
}

// Any element strides (also the misaligned head/tail of the vector path).
__global__ void __launch_bounds__(kThreads) vadd_strided_kernel(const float *__restrict__ a, int64_t sa,
                                                                const float *__restrict__ b, int64_t sb,
                                                                float *__restrict__ c, int64_t sc, int64_t n) {
    pdl_wait();
    const int64_t step = static_cast<int64_t>(gridDim.x) * kThreads;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x; i < n; i += step)
        c[i * sc] = a[i * sa] + b[i * sb];
    pdl_trigger();
}

// 2D rectangle with arbitrary strides: rows x cols, one thread per element of
// a row-major enumeration so that unit column strides stay coalesced.
__global__ void __launch_bounds__(kThreads) vadd_2d_kernel(const float *__restrict__ a, int64_t sa0, int64_t sa1,
                                                           const float *__restrict__ b, int64_t sb0, int64_t sb1,
                                                           float *__restrict__ c, int64_t sc0, int64_t sc1,
                                                           int64_t rows, int64_t cols) {
    pdl_wait();
    const int64_t total = rows * cols;
    const int64_t step = static_cast<int64_t>(gridDim.x) * kThreads;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x; i < total; i += step) {
        const int64_t r = i / cols, q = i - r * cols;
        c[r * sc0 + q * sc1] = a[r * sa0 + q * sa1] + b[r * sb0 + q * sb1];
    }
    pdl_trigger();
}

int grid_for(int64_t work_items, int per_cta, int sm_count) {
    const int64_t want = cdiv(work_items, per_cta);
    const int64_t cap = static_cast<int64_t>(sm_count > 0 ? sm_count : 148) * kCtasPerSm;
    int64_t g = want < cap ? want : cap;
    return static_cast<int>(g > 0 ? g : 1);
}

}  // namespace

int launch_vector_add_1d(const float *a, int64_t sa, const float *b, int64_t sb, float *c, int64_t sc, int64_t n,
                         int sm_count, cudaStream_t stream) {
    if (n <= 0) return ST_OK;
    const uintptr_t pa = reinterpret_cast<uintptr_t>(a), pb = reinterpret_cast<uintptr_t>(b),
                    pc = reinterpret_cast<uintptr_t>(c);
    const bool unit = sa == 1 && sb == 1 && sc == 1;
    const bool same_phase = (pa % 16) == (pb % 16) && (pa % 16) == (pc % 16) && (pa % 4) == 0;
    if (!unit || !same_phase || n < 64) {
        ST_CUDA_TRY(launch_kernel(vadd_strided_kernel, grid_for(n, kThreads, sm_count), kThreads, 0, stream, a, sa, b,
                                  sb, c, sc, n));
        note_launch();
        return cudaPeekAtLastError() == cudaSuccess ? ST_OK : cuda_fail(cudaGetLastError(), "vadd_strided_kernel");
    }
    // scalar head up to the first 16-byte boundary, vector body, scalar tail
    const int64_t head = static_cast<int64_t>(((16 - (pa % 16)) % 16) / 4);
    const int64_t body4 = (n - head) / 4;
    const int64_t tail_start = head + body4 * 4;
    if (head > 0) {
        ST_CUDA_TRY(launch_kernel(vadd_strided_kernel, 1, kThreads, 0, stream, a, 1, b, 1, c, 1, head));
        note_launch();
    }
    if (body4 > 0) {
        ST_CUDA_TRY(launch_kernel(vadd_vec4_kernel, grid_for(body4, kThreads * kUnroll, sm_count), kThreads, 0, stream,
                                  reinterpret_cast<const float4 *>(a + head),
                                  reinterpret_cast<const float4 *>(b + head), reinterpret_cast<float4 *>(c + head),
                                  body4));
        note_launch();
    }
    if (tail_start < n) {
        ST_CUDA_TRY(launch_kernel(vadd_strided_kernel, 1, kThreads, 0, stream, a + tail_start, 1, b + tail_start, 1,
                                  c + tail_start, 1, n - tail_start));
        note_launch();
    }
    const cudaError_t e = cudaPeekAtLastError();
    return e == cudaSuccess ? ST_OK : cuda_fail(cudaGetLastError(), "vadd_vec4_kernel");
}

int launch_vector_add_2d(const float *a, const int64_t sa[2], const float *b, const int64_t sb[2], float *c,
                         const int64_t sc[2], int64_t rows, int64_t cols, int sm_count, cudaStream_t stream) {
    if (rows <= 0 || cols <= 0) return ST_OK;
    // rows laid end to end in all three arrays: one contiguous range
    const bool dense = sa[1] == 1 && sb[1] == 1 && sc[1] == 1 && sa[0] == cols && sb[0] == cols && sc[0] == cols;
    if (dense || rows == 1) {
        if (rows == 1) return launch_vector_add_1d(a, sa[1], b, sb[1], c, sc[1], cols, sm_count, stream);
        return launch_vector_add_1d(a, 1, b, 1, c, 1, rows * cols, sm_count, stream);
    }
    // unit column stride: one vectorised launch per row is wasteful for many
    // short rows, so use the 2D kernel unless rows are long
    if (sa[1] == 1 && sb[1] == 1 && sc[1] == 1 && cols >= 4096 && rows <= 64) {
        for (int64_t r = 0; r < rows; ++r)
            ST_TRY(launch_vector_add_1d(a + r * sa[0], 1, b + r * sb[0], 1, c + r * sc[0], 1, cols, sm_count,
                                        stream));
        return ST_OK;
    }
    ST_CUDA_TRY(launch_kernel(vadd_2d_kernel, grid_for(rows * cols, kThreads, sm_count), kThreads, 0, stream, a, sa[0],
                              sa[1], b, sb[0], sb[1], c, sc[0], sc[1], rows, cols));
    note_launch();
    const cudaError_t e = cudaPeekAtLastError();
    return e == cudaSuccess ? ST_OK : cuda_fail(cudaGetLastError(), "vadd_2d_kernel");
}

}  // namespace st
