// elementwise.cu -- the other elementwise ops the reference lowering
// materialises: fused multiply-add (`fma`, tileops.hpp:616-623, emitted as
// GLSL.std.450 Fma) and floating-point conversion (`ftof`,
// tileops.hpp:257-258, a pass-through in the f32-only reference).
//
// Both are HBM-bound streams like the tile add: contiguous views with a
// common 16-byte phase move 16-byte vectors; anything else runs a coalesced
// element-wise 2D loop (a rank-1 view is one row).
//   fma:  C = A * B + D rounded once (IEEE fused multiply-add)
//   cast: C = A converted to C's type (f32 / f16 / bf16), round to nearest
//         even when narrowing, exact when widening
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "common.h"

namespace st {
namespace {

constexpr int kThreads = 256;

int grid_for(int64_t items, int sm_count) {
    int64_t g = cdiv(items, kThreads);
    const int64_t cap = static_cast<int64_t>(sm_count > 0 ? sm_count : 148) * 8;
    if (g > cap) g = cap;
    return static_cast<int>(g > 0 ? g : 1);
}

// ------------------------------------------------------------------ fma
__global__ void __launch_bounds__(kThreads) fma_vec4_kernel(const float4 *__restrict__ a, const float4 *__restrict__ b,
                                                            const float4 *__restrict__ d, float4 *__restrict__ c,
                                                            int64_t n4) {
    pdl_wait();
    const int64_t step = static_cast<int64_t>(gridDim.x) * kThreads;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x; i < n4; i += step) {
        const float4 x = __ldcs(a + i), y = __ldcs(b + i), z = __ldcs(d + i);
        float4 r;
        r.x = __fmaf_rn(x.x, y.x, z.x);
        r.y = __fmaf_rn(x.y, y.y, z.y);
        r.z = __fmaf_rn(x.z, y.z, z.z);
        r.w = __fmaf_rn(x.w, y.w, z.w);
        __stcs(c + i, r);
    }
    pdl_trigger();
}

struct View2 {
    const void *p;
    int64_t s0, s1;
};

__global__ void __launch_bounds__(kThreads) fma_2d_kernel(View2 a, View2 b, View2 d, float *__restrict__ c, int64_t sc0,
                                                          int64_t sc1, int64_t rows, int64_t cols) {
    pdl_wait();
    const int64_t total = rows * cols;
    const int64_t step = static_cast<int64_t>(gridDim.x) * kThreads;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x; i < total; i += step) {
        const int64_t r = i / cols, q = i - r * cols;
        const float x = static_cast<const float *>(a.p)[r * a.s0 + q * a.s1];
        const float y = static_cast<const float *>(b.p)[r * b.s0 + q * b.s1];
        const float z = static_cast<const float *>(d.p)[r * d.s0 + q * d.s1];
        c[r * sc0 + q * sc1] = __fmaf_rn(x, y, z);
    }
    pdl_trigger();
}

// ------------------------------------------------------------------ cast
template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename T>
__device__ __forceinline__ T from_f32(float v);
template <>
__device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

// Contiguous: four elements per thread per step (aligned to four elements).
template <typename In, typename Out>
__global__ void __launch_bounds__(kThreads) cast_vec4_kernel(const In *__restrict__ a, Out *__restrict__ c, int64_t n4) {
    pdl_wait();
    struct alignas(4 * sizeof(In)) InVec { In v[4]; };
    struct alignas(4 * sizeof(Out)) OutVec { Out v[4]; };
    const InVec *av = reinterpret_cast<const InVec *>(a);
    OutVec *cv = reinterpret_cast<OutVec *>(c);
    const int64_t step = static_cast<int64_t>(gridDim.x) * kThreads;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x; i < n4; i += step) {
        const InVec x = av[i];
        OutVec y;
#pragma unroll
        for (int j = 0; j < 4; ++j) y.v[j] = from_f32<Out>(to_f32<In>(x.v[j]));
        cv[i] = y;
    }
    pdl_trigger();
}

template <typename In, typename Out>
__global__ void __launch_bounds__(kThreads) cast_2d_kernel(const In *__restrict__ a, int64_t sa0, int64_t sa1,
                                                           Out *__restrict__ c, int64_t sc0, int64_t sc1, int64_t rows,
                                                           int64_t cols) {
    pdl_wait();
    const int64_t total = rows * cols;
    const int64_t step = static_cast<int64_t>(gridDim.x) * kThreads;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x; i < total; i += step) {
        const int64_t r = i / cols, q = i - r * cols;
        c[r * sc0 + q * sc1] = from_f32<Out>(to_f32<In>(a[r * sa0 + q * sa1]));
    }
    pdl_trigger();
}

template <typename In, typename Out>
int cast_typed(const void *a, const int64_t sa[2], void *c, const int64_t sc[2], int64_t rows, int64_t cols,
               int sm_count, cudaStream_t stream) {
    const In *ap = static_cast<const In *>(a);
    Out *cp = static_cast<Out *>(c);
    const bool dense = (sa[1] == 1 || cols == 1) && (sc[1] == 1 || cols == 1) && (rows == 1 || (sa[0] == cols && sc[0] == cols));
    const int64_t n = rows * cols;
    const bool aligned = (reinterpret_cast<uintptr_t>(a) % (4 * sizeof(In))) == 0 &&
                         (reinterpret_cast<uintptr_t>(c) % (4 * sizeof(Out))) == 0;
    if (dense && aligned && n >= 4) {
        const int64_t n4 = n / 4;
        ST_CUDA_TRY(launch_kernel(cast_vec4_kernel<In, Out>, grid_for(n4, sm_count), kThreads, 0, stream, ap, cp, n4));
        note_launch();
        if (n4 * 4 < n) {
            const int64_t s1[2] = {0, 1};
            ST_CUDA_TRY(launch_kernel(cast_2d_kernel<In, Out>, 1, kThreads, 0, stream, ap + n4 * 4, s1[0], s1[1],
                                      cp + n4 * 4, 0, 1, 1, n - n4 * 4));
            note_launch();
        }
    } else {
        ST_CUDA_TRY(launch_kernel(cast_2d_kernel<In, Out>, grid_for(n, sm_count), kThreads, 0, stream, ap, sa[0], sa[1],
                                  cp, sc[0], sc[1], rows, cols));
        note_launch();
    }
    const cudaError_t e = cudaPeekAtLastError();
    return e == cudaSuccess ? ST_OK : cuda_fail(cudaGetLastError(), "cast kernel");
}

template <typename In>
int cast_from(const void *a, const int64_t sa[2], void *c, int c_dtype, const int64_t sc[2], int64_t rows, int64_t cols,
              int sm_count, cudaStream_t stream) {
    switch (c_dtype) {
    case ST_F32: return cast_typed<In, float>(a, sa, c, sc, rows, cols, sm_count, stream);
    case ST_F16: return cast_typed<In, __half>(a, sa, c, sc, rows, cols, sm_count, stream);
    case ST_BF16: return cast_typed<In, __nv_bfloat16>(a, sa, c, sc, rows, cols, sm_count, stream);
    default: return fail(ST_ERR_INVALID_ARGUMENT, "cast: C must be ST_F32, ST_F16 or ST_BF16");
    }
}

}  // namespace

int launch_vector_fma(const float *a, const int64_t sa[2], const float *b, const int64_t sb[2], const float *d,
                      const int64_t sd[2], float *c, const int64_t sc[2], int64_t rows, int64_t cols, int sm_count,
                      cudaStream_t stream) {
    if (rows <= 0 || cols <= 0) return ST_OK;
    const int64_t n = rows * cols;
    const bool dense = [&] {
        for (const int64_t *s : {sa, sb, sd, sc})
            if (!((s[1] == 1 || cols == 1) && (rows == 1 || s[0] == cols))) return false;
        return true;
    }();
    const uintptr_t pa = reinterpret_cast<uintptr_t>(a);
    const bool aligned = pa % 16 == 0 && reinterpret_cast<uintptr_t>(b) % 16 == 0 &&
                         reinterpret_cast<uintptr_t>(d) % 16 == 0 && reinterpret_cast<uintptr_t>(c) % 16 == 0;
    if (dense && aligned && n >= 4) {
        const int64_t n4 = n / 4;
        ST_CUDA_TRY(launch_kernel(fma_vec4_kernel, grid_for(n4, sm_count), kThreads, 0, stream,
                                  reinterpret_cast<const float4 *>(a), reinterpret_cast<const float4 *>(b),
                                  reinterpret_cast<const float4 *>(d), reinterpret_cast<float4 *>(c), n4));
        note_launch();
        if (n4 * 4 < n) {
            const int64_t off = n4 * 4;
            ST_CUDA_TRY(launch_kernel(fma_2d_kernel, 1, kThreads, 0, stream, View2{a + off, 0, 1},
                                      View2{b + off, 0, 1}, View2{d + off, 0, 1}, c + off, 0, 1, 1, n - off));
            note_launch();
        }
    } else {
        ST_CUDA_TRY(launch_kernel(fma_2d_kernel, grid_for(n, sm_count), kThreads, 0, stream, View2{a, sa[0], sa[1]},
                                  View2{b, sb[0], sb[1]}, View2{d, sd[0], sd[1]}, c, sc[0], sc[1], rows, cols));
        note_launch();
    }
    const cudaError_t e = cudaPeekAtLastError();
    return e == cudaSuccess ? ST_OK : cuda_fail(cudaGetLastError(), "fma kernel");
}

int launch_cast(const void *a, int a_dtype, const int64_t sa[2], void *c, int c_dtype, const int64_t sc[2],
                int64_t rows, int64_t cols, int sm_count, cudaStream_t stream) {
    if (rows <= 0 || cols <= 0) return ST_OK;
    switch (a_dtype) {
    case ST_F32: return cast_from<float>(a, sa, c, c_dtype, sc, rows, cols, sm_count, stream);
    case ST_F16: return cast_from<__half>(a, sa, c, c_dtype, sc, rows, cols, sm_count, stream);
    case ST_BF16: return cast_from<__nv_bfloat16>(a, sa, c, c_dtype, sc, rows, cols, sm_count, stream);
    default: return fail(ST_ERR_INVALID_ARGUMENT, "cast: A must be ST_F32, ST_F16 or ST_BF16");
    }
}

}  // namespace st
