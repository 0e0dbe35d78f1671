/*
 * CPU oracle for the spTiles hot path -- TEST INFRASTRUCTURE ONLY.
 *
 * This file restates, in plain C, the arithmetic that the spTiles lowering
 * (src/tileops.hpp, src/lower.hpp) emits as SPIR-V for the two cuda_tile
 * workloads, so that the CUDA kernels can be checked against it.  It is the
 * checker, never the product: only tests, the smoke check and the CPU
 * baseline leg of the benchmark load it.
 *
 * Parity pin: the reference's own known-answer tests (src/examples.cpp
 * 477-480 and 590-596, shaders/spirv_vector_add.py 105-108,
 * shaders/spirv_matmul.py 126-136) are checked against this file by the
 * CPU test suite through golden fixtures generated from the reference's own
 * Python code.  The reference translator itself cannot be built here (the
 * ext/cuda-tile submodule is empty and there is no LLVM/MLIR), and its
 * Vulkan runners need a graphics stack, so ulp-level parity with a Vulkan
 * driver's execution of the SPIR-V is not pinned; the fp32 semantics below
 * and the reference's stated tolerances are.
 *
 * Must be compiled with -ffp-contract=off: the SPIR-V issues OpFMul and
 * OpFAdd as separate, separately rounded operations (tileops.hpp:733-734).
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define OR_F32 0
#define OR_F16 1
#define OR_BF16 2

#define OR_OK 0
#define OR_ERR_ARG 1
#define OR_ERR_MEM 2

/* ------------------------------------------------------------------------ */
/* Scalar conversions (IEEE-754 bit arithmetic, round-to-nearest-even).     */
/* ------------------------------------------------------------------------ */

static inline uint32_t f32_bits(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    return u;
}

static inline float bits_f32(uint32_t u) {
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* binary16 -> binary32, exact. */
float or_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1fu;
    uint32_t man = h & 0x3ffu;
    if (exp == 0x1f) /* inf / nan */
        return bits_f32(sign | 0x7f800000u | (man << 13));
    if (exp == 0) {
        if (man == 0) return bits_f32(sign);
        /* subnormal: value = man * 2^-24 (exact in binary32) */
        float v = (float)man * 5.9604644775390625e-08f;
        return sign ? -v : v;
    }
    return bits_f32(sign | ((exp + 112u) << 23) | (man << 13));
}

/* bfloat16 -> binary32, exact (upper half of the binary32 pattern). */
float or_bf16_to_f32(uint16_t b) { return bits_f32((uint32_t)b << 16); }

/* binary32 -> bfloat16, round to nearest even; NaN stays NaN. */
uint16_t or_f32_to_bf16(float f) {
    uint32_t u = f32_bits(f);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
    uint32_t lsb = (u >> 16) & 1u;
    u += 0x7fffu + lsb;
    return (uint16_t)(u >> 16);
}

/* binary32 -> binary16, round to nearest even, overflow to inf. */
uint16_t or_f32_to_f16(float f) {
    uint32_t u = f32_bits(f);
    uint32_t sign = (u >> 16) & 0x8000u;
    uint32_t a = u & 0x7fffffffu;
    if (a > 0x7f800000u) return (uint16_t)(sign | 0x7e00u); /* nan */
    if (a >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u); /* >= 65520 rounds to inf */
    if (a < 0x38800000u) {
        /* result is subnormal or zero: value / 2^-24, rounded to an integer */
        float v = bits_f32(a) * 16777216.0f; /* exact scaling by 2^24 */
        /* nearbyintf rounds half to even under the default rounding mode */
        uint32_t m = (uint32_t)nearbyintf(v);
        return (uint16_t)(sign | m); /* m == 0x400 carries into the exponent */
    }
    /* normal range: re-bias exponent, round mantissa 23 -> 10 bits */
    uint32_t r = a - 0x38000000u; /* exponent bias 127 -> 15 */
    uint32_t lsb = (r >> 13) & 1u;
    r += 0x0fffu + lsb;
    return (uint16_t)(sign | (r >> 13));
}

/* ------------------------------------------------------------------------ */
/* vector_add: elementwise tile add (tileops.hpp:497-614, 1054-1097).       */
/* ------------------------------------------------------------------------ */

/*
 * 1D tile add.  Tile block b of the cuda_tile grid owns elements
 * [b*T, (b+1)*T) (vecadd.py:7-20: ct.load index=(pid,), shape=(T,)).  The
 * store is guarded by idx < C.size (materialize_partition_view_in_bounds,
 * tileops.hpp:451-472); the loads carry no padding (vecadd.py loads without
 * padding_mode), so the caller must make A and B cover every stored index.
 * Each stored value is one IEEE binary32 add, OpFAdd (tileops.hpp:610-614).
 * Strides are in elements (tileops.hpp:330-345: offset = idx * stride).
 */
int or_vector_add_1d(const float *a, int64_t a_size, int64_t a_stride,
                     const float *b, int64_t b_size, int64_t b_stride,
                     float *c, int64_t c_size, int64_t c_stride,
                     int64_t tile, int64_t grid_tiles) {
    if (tile <= 0 || grid_tiles < 0) return OR_ERR_ARG;
    int64_t end = grid_tiles * tile;
    if (end > c_size) end = c_size;
    if (end > a_size || end > b_size) return OR_ERR_ARG;
    for (int64_t i = 0; i < end; ++i) c[i * c_stride] = a[i * a_stride] + b[i * b_stride];
    return OR_OK;
}

/*
 * 2D tile add.  Tile block (bx, by) of a (grid_x, grid_y) grid owns rows
 * [bx*tm, bx*tm+tm) and columns [by*tn, by*tn+tn); the store is guarded by
 * row < dim0 && col < dim1 (tileops.hpp:474-494) and addresses are
 * row*stride0 + col*stride1 (tileops.hpp:348-371).
 */
int or_vector_add_2d(const float *a, const int64_t a_shape[2], const int64_t a_strides[2],
                     const float *b, const int64_t b_shape[2], const int64_t b_strides[2],
                     float *c, const int64_t c_shape[2], const int64_t c_strides[2],
                     int64_t tm, int64_t tn, int64_t grid_x, int64_t grid_y) {
    if (tm <= 0 || tn <= 0 || grid_x < 0 || grid_y < 0) return OR_ERR_ARG;
    int64_t rows = grid_x * tm, cols = grid_y * tn;
    if (rows > c_shape[0]) rows = c_shape[0];
    if (cols > c_shape[1]) cols = c_shape[1];
    if (rows > a_shape[0] || rows > b_shape[0] || cols > a_shape[1] || cols > b_shape[1])
        return OR_ERR_ARG;
    for (int64_t r = 0; r < rows; ++r)
        for (int64_t q = 0; q < cols; ++q)
            c[r * c_strides[0] + q * c_strides[1]] =
                a[r * a_strides[0] + q * a_strides[1]] + b[r * b_strides[0] + q * b_strides[1]];
    return OR_OK;
}

/* ------------------------------------------------------------------------ */
/* matmul: tiled mmaf with an fp32 accumulator.                             */
/* ------------------------------------------------------------------------ */
/*
 * Per output element (m, n) the reference shader runs the outer K-tile loop
 * (materialize_for, tileops.hpp:859-1001; matmul.py:77-98) and inside it the
 * mmaf loop (materialize_mmaf_for, tileops.hpp:625-748) with
 *     acc = OpFAdd(acc, OpFMul(a, b))          (tileops.hpp:733-734)
 * for k ascending from acc = 0 (ct.full(..., 0), matmul.py:71).  Zero padding
 * of edge tiles (tileops.hpp:562-607) only appends +0 products, which leave
 * acc unchanged, so the result equals the plain k = 0..K-1 chain.  The
 * astype(tfloat32) / astype(C.dtype) casts lower to identity
 * (tileops.hpp:257-258), so fp32 inputs are used at full precision.
 *
 * fp16 / bf16 inputs (which the SPIR-V path cannot run: it is f32-only,
 * lower.hpp:197-209) follow the same chain on the exactly widened values.
 * An optional bias vector (length N) is added once after the K chain,
 * acc = fl(acc + bias[n]), and the sum is rounded to the output type.
 */

typedef struct {
    int in_dtype, out_dtype, bias_dtype;
    const void *a, *b, *bias;
    void *c;
    int64_t M, N, K;
    int64_t sa0, sa1, sb0, sb1, sc0, sc1;
    const float *bw; /* B widened to fp32, K x N row-major */
    int64_t row_begin, row_end;
    int err;
} mm_job;

static inline float load_elem(int dtype, const void *p, int64_t i) {
    switch (dtype) {
    case OR_F16: return or_f16_to_f32(((const uint16_t *)p)[i]);
    case OR_BF16: return or_bf16_to_f32(((const uint16_t *)p)[i]);
    default: return ((const float *)p)[i];
    }
}

static inline void store_elem(int dtype, void *p, int64_t i, float v) {
    switch (dtype) {
    case OR_F16: ((uint16_t *)p)[i] = or_f32_to_f16(v); break;
    case OR_BF16: ((uint16_t *)p)[i] = or_f32_to_bf16(v); break;
    default: ((float *)p)[i] = v; break;
    }
}

static void *mm_worker(void *arg) {
    mm_job *j = (mm_job *)arg;
    const int64_t N = j->N, K = j->K;
    float *acc = (float *)malloc((size_t)(N > 0 ? N : 1) * sizeof(float));
    float *arow = (float *)malloc((size_t)(K > 0 ? K : 1) * sizeof(float));
    if (!acc || !arow) {
        free(acc);
        free(arow);
        j->err = OR_ERR_MEM;
        return NULL;
    }
    for (int64_t m = j->row_begin; m < j->row_end; ++m) {
        for (int64_t k = 0; k < K; ++k) arow[k] = load_elem(j->in_dtype, j->a, m * j->sa0 + k * j->sa1);
        for (int64_t n = 0; n < N; ++n) acc[n] = 0.0f;
        for (int64_t k = 0; k < K; ++k) {
            const float av = arow[k];
            const float *brow = j->bw + k * N;
            /* one separately rounded multiply, then one add, per k step */
            for (int64_t n = 0; n < N; ++n) {
                float p = av * brow[n];
                acc[n] = acc[n] + p;
            }
        }
        if (j->bias)
            for (int64_t n = 0; n < N; ++n) acc[n] = acc[n] + load_elem(j->bias_dtype, j->bias, n);
        for (int64_t n = 0; n < N; ++n) store_elem(j->out_dtype, j->c, m * j->sc0 + n * j->sc1, acc[n]);
    }
    free(acc);
    free(arow);
    return NULL;
}

typedef struct {
    int dtype;
    const void *b;
    float *bw;
    int64_t K, N, sb0, sb1, k0, k1;
} widen_job;

static void *widen_worker(void *arg) {
    widen_job *w = (widen_job *)arg;
    for (int64_t k = w->k0; k < w->k1; ++k)
        for (int64_t n = 0; n < w->N; ++n) w->bw[k * w->N + n] = load_elem(w->dtype, w->b, k * w->sb0 + n * w->sb1);
    return NULL;
}

/*
 * C[row_begin:row_end, :] = A @ B (+ bias), rows split over nthreads
 * threads.  Strides are in elements.  Rows outside [row_begin, row_end) of
 * C are not touched.
 */
int or_matmul(int in_dtype, const void *a, int64_t sa0, int64_t sa1,
              const void *b, int64_t sb0, int64_t sb1,
              int bias_dtype, const void *bias,
              int out_dtype, void *c, int64_t sc0, int64_t sc1,
              int64_t M, int64_t N, int64_t K,
              int64_t row_begin, int64_t row_end, int nthreads) {
    if (M < 0 || N < 0 || K < 0 || row_begin < 0 || row_end > M || row_begin > row_end) return OR_ERR_ARG;
    if (in_dtype < OR_F32 || in_dtype > OR_BF16 || out_dtype < OR_F32 || out_dtype > OR_BF16) return OR_ERR_ARG;
    if (nthreads < 1) nthreads = 1;
    if (row_end == row_begin || N == 0) return OR_OK;

    float *bw = (float *)malloc((size_t)(K > 0 ? K : 1) * (size_t)N * sizeof(float));
    if (!bw) return OR_ERR_MEM;

    pthread_t *tid = (pthread_t *)calloc((size_t)nthreads, sizeof(pthread_t));
    widen_job *wj = (widen_job *)calloc((size_t)nthreads, sizeof(widen_job));
    mm_job *jobs = (mm_job *)calloc((size_t)nthreads, sizeof(mm_job));
    if (!tid || !wj || !jobs) {
        free(bw);
        free(tid);
        free(wj);
        free(jobs);
        return OR_ERR_MEM;
    }

    /* widen B once (exact conversion; it does not change any rounding) */
    int wt = nthreads;
    if (wt > K) wt = K > 0 ? (int)K : 1;
    for (int t = 0; t < wt; ++t) {
        wj[t] = (widen_job){in_dtype, b, bw, K, N, sb0, sb1, K * t / wt, K * (t + 1) / wt};
        if (pthread_create(&tid[t], NULL, widen_worker, &wj[t]) != 0) widen_worker(&wj[t]), tid[t] = 0;
    }
    for (int t = 0; t < wt; ++t)
        if (tid[t]) pthread_join(tid[t], NULL);

    int64_t rows = row_end - row_begin;
    int nt = nthreads;
    if (nt > rows) nt = (int)rows;
    for (int t = 0; t < nt; ++t) {
        mm_job *j = &jobs[t];
        j->in_dtype = in_dtype;
        j->out_dtype = out_dtype;
        j->bias_dtype = bias_dtype;
        j->a = a;
        j->b = b;
        j->bias = bias;
        j->c = c;
        j->M = M;
        j->N = N;
        j->K = K;
        j->sa0 = sa0;
        j->sa1 = sa1;
        j->sb0 = sb0;
        j->sb1 = sb1;
        j->sc0 = sc0;
        j->sc1 = sc1;
        j->bw = bw;
        j->row_begin = row_begin + rows * t / nt;
        j->row_end = row_begin + rows * (t + 1) / nt;
        j->err = OR_OK;
        tid[t] = 0;
        if (pthread_create(&tid[t], NULL, mm_worker, j) != 0) mm_worker(j), tid[t] = 0;
    }
    int err = OR_OK;
    for (int t = 0; t < nt; ++t) {
        if (tid[t]) pthread_join(tid[t], NULL);
        if (jobs[t].err) err = jobs[t].err;
    }
    free(bw);
    free(tid);
    free(wj);
    free(jobs);
    return err;
}

/*
 * Naive i-j-k fp32 matmul with `sum += a * b`, the CPU reference of the
 * reference's own matmul test (examples.cpp:533-551), row-major, contiguous.
 */
int or_reference_matmul_f32(const float *a, const float *b, float *c, int64_t m, int64_t n, int64_t k) {
    for (int64_t row = 0; row < m; ++row)
        for (int64_t col = 0; col < n; ++col) {
            float sum = 0.0f;
            for (int64_t kk = 0; kk < k; ++kk) sum += a[row * k + kk] * b[kk * n + col];
            c[row * n + col] = sum;
        }
    return OR_OK;
}

/* Tolerance check of the reference's tests: |lhs - rhs| <= 1e-3
 * (almost_equal, examples.cpp:450-452).  Returns the first failing index or
 * -1 when every element passes. */
int64_t or_first_mismatch_abs(const float *got, const float *want, int64_t count, float atol) {
    for (int64_t i = 0; i < count; ++i)
        if (!(fabsf(got[i] - want[i]) <= atol)) return i;
    return -1;
}

/* Known-answer generators of the reference's tests:
 *   vector_add: a[i] = i, b[i] = 1000 + i        (examples.cpp:477-480)
 *   matmul:     a[i] = ((i % 17) - 8) * 0.25     (examples.cpp:590-592)
 *               b[i] = ((i % 13) - 6) * 0.5      (examples.cpp:594-596)
 * (value = (i % modulus - offset) * scale). */
void or_kat_values(float *out, int64_t count, int64_t modulus, int64_t offset, float scale) {
    for (int64_t i = 0; i < count; ++i) out[i] = (float)((int32_t)(i % modulus) - (int32_t)offset) * scale;
}

void or_kat_iota(float *out, int64_t count, int64_t start) {
    for (int64_t i = 0; i < count; ++i) out[i] = (float)(start + i);
}

/* ------------------------------------------------------------------------ */
/* fma: elementwise fused multiply-add (tileops.hpp:616-623).               */
/* ------------------------------------------------------------------------ */

/*
 * C[i] = fma(A[i], B[i], D[i]) for i < min(grid_tiles * tile, C.size).  The
 * lowering emits GLSL.std.450 Fma (materialize_fma, tileops.hpp:616-623);
 * this restatement uses the IEEE-754 fused operation, a*b+d rounded once to
 * nearest even (C99 fmaf).  Tile coverage is that of the tile add.
 */
int or_vector_fma_1d(const float *a, int64_t a_size, int64_t a_stride, const float *b, int64_t b_size,
                     int64_t b_stride, const float *d, int64_t d_size, int64_t d_stride, float *c, int64_t c_size,
                     int64_t c_stride, int64_t tile, int64_t grid_tiles) {
    if (tile <= 0 || grid_tiles < 0) return OR_ERR_ARG;
    int64_t end = grid_tiles * tile;
    if (end > c_size) end = c_size;
    if (end > a_size || end > b_size || end > d_size) return OR_ERR_ARG;
    for (int64_t i = 0; i < end; ++i) c[i * c_stride] = fmaf(a[i * a_stride], b[i * b_stride], d[i * d_stride]);
    return OR_OK;
}

/* ------------------------------------------------------------------------ */
/* ftof: elementwise floating-point conversion (tileops.hpp:257-258).       */
/* ------------------------------------------------------------------------ */

/*
 * C[i] = (out type) A[i] for i < n, element strides in elements.  The
 * reference lowering passes ftof through unchanged (its path is f32-only,
 * tileops.hpp:257-258), which is the f32 -> f32 case here; the narrowing
 * conversions round to nearest even, widening ones are exact.
 */
int or_cast(int in_dtype, const void *a, int64_t a_stride, int out_dtype, void *c, int64_t c_stride, int64_t n) {
    if (in_dtype < OR_F32 || in_dtype > OR_BF16 || out_dtype < OR_F32 || out_dtype > OR_BF16 || n < 0)
        return OR_ERR_ARG;
    for (int64_t i = 0; i < n; ++i) store_elem(out_dtype, c, i * c_stride, load_elem(in_dtype, a, i * a_stride));
    return OR_OK;
}
