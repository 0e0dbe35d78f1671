// gemm.cu -- the tiled mmaf matmul on the sm_100a tensor cores.
//
// Reference semantics (src/tileops.hpp:625-748 with the K-tile loop of
// 859-1001, shaders/matmul.py:33-103): every output tile accumulates
// A_tile @ B_tile over all K tiles in fp32 starting from zero, edge tiles
// are zero padded, the accumulator is cast to C's type and stored with a
// bounds check.  Here the same contraction runs as one persistent,
// warp-specialised kernel per call:
//
//   warp 0      TMA producer: 128B-swizzled A and B tiles into a ring of
//               shared-memory stages (zero fill at the edges gives the
//               reference's padding for free)
//   warp 1      MMA issuer: tcgen05.mma (kind::f16 for f16/bf16, kind::tf32
//               for the 3xTF32 operands) into a TMEM accumulator; it also
//               owns the TMEM allocation
//   warps 2-5   epilogue: tcgen05.ld the accumulator, add the bias, convert,
//               store with the reference's bounds check
//
// The TMEM accumulator is double buffered (2 x BLOCK_N columns) so the
// epilogue of tile i overlaps the main loop of tile i+1.  Tiles are visited
// in the GROUP_SIZE_M = 8 raster of matmul.py:14-24 for L2 reuse.
// Every barrier wait is bounded; on time-out a role raises the CTA's abort
// flag, records an error code in the device error word and unwinds.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <type_traits>

#include "common.h"
#include "sm100.cuh"

namespace st {

int launch_c_init_f32(const GemmArgs &g, int sm_count, cudaStream_t stream);

// Tile raster of the cuTile matmul (matmul.py:14-24), shared by host and device.
__host__ __device__ __forceinline__ void tile_raster(int64_t num_m, int64_t num_n, int64_t group_m, int64_t bid,
                                                     int64_t &bm, int64_t &bn) {
    const int64_t in_group = group_m * num_n;
    const int64_t gid = bid / in_group;
    const int64_t first_m = gid * group_m;
    const int64_t rest = num_m - first_m;
    const int64_t gsz = rest < group_m ? rest : group_m;
    bm = first_m + (bid % gsz);
    bn = (bid % in_group) / gsz;
}

namespace {

constexpr int kBlockM = 128;
constexpr int kRowBytes = 128;  // K bytes per stage row = one 128-byte swizzle span
constexpr int kThreads = 192;   // 6 warps
constexpr int kEpilogueWarps = 4;
#ifndef ST_GROUP_M
#define ST_GROUP_M 8
#endif
#ifndef ST_C_STORE_DEFAULT
#define ST_C_STORE_DEFAULT 1  // local C: 1 TMA-store epilogue, 0 per-lane direct stores
#endif
#ifndef ST_C_POLICY
#define ST_C_POLICY 0  // C stores: 0 default, 1 L2 evict_first
#endif
constexpr int kGroupM = ST_GROUP_M;

// C staging for the TMA-store epilogue: per epilogue warp two buffers of one
// 32-row x 128-byte box (32 fp32 or 64 16-bit columns), 128-byte swizzled.
constexpr int kStageBoxBytes = 32 * 128;
constexpr int kCStagingBytes = kEpilogueWarps * 2 * kStageBoxBytes;
constexpr int kBarRegion = 1024;  // barriers + TMEM slot + abort flag; keeps the staging 1024-aligned

template <int BN>
struct TileCfg {
    static constexpr int kABytes = kBlockM * kRowBytes;
    static constexpr int kBBytes = BN * kRowBytes;
    static constexpr int kStageBytes = kABytes + kBBytes;
    static constexpr int kStages = BN == 256 ? 4 : (BN == 128 ? 6 : 8);
    static constexpr int kTmemCols = 2 * BN;  // two accumulators; 128, 256 or 512 (powers of two)
    static constexpr int kSmemBytes = kStages * kStageBytes + kBarRegion + kCStagingBytes + 1024;  // + alignment slack
    static_assert(kSmemBytes <= 232448, "over the per-block shared memory limit");
};

struct KParams {
    int m, n, k;
    int num_m_tiles, num_n_tiles, num_k_blocks, total_tiles;
    float *sk_ws;    // stream-K partials (CTA-pair kernel); null: whole tiles only
    int sk_mode;     // stream_k_split mode
    int *sk_flags;   // per (pair, CTA, epilogue warp): partials stored and not yet folded
    // split tiles of an fp32 C fold in L2: 1 every unit TMA-reduce-adds its
    // partial onto C preset to the bias; 2 (ordered) a tile's first unit
    // stores its partial plus the bias outright and raises its flags, the
    // tile's other units add onto that once the flags are up (no preset)
    int sk_l2add;
    int k_snake;     // 1: a CTA's (pair's) odd-numbered whole tiles load their K blocks last to first
    void *c;
    void *c_peers[kMaxPeers];  // the same rows of C in other GPUs' copies (may be empty)
    int n_peers;
    int staged;  // 1: C leaves through shared memory and TMA stores (CStoreMaps), 0: direct stores
    long long ldc;
    int c_dtype;
    const void *bias;
    int bias_dtype;
    int *err;
    unsigned long long timeout_ns;
};

__device__ __forceinline__ float load_bias(const void *bias, int dtype, int i) {
    if (dtype == ST_F32) return static_cast<const float *>(bias)[i];
    if (dtype == ST_F16) return __half2float(static_cast<const __half *>(bias)[i]);
    return __bfloat162float(static_cast<const __nv_bfloat16 *>(bias)[i]);
}

// Add the bias of columns [col0, col0 + 32) to one accumulator chunk.  Lane
// l loads the bias of column col0 + l (one coalesced load per warp) and the
// values reach every lane by shuffle.  Called by all 32 lanes; columns past
// N get 0 and are never stored.
__device__ __forceinline__ void add_bias_chunk(const KParams &p, int col0, int lane, uint32_t (&r)[32]) {
    const int col = col0 + lane;
    const float mine = col < p.n ? load_bias(p.bias, p.bias_dtype, col) : 0.0f;
#pragma unroll
    for (int j = 0; j < 32; ++j)
        r[j] = __float_as_uint(__fadd_rn(__uint_as_float(r[j]), __shfl_sync(0xffffffffu, mine, j)));
}

// Store 32 accumulator columns [col0, col0+32) of one row (bias already
// added): conversion once, then the same bytes to this GPU's C and to every
// peer copy.
__device__ __forceinline__ void store_row_chunk(const KParams &p, int row, int col0, const uint32_t (&r)[32]) {
    float v[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
    const int cnt = p.n - col0 < 32 ? p.n - col0 : 32;
    const long long off = static_cast<long long>(row) * p.ldc + col0;
    if (p.c_dtype == ST_F32) {
        for (int d = -1; d < p.n_peers; ++d) {
            float *dst = static_cast<float *>(d < 0 ? p.c : p.c_peers[d]) + off;
            if (cnt == 32 && (reinterpret_cast<uintptr_t>(dst) & 15u) == 0) {
#if ST_C_POLICY == 1
                const uint64_t pol = l2_policy_evict_first();
#pragma unroll
                for (int j = 0; j < 32; j += 4)
                    asm volatile("st.global.L2::cache_hint.v4.f32 [%0], {%1, %2, %3, %4}, %5;" ::"l"(dst + j),
                                 "f"(v[j]), "f"(v[j + 1]), "f"(v[j + 2]), "f"(v[j + 3]), "l"(pol)
                                 : "memory");
#else
#pragma unroll
                for (int j = 0; j < 32; j += 4)
                    *reinterpret_cast<float4 *>(dst + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
#endif
            } else {
#pragma unroll
                for (int j = 0; j < 32; ++j)
                    if (j < cnt) dst[j] = v[j];
            }
        }
        return;
    }
    uint16_t h[32];
    if (p.c_dtype == ST_F16) {
#pragma unroll
        for (int j = 0; j < 32; ++j) h[j] = __half_as_ushort(__float2half_rn(v[j]));
    } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) h[j] = __bfloat16_as_ushort(__float2bfloat16_rn(v[j]));
    }
    uint4 q[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        q[j].x = h[8 * j] | (static_cast<uint32_t>(h[8 * j + 1]) << 16);
        q[j].y = h[8 * j + 2] | (static_cast<uint32_t>(h[8 * j + 3]) << 16);
        q[j].z = h[8 * j + 4] | (static_cast<uint32_t>(h[8 * j + 5]) << 16);
        q[j].w = h[8 * j + 6] | (static_cast<uint32_t>(h[8 * j + 7]) << 16);
    }
    for (int d = -1; d < p.n_peers; ++d) {
        uint16_t *dst = static_cast<uint16_t *>(d < 0 ? p.c : p.c_peers[d]) + off;
        if (cnt == 32 && (reinterpret_cast<uintptr_t>(dst) & 15u) == 0) {
#pragma unroll
            for (int j = 0; j < 4; ++j) reinterpret_cast<uint4 *>(dst)[j] = q[j];
        } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
                if (j < cnt) dst[j] = h[j];
        }
    }
}

// Tensor maps of the TMA-store epilogue: [0] this GPU's C, [1 + d] peer copy d.
// Box = 32 rows x 128 bytes, 128-byte swizzle; extents = this call's C rows x N.
struct CStoreMaps {
    CUtensorMap map[1 + kMaxPeers];
};

// One 128-byte row per lane of a 32-row staging box in the 128-byte swizzle
// (16-byte chunk j of row l at j ^ (l mod 8): conflict-free for a warp).
__device__ __forceinline__ void box_put_row(uint32_t box, int lane, const uint32_t (&w)[32]) {
    const uint32_t row_addr = box + static_cast<uint32_t>(lane * 128);
#pragma unroll
    for (int q = 0; q < 8; ++q) {
        const uint32_t a = row_addr + (static_cast<uint32_t>(q ^ (lane & 7)) << 4);
        asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(w[4 * q]), "r"(w[4 * q + 1]),
                     "r"(w[4 * q + 2]), "r"(w[4 * q + 3])
                     : "memory");
    }
}

__device__ __forceinline__ void box_get_row(uint32_t box, int lane, uint32_t (&w)[32]) {
    const uint32_t row_addr = box + static_cast<uint32_t>(lane * 128);
#pragma unroll
    for (int q = 0; q < 8; ++q) {
        const uint32_t a = row_addr + (static_cast<uint32_t>(q ^ (lane & 7)) << 4);
        asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                     : "=r"(w[4 * q]), "=r"(w[4 * q + 1]), "=r"(w[4 * q + 2]), "=r"(w[4 * q + 3])
                     : "r"(a)
                     : "memory");
    }
}

// One tile's worth of a warp's 32 accumulator rows (TMEM lanes at t_row,
// columns [n0, n0 + NCOLS)) through shared memory: bias add and conversion,
// one 128-byte row per lane written into a swizzled staging box, then one
// TMA store of the box to C and to every peer copy.  The two staging buffers
// alternate; before reusing one, lane 0 waits until the store issued from it
// has finished reading shared memory.  TMA clips the box at C's extents.
template <int NCOLS>
__device__ __forceinline__ void store_tile_staged(const KParams &p, const CStoreMaps &cm, uint32_t t_row, int row0,
                                                  int n0, uint32_t staging, int &buf, int lane, int c_begin = 0,
                                                  int c_end = NCOLS, bool reduce = false) {
    if (row0 >= p.m) return;
    const bool f32 = p.c_dtype == ST_F32;
    const int box_cols = f32 ? 32 : 64;
#pragma unroll 1
    for (int c0 = c_begin; c0 < c_end; c0 += box_cols) {
        const int col0 = n0 + c0;
        if (col0 >= p.n) break;
        uint32_t w[32];  // this lane's 128-byte row of the box
        if (f32) {
            tmem_load_32(t_row + c0, w);
            tmem_load_wait();
            if (p.bias != nullptr && !reduce) add_bias_chunk(p, col0, lane, w);
        } else {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                uint32_t r[32];
                tmem_load_32(t_row + c0 + 32 * h, r);
                tmem_load_wait();
                if (p.bias != nullptr) add_bias_chunk(p, col0 + 32 * h, lane, r);
#pragma unroll
                for (int j = 0; j < 32; j += 2) {
                    const float v0 = __uint_as_float(r[j]), v1 = __uint_as_float(r[j + 1]);
                    uint32_t lo, hi;
                    if (p.c_dtype == ST_F16) {
                        lo = __half_as_ushort(__float2half_rn(v0));
                        hi = __half_as_ushort(__float2half_rn(v1));
                    } else {
                        lo = __bfloat16_as_ushort(__float2bfloat16_rn(v0));
                        hi = __bfloat16_as_ushort(__float2bfloat16_rn(v1));
                    }
                    w[16 * h + j / 2] = lo | (hi << 16);
                }
            }
        }
        if (lane == 0) bulk_wait_group_read<1>();  // the store that last used this buffer is done reading it
        __syncwarp();
        const uint32_t box = staging + static_cast<uint32_t>(buf * kStageBoxBytes);
        box_put_row(box, lane, w);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
            if (reduce) {  // fp32, this GPU's C only
                tma_reduce_add_2d(&cm.map[0], box, col0, row0);
            } else {
#if ST_C_POLICY == 1
                const uint64_t pol = l2_policy_evict_first();
                for (int d = 0; d <= p.n_peers; ++d) tma_store_2d_hint(&cm.map[d], box, col0, row0, pol);
#else
                for (int d = 0; d <= p.n_peers; ++d) tma_store_2d(&cm.map[d], box, col0, row0);
#endif
            }
            bulk_commit_group();
        }
        buf ^= 1;
    }
}

// After a CTA's last peer store: make its NVLink writes visible system-wide
// before the kernel counts as complete.
__device__ __forceinline__ void publish_peer_writes(const KParams &p) {
    if (p.n_peers > 0) __threadfence_system();
}

// FMT: 0 = f16, 1 = bf16, 2 = tf32.  B_MN: B tiles are N-contiguous.
template <int FMT, bool B_MN, int BN>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                   const KParams p, const __grid_constant__ CStoreMaps cmaps) {
    using Cfg = TileCfg<BN>;
    constexpr bool kTf32 = FMT == 2;
    constexpr int kElem = kTf32 ? 4 : 2;
    constexpr int kBK = kRowBytes / kElem;  // K elements per stage
    constexpr int kMmaK = 32 / kElem;       // K elements per tcgen05.mma
    constexpr int kKSteps = kBK / kMmaK;
    constexpr uint32_t kIdesc = mma_idesc(FMT, false, B_MN, kBlockM, BN);
    static_assert(!(kTf32 && B_MN), "tf32 operands are packed K-major");

    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + Cfg::kStages * Cfg::kStageBytes);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 2 * Cfg::kStages + 5);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t bar0 = smem_addr(bars);
    auto full_bar = [&](int s) { return bar0 + 8u * s; };
    auto empty_bar = [&](int s) { return bar0 + 8u * (Cfg::kStages + s); };
    auto tfull_bar = [&](int a) { return bar0 + 8u * (2 * Cfg::kStages + a); };
    auto tempty_bar = [&](int a) { return bar0 + 8u * (2 * Cfg::kStages + 2 + a); };
    const uint32_t drain_bar = bar0 + 8u * (2 * Cfg::kStages + 4);

    if (threadIdx.x == 0) {
        for (int s = 0; s < Cfg::kStages; ++s) {
            mbar_init(full_bar(s), 1);
            mbar_init(empty_bar(s), 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(tfull_bar(a), 1);
            mbar_init(tempty_bar(a), kEpilogueWarps);
        }
        mbar_init(drain_bar, 1);
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_map(&tmap_a);
        tma_prefetch_map(&tmap_b);
    }
    if (warp == 1) {
        tmem_alloc(smem_addr(tmem_slot), Cfg::kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before_sync();
    __syncthreads();
    tc_fence_after_sync();
    const uint32_t tmem_base = *tmem_slot;
    pdl_begin();  // nothing above touches global memory

    if (warp == 0) {
        // ------------------------------------------------ TMA producer
        if (lane == 0) {
            const uint64_t pol_a = l2_policy_evict_last();
            const uint64_t pol_b = l2_policy_evict_last();
            int s = 0;
            uint32_t ph = 0;
            uint32_t pending = 0;        // stages with a load in flight that nobody consumed yet
            uint32_t pending_ph = 0;     // parity each pending load completes with
            bool ok = true;
            for (int t = blockIdx.x; ok && t < p.total_tiles; t += gridDim.x) {
                int64_t tm, tn;
                tile_raster(p.num_m_tiles, p.num_n_tiles, kGroupM, t, tm, tn);
                const int m0 = static_cast<int>(tm) * kBlockM;
                const int n0 = static_cast<int>(tn) * BN;
                // k_snake: this CTA's odd-numbered tiles load K last to first, so a
                // tile starts on the K blocks its predecessor read last, while they
                // are still in L2 (the MMA only counts blocks; the sum order changes)
                const bool rev = p.k_snake && ((t - static_cast<int>(blockIdx.x)) / static_cast<int>(gridDim.x)) & 1;
                for (int kb = 0; kb < p.num_k_blocks; ++kb) {
                    if (!mbar_wait(empty_bar(s), ph ^ 1u, abort_flag, p.timeout_ns)) {
                        ok = false;
                        break;
                    }
                    pending &= ~(1u << s);
                    const uint32_t sa = smem_addr(smem + s * Cfg::kStageBytes);
                    const uint32_t sb = sa + Cfg::kABytes;
                    const int kx = (rev ? p.num_k_blocks - 1 - kb : kb) * kBK;
                    mbar_arrive_expect_tx(full_bar(s), Cfg::kStageBytes);
                    tma_load_2d(sa, &tmap_a, full_bar(s), kx, m0, pol_a);
                    if constexpr (B_MN) {
#pragma unroll
                        for (int j = 0; j < BN / 64; ++j)
                            tma_load_2d(sb + j * (kBK * 128), &tmap_b, full_bar(s), n0 + 64 * j, kx, pol_b);
                    } else {
                        tma_load_2d(sb, &tmap_b, full_bar(s), kx, n0, pol_b);
                    }
                    pending |= 1u << s;
                    pending_ph = (pending_ph & ~(1u << s)) | (ph << s);
                    if (++s == Cfg::kStages) {
                        s = 0;
                        ph ^= 1u;
                    }
                }
            }
            if (!ok) {
                *abort_flag = 1;
                atomicExch(p.err, kDevAbortGemmProducer);
                // let the loads already in flight land before the CTA exits
                for (int q = 0; q < Cfg::kStages; ++q)
                    if (pending & (1u << q))
                        (void)mbar_wait(full_bar(q), (pending_ph >> q) & 1u, abort_flag, p.timeout_ns);
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer
        if (lane == 0) {
            int s = 0;
            uint32_t ph = 0;
            int iter = 0;
            bool ok = true;
            for (int t = blockIdx.x; ok && t < p.total_tiles; t += gridDim.x, ++iter) {
                const int acc = iter & 1;
                const uint32_t acc_ph = static_cast<uint32_t>(iter >> 1) & 1u;
                if (!mbar_wait(tempty_bar(acc), acc_ph ^ 1u, abort_flag, p.timeout_ns)) {
                    ok = false;
                    break;
                }
                tc_fence_after_sync();
                const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
                for (int kb = 0; kb < p.num_k_blocks; ++kb) {
                    if (!mbar_wait(full_bar(s), ph, abort_flag, p.timeout_ns)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after_sync();
                    const uint32_t sa = smem_addr(smem + s * Cfg::kStageBytes);
                    const uint32_t sb = sa + Cfg::kABytes;
#pragma unroll
                    for (int ks = 0; ks < kKSteps; ++ks) {
                        // K-major operand: advance 32 bytes of K inside the swizzle row
                        const uint64_t adesc = smem_desc_sw128(sa + ks * 32, 16, 1024);
                        uint64_t bdesc;
                        if constexpr (B_MN) {
                            // N-contiguous operand: LBO = next 64-column chunk, SBO = next 8 K rows
                            bdesc = smem_desc_sw128(sb + ks * (kMmaK * 128), kBK * 128, 1024);
                        } else {
                            bdesc = smem_desc_sw128(sb + ks * 32, 16, 1024);
                        }
                        tc_mma<kTf32>(d_tmem, adesc, bdesc, kIdesc, (kb | ks) != 0 ? 1u : 0u);
                    }
                    tc_commit(empty_bar(s));  // frees the stage when these MMAs retire
                    if (++s == Cfg::kStages) {
                        s = 0;
                        ph ^= 1u;
                    }
                }
                if (!ok) break;
                tc_commit(tfull_bar(acc));  // accumulator complete
            }
            if (!ok) {
                *abort_flag = 1;
                atomicExch(p.err, kDevAbortGemmMma);
            }
            // all MMAs issued by this thread have retired once drain_bar flips
            tc_commit(drain_bar);
            (void)mbar_wait(drain_bar, 0, abort_flag, p.timeout_ns);
        }
    } else {
        // ------------------------------------------------ epilogue (warps 2..5)
        const int g = warp & 3;  // TMEM lanes 32g..32g+31 are the ones this warp may read
        const uint32_t staging = smem_addr(smem + Cfg::kStages * Cfg::kStageBytes + kBarRegion) +
                                 static_cast<uint32_t>(g * 2 * kStageBoxBytes);
        int sbuf = 0;
        int iter = 0;
        for (int t = blockIdx.x; t < p.total_tiles; t += gridDim.x, ++iter) {
            const int acc = iter & 1;
            const uint32_t acc_ph = static_cast<uint32_t>(iter >> 1) & 1u;
            int64_t tm, tn;
            tile_raster(p.num_m_tiles, p.num_n_tiles, kGroupM, t, tm, tn);
            const int m0 = static_cast<int>(tm) * kBlockM;
            const int n0 = static_cast<int>(tn) * BN;
            const bool ready = mbar_wait(tfull_bar(acc), acc_ph, abort_flag, p.timeout_ns);
            if (!__all_sync(0xffffffffu, ready)) {
                *abort_flag = 1;
                if (lane == 0) atomicExch(p.err, kDevAbortGemmEpilogue);
                break;
            }
            tc_fence_after_sync();
            const int row = m0 + g * 32 + lane;
            const uint32_t t_row = tmem_base + (static_cast<uint32_t>(g * 32) << 16) + static_cast<uint32_t>(acc * BN);
            if (p.staged) {
                store_tile_staged<BN>(p, cmaps, t_row, m0 + g * 32, n0, staging, sbuf, lane);
            } else {
#pragma unroll 1
                for (int c = 0; c < BN / 32; ++c) {
                    const int col0 = n0 + c * 32;
                    if (col0 >= p.n) break;
                    uint32_t r[32];
                    tmem_load_32(t_row + c * 32, r);
                    tmem_load_wait();
                    if (p.bias != nullptr) add_bias_chunk(p, col0, lane, r);
                    if (row < p.m) store_row_chunk(p, row, col0, r);
                }
            }
            tc_fence_before_sync();
            __syncwarp();
            if (lane == 0) mbar_arrive(tempty_bar(acc));
        }
        if (p.staged && lane == 0) bulk_wait_group_all();  // every TMA store of C has landed
    }

    publish_peer_writes(p);
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after_sync();
        tmem_dealloc(tmem_base, Cfg::kTmemCols);
    }
}

// ---------------------------------------------------------------- CTA-pair kernel
// Two CTAs of a cluster (one TPC) share one 256 x 256 output tile: each
// stages 128 rows of A and 128 columns of B per K step, and the even CTA
// issues tcgen05.mma.cta_group::2, which reads both CTAs' shared memory and
// writes rows 0-127 of the accumulator into its own TMEM and rows 128-255
// into its partner's.  Per SM this halves the B bytes staged and read per
// MMA compared with the one-CTA kernel.
//
// Signalling between the two CTAs (no multicast anywhere):
//   full[s]   lives in the even CTA; both CTAs' TMA loads complete on it
//             (cta_group::2 form), the even producer arrives with the
//             pair's byte count.
//   empty[s]  the even CTA's MMA commit frees its own stage; its producer,
//             having seen that, arrives remotely on the odd CTA's empty[s].
//   tfull[a]  the commit completes the even CTA's barrier; its first
//             epilogue warp forwards it to the odd CTA's tfull[a].
//   tempty[a] lives in the even CTA and counts all 8 epilogue warps of the
//             pair (the odd CTA's arrive remotely).
constexpr int kPairN = 256;      // N of one pair MMA
constexpr int kPairHalfN = 128;  // columns of B each CTA stages

#ifndef ST_PAIR_STAGES
#define ST_PAIR_STAGES 6
#endif
#ifndef ST_L2_POLICY
// operand loads: 0 evict_normal, 1 evict_last, 2 A evict_last and B evict_first,
// 3 A evict_last and B evict_normal
#define ST_L2_POLICY 1
#endif

#if ST_L2_POLICY == 0 || ST_L2_POLICY == 3
__device__ __forceinline__ uint64_t l2_policy_evict_normal() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(p));
    return p;
}
#endif

__device__ __forceinline__ uint64_t operand_l2_policy_a() {
#if ST_L2_POLICY == 0
    return l2_policy_evict_normal();
#else
    return l2_policy_evict_last();
#endif
}

__device__ __forceinline__ uint64_t operand_l2_policy_b() {
#if ST_L2_POLICY == 0 || ST_L2_POLICY == 3
    return l2_policy_evict_normal();
#elif ST_L2_POLICY == 2
    return l2_policy_evict_first();
#else
    return l2_policy_evict_last();
#endif
}

// ---- work of one CTA pair: whole tiles, then a stream-K tail
//
// With T tiles, P pairs and KB K blocks per tile, tiles go out whole in the
// strided order (tile t to pair t mod P), which keeps the pairs on
// neighbouring tiles of the raster for L2 reuse.  With fewer tiles than pairs
// (T < P) that would leave P - T pairs idle; instead the T * KB K blocks are
// split into equal contiguous ranges over S > T pairs (at least KB / 4 blocks
// each, so a tile has at most ~5 units).  The split is written for a tail
// after whole-tile waves too (dp_tiles > 0).  A split tile's units finish
// together and reduce-scatter: each publishes the output columns the others
// own (fp32, without waiting), then waits for the others' parts of its own
// columns, adds them and stores those columns of C.  No unit waits before
// every unit of its pair has published, and the grid never exceeds the
// co-resident clusters, so the waits end.  Where every tile is split and C is
// fp32 on this GPU only (sk_l2add), there is no exchange: each unit adds its
// whole partial tile onto C with TMA reduce-adds, which L2 performs (the
// order of the units' adds, and so the last bit of a sum, can differ between
// runs).  With stream-K flags (ordered mode) a tile's first unit -- the one
// holding its K block 0, always the first split unit of its pair, which
// never waits -- stores its partial plus the bias outright and raises one
// flag per (CTA, epilogue warp) by the number of other units; each other
// unit's warp waits (bounded) for the flag of its own rows, takes one count
// off it and adds.  Without flags C is preset to the bias on the split
// tiles first.  Stream-K index q = P - 1 - pair.
enum : int { kUnitWhole = 0, kUnitSplit = 1 };

struct PairWork {
    int tile, k0, k1, kind;
};

// mode 0: whole tiles only; 1: split when there are fewer tiles than pairs;
// 2: also split the partial last wave after whole-tile waves (when its idle
// pairs cost >= 3 % of the launch)
__host__ __device__ __forceinline__ void stream_k_split(int total, int num_pairs, int kb, int mode, int &dp_tiles,
                                                        int &sk_pairs, long long &sk_iters) {
    dp_tiles = total;
    sk_pairs = 0;
    sk_iters = 0;
    if (mode <= 0 || num_pairs <= 0 || total == 0 || kb < 8) return;
    if (total >= num_pairs && mode < 2) return;
    const int r = total % num_pairs;
    if (r == 0) return;
    const long long full = total / num_pairs;
    if (full > 0 && static_cast<long long>(num_pairs - r) * 100 < 3LL * num_pairs * (full + 1)) return;
    const long long iters = static_cast<long long>(r) * kb;
    const long long per = kb / 4 > 4 ? kb / 4 : 4;
    long long s = iters / per;
    if (s > num_pairs) s = num_pairs;
    if (s <= r) return;  // no better than one whole tile on each of r pairs
    dp_tiles = total - r;
    sk_pairs = static_cast<int>(s);
    sk_iters = iters;
}

struct PairSchedule {
    int num_pairs, kb, dp_tiles, sk_pairs, sk_index;
    long long sk_iters;
    __device__ __forceinline__ void init(const KParams &p, int pair, int num_pairs_, int total) {
        num_pairs = num_pairs_;
        kb = p.num_k_blocks;
        const bool can_fold = p.sk_ws != nullptr || p.sk_l2add != 0;
        stream_k_split(total, num_pairs, kb, can_fold ? p.sk_mode : 0, dp_tiles, sk_pairs, sk_iters);
        sk_index = num_pairs - 1 - pair;
    }
    __device__ __forceinline__ long long sk_begin(int q) const {
        return static_cast<long long>(q) * sk_iters / sk_pairs;
    }
};

// A pair's units in MMA order.  A stream-K range is at most one tile long
// (r < P tiles over P pairs, or at most 2 * (kb / 4) blocks each), so it is
// one unit or two: the end of tile s and the start of tile s + 1.  The
// start of tile s + 1 goes first, so that every pair starts
// its range at K block 0 and ends it at the last K block: the pairs sweep
// the tiles' K blocks together, which keeps A and B reads shared in L2.
struct PairUnits {
    int t;       // next whole tile
    int n, i;    // stream-K units of this pair and the next one to hand out
    PairWork u0, u1;
    __device__ __forceinline__ void init(const PairSchedule &s, int pair) {
        t = pair;
        n = i = 0;
        if (s.sk_index >= s.sk_pairs) return;
        const long long a = s.sk_begin(s.sk_index), b = s.sk_begin(s.sk_index + 1);
        if (b <= a) return;
        const long long sa = a / s.kb, sb = (b - 1) / s.kb;
        auto unit = [&](long long tile_rel, long long lo, long long hi) {
            PairWork w;
            w.tile = s.dp_tiles + static_cast<int>(tile_rel);
            w.k0 = static_cast<int>(lo - tile_rel * s.kb);
            w.k1 = static_cast<int>(hi - tile_rel * s.kb);
            w.kind = (w.k0 > 0 || w.k1 < s.kb) ? kUnitSplit : kUnitWhole;
            return w;
        };
        if (sa == sb) {
            u0 = unit(sa, a, b);
            n = 1;
        } else {  // sb == sa + 1: the start of tile sb first, then the end of tile sa
            u0 = unit(sb, sb * s.kb, b);
            u1 = unit(sa, a, sb * s.kb);
            n = 2;
        }
    }
    __device__ __forceinline__ bool next(const PairSchedule &s, PairWork &w) {
        if (t < s.dp_tiles) {
            w = PairWork{t, 0, s.kb, kUnitWhole};
            t += s.num_pairs;
            return true;
        }
        if (i >= n) return false;
        w = i == 0 ? u0 : u1;
        ++i;
        return true;
    }
};

// A split unit's partial accumulator in the workspace: per (slot, CTA rank,
// epilogue warp g) 8 boxes of 4 KB; box c holds accumulator columns [32c, 32c + 32) of the
// warp's 32 rows in the staging layout (one 128-byte row per lane, 16-byte
// chunk j of row l at position j ^ (l mod 8)).
constexpr int kSkBoxes = 256 / 32;
constexpr int kLandBoxes = 12;  // 48 KB of the operand ring per epilogue warp

// Workspace slot of the unit of stream-K index q that covers tile `rel` (0-based
// among the split tiles): a range covers at most two tiles, so each index
// owns slots 2q (the tile its range starts in) and 2q + 1 (the next one).
__device__ __forceinline__ int sk_slot(const PairSchedule &s, int q, long long rel) {
    return 2 * q + (rel == s.sk_begin(q) / s.kb ? 0 : 1);
}

__device__ __forceinline__ uint8_t *sk_box(const KParams &p, int slot, uint32_t rank, int g, int c) {
    const size_t box = ((static_cast<size_t>(slot) * 2 + rank) * kEpilogueWarps + g) * kSkBoxes + c;
    return reinterpret_cast<uint8_t *>(p.sk_ws) + box * kStageBoxBytes;
}

__device__ __forceinline__ int *sk_flag(const KParams &p, int slot, uint32_t rank, int g) {
    return p.sk_flags + (slot * 2 + static_cast<int>(rank)) * kEpilogueWarps + g;
}

// The units of one split tile: stream-K slots q0 .. q0 + n - 1 hold its K
// blocks in order; this unit is number j.  The tile's output boxes (8 of 32
// fp32 columns, or 4 of 64 16-bit columns, per row quarter) are divided
// among the units: unit j reduces and stores boxes [nb j / n, nb (j + 1) / n).
struct SplitTile {
    int q0, n, j;
    long long rel;       // the tile among the split tiles
    int c_begin, c_end;  // this unit's own accumulator columns [c_begin, c_end)
};

__device__ __forceinline__ SplitTile split_tile(const KParams &p, const PairSchedule &s, const PairWork &w) {
    const long long tile_start = static_cast<long long>(w.tile - s.dp_tiles) * s.kb, tile_end = tile_start + s.kb;
    int q0 = s.sk_index;
    while (q0 > 0 && s.sk_begin(q0) > tile_start) --q0;
    int q1 = s.sk_index + 1;
    while (q1 < s.sk_pairs && s.sk_begin(q1) < tile_end) ++q1;
    SplitTile t;
    t.q0 = q0;
    t.n = q1 - q0;
    t.j = s.sk_index - q0;
    t.rel = w.tile - s.dp_tiles;
    const int nb = p.c_dtype == ST_F32 ? 8 : 4, box_cols = 256 / nb;
    t.c_begin = nb * t.j / t.n * box_cols;
    t.c_end = nb * (t.j + 1) / t.n * box_cols;
    return t;
}

// Reduce-scatter, step 1 (never waits): this warp's 32 accumulator rows of
// every column chunk outside the unit's own range leave as fp32 through the
// staging boxes and bulk stores to the unit's workspace slot; once they have
// landed the warp's flag is raised by n - 1 (one per reader, release).
__device__ __forceinline__ void sk_publish(const KParams &p, const PairSchedule &s, const SplitTile &t,
                                           uint32_t rank, int g, int lane, uint32_t t_row, uint32_t staging,
                                           int &buf) {
    const int slot = sk_slot(s, t.q0 + t.j, t.rel);
#pragma unroll 1
    for (int c = 0; c < kSkBoxes; ++c) {
        if (c * 32 >= t.c_begin && c * 32 < t.c_end) continue;
        uint32_t r[32];
        tmem_load_32(t_row + c * 32, r);
        tmem_load_wait();
        if (lane == 0) bulk_wait_group_read<1>();  // the store that last used this buffer is done reading it
        __syncwarp();
        const uint32_t box = staging + static_cast<uint32_t>(buf * kStageBoxBytes);
        box_put_row(box, lane, r);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
            bulk_store(sk_box(p, slot, rank, g, c), box, kStageBoxBytes);
            bulk_commit_group();
        }
        buf ^= 1;
    }
    if (lane == 0) {
        bulk_wait_group_all();  // the chunks are in global memory
        fence_proxy_async_global();
        red_release_gpu_add(sk_flag(p, slot, rank, g), t.n - 1);
    }
    __syncwarp();
}

// Reduce-scatter, step 2a: wait (bounded) until every other unit of the
// pair's split tiles (at most 2 x 5 flags) has published.  Lane l polls flag
// l, so each pass is one round trip for all of them; the warp barrier at the
// end orders lane 0's later bulk loads after every lane's acquire.
__device__ __forceinline__ bool sk_wait_others(const KParams &p, const PairSchedule &s, const SplitTile *t, int nt,
                                               uint32_t rank, int g, int lane, const volatile int *abort_flag) {
    const int *mine = nullptr;
    int l = 0;
    for (int u = 0; u < nt; ++u)
        for (int i = 0; i < t[u].n; ++i) {
            if (i == t[u].j) continue;
            if (l == lane) mine = sk_flag(p, sk_slot(s, t[u].q0 + i, t[u].rel), rank, g);
            ++l;
        }
    const uint64_t t0 = global_timer_ns();
    for (;;) {
        const bool here = mine == nullptr || ld_acquire_gpu(mine) >= 1;
        if (__all_sync(0xffffffffu, here)) break;
        if (__any_sync(0xffffffffu, *abort_flag != 0 || global_timer_ns() - t0 > p.timeout_ns)) return false;
    }
    __syncwarp();
    return true;
}

__device__ __forceinline__ int sk_land_boxes(const SplitTile &t) { return (t.c_end - t.c_begin) / 32 * (t.n - 1); }

// Step 2b: bulk-load the other units' boxes of the own columns of split
// units [u0, u1) into `land` (the idle operand ring), add them in slot order
// to this warp's accumulator rows in TMEM.  False when a load did not land
// in time.
__device__ __forceinline__ bool sk_land_and_add(const KParams &p, const PairSchedule &s, const SplitTile *t,
                                                const uint32_t *t_row, int u0, int u1, uint32_t rank, int g,
                                                int lane, uint32_t land, uint32_t fold_bar, uint32_t &phase,
                                                const volatile int *abort_flag) {
    int boxes = 0;
    for (int u = u0; u < u1; ++u) boxes += sk_land_boxes(t[u]);
    if (boxes == 0) return true;
    if (boxes > kLandBoxes) return false;  // cannot happen: one unit lands <= 12 boxes
    if (lane == 0) {
        fence_proxy_async_global();  // the acquired flags come before these async-proxy reads
        mbar_arrive_expect_tx(fold_bar, static_cast<uint32_t>(boxes * kStageBoxBytes));
        int b = 0;
        for (int u = u0; u < u1; ++u)
            for (int c = t[u].c_begin / 32; c < t[u].c_end / 32; ++c)
                for (int i = 0; i < t[u].n; ++i) {
                    if (i == t[u].j) continue;
                    bulk_load(land + static_cast<uint32_t>(b++ * kStageBoxBytes),
                              sk_box(p, sk_slot(s, t[u].q0 + i, t[u].rel), rank, g, c), kStageBoxBytes, fold_bar);
                }
    }
    const bool landed = mbar_wait(fold_bar, phase, abort_flag, p.timeout_ns);
    if (!__all_sync(0xffffffffu, landed)) return false;
    phase ^= 1u;
    int b = 0;
    for (int u = u0; u < u1; ++u) {
        const int others = t[u].n - 1;
#pragma unroll 1
        for (int c = t[u].c_begin / 32; c < t[u].c_end / 32; ++c) {
            uint32_t r[32];
            tmem_load_32(t_row[u] + static_cast<uint32_t>(c * 32), r);
            tmem_load_wait();
            for (int o = 0; o < others; ++o, ++b) {
                uint32_t v[32];
                box_get_row(land + static_cast<uint32_t>(b * kStageBoxBytes), lane, v);
#pragma unroll
                for (int k = 0; k < 32; ++k)
                    r[k] = __float_as_uint(__fadd_rn(__uint_as_float(r[k]), __uint_as_float(v[k])));
            }
            tmem_store_32(t_row[u] + static_cast<uint32_t>(c * 32), r);
        }
    }
    tmem_store_wait();
    fence_proxy_async_smem();  // these reads come before any later bulk write into the landing slice
    __syncwarp();
    return true;
}

// Step 2c: one reader count off each flag this warp read.
__device__ __forceinline__ void sk_release_reads(const KParams &p, const PairSchedule &s, const SplitTile *t, int nt,
                                                 uint32_t rank, int g, int lane) {
    if (lane != 0) return;
    for (int u = 0; u < nt; ++u)
        for (int i = 0; i < t[u].n; ++i)
            if (i != t[u].j) atomicSub(sk_flag(p, sk_slot(s, t[u].q0 + i, t[u].rel), rank, g), 1);
}

struct PairCfg {
    static constexpr int kABytes = kBlockM * kRowBytes;
    static constexpr int kBBytes = kPairHalfN * kRowBytes;
    static constexpr int kStageBytes = kABytes + kBBytes;
    static constexpr int kStages = ST_PAIR_STAGES;
    static constexpr int kRawStages = 0;
    static constexpr int kRawStageBytes = 0;
    static constexpr int kRingBytes = kStages * kStageBytes;
    static constexpr int kThreadCount = kThreads;
    static constexpr int kTmemCols = 512;  // two 256-column accumulators
    static constexpr int kSmemBytes = kRingBytes + kBarRegion + kCStagingBytes + 1024;
    static_assert(kSmemBytes <= 232448, "over the per-block shared memory limit");
    static_assert(kRingBytes >= kEpilogueWarps * kLandBoxes * kStageBoxBytes,
                  "the operand ring must hold every epilogue warp's stream-K landing slice");
};

// fp32 A and B split into tf32 inside the CTA-pair kernel (3xTF32): TMA
// brings raw fp32 tiles (A: 128 rows x 32 K; B: 128 columns x 32 K, as K-major
// rows or as four N-contiguous 32 x 32 boxes) into a raw ring; converter
// warps write hi = x with its 13 low mantissa bits cleared and lo = (x - hi)
// likewise cleared -- exact tf32 values, whatever the tensor core does with
// dropped bits -- into the MMA ring, K-major (an N-contiguous B is transposed
// on the way); the even CTA issues lo*hi, hi*lo and hi*hi per K step of 8.
// x - hi is exact in fp32, so x = hi + lo up to 2^-20 |x|.
#ifndef ST_X3_CONV_WARPS
#define ST_X3_CONV_WARPS 8
#endif
constexpr int kX3ConvWarps = ST_X3_CONV_WARPS;
struct X3PairCfg {
    static constexpr int kABytes = kBlockM * kRowBytes;       // 128 rows x 32 fp32
    static constexpr int kBBytes = kPairHalfN * kRowBytes;    // 128 columns x 32 fp32
    static constexpr int kStageBytes = 2 * kABytes + 2 * kBBytes;  // A hi, A lo, B hi, B lo
    static constexpr int kStages = 2;
    static constexpr int kRawStageBytes = kABytes + kBBytes;  // raw A, raw B
    static constexpr int kRawStages = 2;
    static constexpr int kRingBytes = kStages * kStageBytes + kRawStages * kRawStageBytes;
    static constexpr int kThreadCount = kThreads + 32 * kX3ConvWarps;
    static constexpr int kTmemCols = 512;
    static constexpr int kSmemBytes = kRingBytes + kBarRegion + kCStagingBytes + 1024;
    static_assert(kSmemBytes <= 232448, "over the per-block shared memory limit");
    static_assert(kRingBytes >= kEpilogueWarps * kLandBoxes * kStageBoxBytes,
                  "the operand ring must hold every epilogue warp's stream-K landing slice");
};

// x with its 13 low mantissa bits cleared: exactly representable in tf32.
__device__ __forceinline__ float tf32_trunc(float x) { return __uint_as_float(__float_as_uint(x) & 0xffffe000u); }

// hi / lo of four values: hi = tf32_trunc(x), lo = tf32_trunc(x - hi).
__device__ __forceinline__ void split4(const float4 &x, float4 &hi, float4 &lo) {
    hi = make_float4(tf32_trunc(x.x), tf32_trunc(x.y), tf32_trunc(x.z), tf32_trunc(x.w));
    lo = make_float4(tf32_trunc(x.x - hi.x), tf32_trunc(x.y - hi.y), tf32_trunc(x.z - hi.z), tf32_trunc(x.w - hi.w));
}

template <int FMT, bool B_MN, bool X3 = false>
__global__ void __cluster_dims__(2, 1, 1)
    __launch_bounds__(X3 ? X3PairCfg::kThreadCount : PairCfg::kThreadCount, 1)
    gemm_tc_pair_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                        const KParams p, const __grid_constant__ CStoreMaps cmaps) {
    using Cfg = std::conditional_t<X3, X3PairCfg, PairCfg>;
    constexpr bool kTf32 = FMT == 2;
    constexpr int kElem = kTf32 ? 4 : 2;
    constexpr int kBK = kRowBytes / kElem;
    constexpr int kMmaK = 32 / kElem;
    constexpr int kKSteps = kBK / kMmaK;
    // the split variant hands the tensor core K-major tiles whatever B's layout
    constexpr uint32_t kIdesc = mma_idesc(FMT, false, B_MN && !X3, 2 * kBlockM, kPairN);
    static_assert(!(kTf32 && B_MN && !X3), "packed tf32 operands are K-major");
    static_assert(!X3 || kTf32, "the in-kernel split is for fp32 operands");

    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + Cfg::kRingBytes);
    uint32_t *tmem_slot =
        reinterpret_cast<uint32_t *>(bars + 2 * Cfg::kStages + 5 + kEpilogueWarps + 2 * Cfg::kRawStages);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = cluster_rank();
    const bool even = rank == 0;
    const int pair = static_cast<int>(blockIdx.x >> 1);
    const int num_pairs = static_cast<int>(gridDim.x >> 1);
    const uint32_t bar0 = smem_addr(bars);
    auto full_bar = [&](int s) { return bar0 + 8u * s; };
    auto empty_bar = [&](int s) { return bar0 + 8u * (Cfg::kStages + s); };
    auto tfull_bar = [&](int a) { return bar0 + 8u * (2 * Cfg::kStages + a); };
    auto tempty_bar = [&](int a) { return bar0 + 8u * (2 * Cfg::kStages + 2 + a); };
    const uint32_t drain_bar = bar0 + 8u * (2 * Cfg::kStages + 4);
    auto fold_bar = [&](int g) { return bar0 + 8u * (2 * Cfg::kStages + 5 + g); };  // stream-K landing, per epilogue warp
    // X3: the raw ring's barriers (this CTA's own TMA loads / its converters)
    auto raw_full_bar = [&](int r) { return bar0 + 8u * (2 * Cfg::kStages + 5 + kEpilogueWarps + r); };
    auto raw_empty_bar = [&](int r) {
        return bar0 + 8u * (2 * Cfg::kStages + 5 + kEpilogueWarps + Cfg::kRawStages + r);
    };
    // X3 stage s of the MMA ring: [A hi | A lo | B hi | B lo]; raw stage r: [A | B]
    auto raw_of = [&](int r) { return smem + Cfg::kStages * Cfg::kStageBytes + r * Cfg::kRawStageBytes; };

    if (threadIdx.x == 0) {
        for (int s = 0; s < Cfg::kStages; ++s) {
            // X3: full[s] of the even CTA counts every converter warp of the pair
            mbar_init(full_bar(s), X3 ? 2 * kX3ConvWarps : 1);
            mbar_init(empty_bar(s), 1);
        }
        for (int r = 0; r < Cfg::kRawStages; ++r) {
            mbar_init(raw_full_bar(r), 1);
            mbar_init(raw_empty_bar(r), kX3ConvWarps);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(tfull_bar(a), 1);
            mbar_init(tempty_bar(a), 2 * kEpilogueWarps);
        }
        mbar_init(drain_bar, 1);
        for (int g = 0; g < kEpilogueWarps; ++g) mbar_init(fold_bar(g), 1);
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_map(&tmap_a);
        tma_prefetch_map(&tmap_b);
    }
    if (warp == 1) {
        tmem_alloc_pair(smem_addr(tmem_slot), Cfg::kTmemCols);
        tmem_relinquish_pair();
    }
    tc_fence_before_sync();
    cluster_sync();  // barriers of both CTAs initialised, TMEM allocated
    tc_fence_after_sync();
    const uint32_t tmem_base = *tmem_slot;
    pdl_begin();  // nothing above touches global memory
    const uint32_t even_full0 = map_to_rank(full_bar(0), 0);  // full[s] of the even CTA: + 8 s

    const int num_m_pairs = (p.m + 2 * kBlockM - 1) / (2 * kBlockM);
    const int num_n_pairs = (p.n + kPairN - 1) / kPairN;
    const int total = num_m_pairs * num_n_pairs;
    PairSchedule sched;
    sched.init(p, pair, num_pairs, total);
    PairWork w;

    if (X3 && warp == 0) {
        // ------------------------------------------------ TMA producer, raw fp32 tiles (both CTAs)
        if (lane == 0) {
            const uint64_t pol_a = operand_l2_policy_a(), pol_b = operand_l2_policy_b();
            int r = 0;
            uint32_t ph = 0;
            bool ok = true;
            PairUnits units;
            units.init(sched, pair);
            while (ok && units.next(sched, w)) {
                int64_t tm, tn;
                tile_raster(num_m_pairs, num_n_pairs, kGroupM, w.tile, tm, tn);
                const int m0 = static_cast<int>(tm) * 2 * kBlockM + static_cast<int>(rank) * kBlockM;
                const int n0 = static_cast<int>(tn) * kPairN + static_cast<int>(rank) * kPairHalfN;
                const bool rev = p.k_snake && w.tile < sched.dp_tiles && ((w.tile - pair) / num_pairs) & 1;
                for (int kb = w.k0; kb < w.k1; ++kb) {
                    if (!mbar_wait(raw_empty_bar(r), ph ^ 1u, abort_flag, p.timeout_ns)) {
                        ok = false;
                        break;
                    }
                    const int kx = (rev ? w.k0 + w.k1 - 1 - kb : kb) * kBK;
                    const uint32_t sa = smem_addr(raw_of(r)), sb = sa + X3PairCfg::kABytes;
                    mbar_arrive_expect_tx(raw_full_bar(r), X3PairCfg::kRawStageBytes);
                    tma_load_2d(sa, &tmap_a, raw_full_bar(r), kx, m0, pol_a);
                    if constexpr (B_MN) {  // four 32-column x 32-K boxes, N contiguous
#pragma unroll
                        for (int j = 0; j < kPairHalfN / 32; ++j)
                            tma_load_2d(sb + j * (kBK * 128), &tmap_b, raw_full_bar(r), n0 + 32 * j, kx, pol_b);
                    } else {
                        tma_load_2d(sb, &tmap_b, raw_full_bar(r), kx, n0, pol_b);
                    }
                    if (++r == Cfg::kRawStages) {
                        r = 0;
                        ph ^= 1u;
                    }
                }
            }
            if (!ok) {
                *abort_flag = 1;
                atomicExch(p.err, kDevAbortGemmProducer);
            }
        }
    } else if (X3 && warp >= kThreads / 32) {
        // ------------------------------------------------ converter warps (both CTAs): raw -> tf32 hi / lo
        const int cw = warp - kThreads / 32;
        const int tid = cw * 32 + lane;
        const uint32_t even_full0 = map_to_rank(full_bar(0), 0);
        int r = 0, s = 0, round = 0;
        uint32_t rph = 0, sph = 0;
        bool ok = true;
        PairUnits units;
        units.init(sched, pair);
        while (ok && units.next(sched, w)) {
            for (int kb = w.k0; kb < w.k1; ++kb) {
                // MMA stage s free (the pair's MMAs of its last round have read it;
                // the even CTA's first converter forwards that to the odd CTA)
                bool ready = mbar_wait(empty_bar(s), sph ^ 1u, abort_flag, p.timeout_ns);
                if (ready && even && cw == 0 && lane == 0 && round > 0)
                    mbar_arrive_cluster(map_to_rank(empty_bar(s), 1));
                ready = ready && mbar_wait(raw_full_bar(r), rph, abort_flag, p.timeout_ns);
                if (!__all_sync(0xffffffffu, ready)) {
                    ok = false;
                    break;
                }
                const uint8_t *raw = raw_of(r);
                uint8_t *stage = smem + s * Cfg::kStageBytes;
                // A: the same swizzled layout in and out, 16-byte chunk by chunk
#pragma unroll
                for (int q = 0; q < X3PairCfg::kABytes / 16 / (32 * kX3ConvWarps); ++q) {
                    const int c = tid + q * 32 * kX3ConvWarps;
                    const float4 x = reinterpret_cast<const float4 *>(raw)[c];
                    float4 hi, lo;
                    split4(x, hi, lo);
                    reinterpret_cast<float4 *>(stage)[c] = hi;
                    reinterpret_cast<float4 *>(stage + X3PairCfg::kABytes)[c] = lo;
                }
                const uint8_t *rawb = raw + X3PairCfg::kABytes;
                uint8_t *bhi = stage + 2 * X3PairCfg::kABytes, *blo = bhi + X3PairCfg::kBBytes;
                if constexpr (B_MN) {
                    // raw box j holds columns [32 j, 32 j + 32) x 32 K rows, N contiguous:
                    // element (n = 32 j + t, k) at k * 128 + ((t / 4) ^ (k % 8)) * 16 + (t % 4) * 4,
                    // so lane t reading column t of one K row hits bank 4 ((t / 4) ^ (k % 8)) + t % 4,
                    // 32 distinct banks.  Lane t takes K rows 4 kq .. 4 kq + 3 of column t and
                    // writes them as one 16-byte chunk of row n of the K-major tile, at
                    // n * 128 + (kq ^ (n % 8)) * 16: 8 distinct chunks per quarter warp.
#pragma unroll
                    for (int t = 0; t < 32 / kX3ConvWarps; ++t) {
                        const int combo = cw * (32 / kX3ConvWarps) + t;
                        const int j = combo >> 3, kq = combo & 7;
                        const uint8_t *box = rawb + j * (kBK * 128) + ((lane & 3) << 2);
                        float v[4];
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            const int k = 4 * kq + i;
                            v[i] = *reinterpret_cast<const float *>(box + k * 128 + (((lane >> 2) ^ (k & 7)) << 4));
                        }
                        const int n = 32 * j + lane;
                        float4 hi, lo;
                        split4(make_float4(v[0], v[1], v[2], v[3]), hi, lo);
                        const int off = n * 128 + ((kq ^ (n & 7)) << 4);
                        *reinterpret_cast<float4 *>(bhi + off) = hi;
                        *reinterpret_cast<float4 *>(blo + off) = lo;
                    }
                } else {
#pragma unroll
                    for (int q = 0; q < X3PairCfg::kBBytes / 16 / (32 * kX3ConvWarps); ++q) {
                        const int c = tid + q * 32 * kX3ConvWarps;
                        const float4 x = reinterpret_cast<const float4 *>(rawb)[c];
                        float4 hi, lo;
                        split4(x, hi, lo);
                        reinterpret_cast<float4 *>(bhi)[c] = hi;
                        reinterpret_cast<float4 *>(blo)[c] = lo;
                    }
                }
                fence_proxy_async_smem();  // these generic writes -> the tensor core's reads
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(raw_empty_bar(r));
                    if (even) mbar_arrive_release_cluster(full_bar(s));
                    else mbar_arrive_cluster_release(even_full0 + 8u * s);
                }
                if (++r == Cfg::kRawStages) {
                    r = 0;
                    rph ^= 1u;
                }
                if (++s == Cfg::kStages) {
                    s = 0;
                    sph ^= 1u;
                    ++round;
                }
            }
        }
        if (!ok) *abort_flag = 1;
    } else if (warp == 0) {
        // ------------------------------------------------ TMA producer (both CTAs)
        if (lane == 0) {
            const uint64_t pol_a = operand_l2_policy_a(), pol_b = operand_l2_policy_b();
            int s = 0;
            uint32_t ph = 0;
            int round = 0;  // passes over the ring completed
            bool ok = true;
            PairUnits units;
            units.init(sched, pair);
            while (ok && units.next(sched, w)) {
                int64_t tm, tn;
                tile_raster(num_m_pairs, num_n_pairs, kGroupM, w.tile, tm, tn);
                const int m0 = static_cast<int>(tm) * 2 * kBlockM + static_cast<int>(rank) * kBlockM;
                const int n0 = static_cast<int>(tn) * kPairN + static_cast<int>(rank) * kPairHalfN;
                // k_snake: the pair's odd-numbered whole tiles load K last to first
                // (stream-K units keep ascending K: their pairs sweep K together)
                const bool rev = p.k_snake && w.tile < sched.dp_tiles && ((w.tile - pair) / num_pairs) & 1;
                for (int kb = w.k0; kb < w.k1; ++kb) {
                    if (!mbar_wait(empty_bar(s), ph ^ 1u, abort_flag, p.timeout_ns)) {
                        ok = false;
                        break;
                    }
                    if (even) {
                        if (round > 0) mbar_arrive_cluster(map_to_rank(empty_bar(s), 1));  // stage free for the odd CTA
                        mbar_arrive_expect_tx(full_bar(s), 2 * Cfg::kStageBytes);
                    }
                    const uint32_t sa = smem_addr(smem + s * Cfg::kStageBytes);
                    const uint32_t sb = sa + Cfg::kABytes;
                    const uint32_t fb = even_full0 + 8u * s;
                    const int kx = (rev ? w.k0 + w.k1 - 1 - kb : kb) * kBK;
                    tma_load_2d_pair(sa, &tmap_a, fb, kx, m0, pol_a);
                    if constexpr (B_MN) {
#pragma unroll
                        for (int j = 0; j < kPairHalfN / 64; ++j)
                            tma_load_2d_pair(sb + j * (kBK * 128), &tmap_b, fb, n0 + 64 * j, kx, pol_b);
                    } else {
                        tma_load_2d_pair(sb, &tmap_b, fb, kx, n0, pol_b);
                    }
                    if (++s == Cfg::kStages) {
                        s = 0;
                        ph ^= 1u;
                        ++round;
                    }
                }
            }
            if (!ok) {
                *abort_flag = 1;
                atomicExch(p.err, kDevAbortGemmProducer);
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer (even CTA)
        if (even && lane == 0) {
            int s = 0;
            uint32_t ph = 0;
            int iter = 0;
            bool ok = true;
            PairUnits units;
            units.init(sched, pair);
            for (; ok && units.next(sched, w); ++iter) {
                const int acc = iter & 1;
                const uint32_t acc_ph = static_cast<uint32_t>(iter >> 1) & 1u;
                if (!mbar_wait(tempty_bar(acc), acc_ph ^ 1u, abort_flag, p.timeout_ns)) {
                    ok = false;
                    break;
                }
                tc_fence_after_sync();
                const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * kPairN);
                for (int kb = w.k0; kb < w.k1; ++kb) {
                    // X3: the converter warps of both CTAs release their writes at cluster scope
                    const bool landed = X3 ? mbar_wait_cluster(full_bar(s), ph, abort_flag, p.timeout_ns)
                                           : mbar_wait(full_bar(s), ph, abort_flag, p.timeout_ns);
                    if (!landed) {
                        ok = false;
                        break;
                    }
                    tc_fence_after_sync();
                    const uint32_t sa = smem_addr(smem + s * Cfg::kStageBytes);
                    if constexpr (X3) {
                        const uint32_t salo = sa + X3PairCfg::kABytes, sbhi = sa + 2 * X3PairCfg::kABytes;
                        const uint32_t sblo = sbhi + X3PairCfg::kBBytes;
#pragma unroll
                        for (int ks = 0; ks < kKSteps; ++ks) {
                            const uint64_t ahi = smem_desc_sw128(sa + ks * 32, 16, 1024);
                            const uint64_t alo = smem_desc_sw128(salo + ks * 32, 16, 1024);
                            const uint64_t bh = smem_desc_sw128(sbhi + ks * 32, 16, 1024);
                            const uint64_t bl = smem_desc_sw128(sblo + ks * 32, 16, 1024);
                            // the small terms first, then the leading product
                            tc_mma_pair<true>(d_tmem, alo, bh, kIdesc, (kb != w.k0 || ks != 0) ? 1u : 0u);
                            tc_mma_pair<true>(d_tmem, ahi, bl, kIdesc, 1u);
                            tc_mma_pair<true>(d_tmem, ahi, bh, kIdesc, 1u);
                        }
                    } else {
                        const uint32_t sb = sa + Cfg::kABytes;
#pragma unroll
                        for (int ks = 0; ks < kKSteps; ++ks) {
                            const uint64_t adesc = smem_desc_sw128(sa + ks * 32, 16, 1024);
                            uint64_t bdesc;
                            if constexpr (B_MN) {
                                bdesc = smem_desc_sw128(sb + ks * (kMmaK * 128), kBK * 128, 1024);
                            } else {
                                bdesc = smem_desc_sw128(sb + ks * 32, 16, 1024);
                            }
                            tc_mma_pair<kTf32>(d_tmem, adesc, bdesc, kIdesc, (kb != w.k0 || ks != 0) ? 1u : 0u);
                        }
                    }
                    tc_commit_pair(empty_bar(s));
                    if (++s == Cfg::kStages) {
                        s = 0;
                        ph ^= 1u;
                    }
                }
                if (!ok) break;
                tc_commit_pair(tfull_bar(acc));
            }
            if (!ok) {
                *abort_flag = 1;
                atomicExch(p.err, kDevAbortGemmMma);
            }
            tc_commit_pair(drain_bar);
            (void)mbar_wait(drain_bar, 0, abort_flag, p.timeout_ns);
        }
    } else {
        // ------------------------------------------------ epilogue (warps 2..5, both CTAs)
        const int g = warp & 3;
        const uint32_t staging = smem_addr(smem + Cfg::kRingBytes + kBarRegion) +
                                 static_cast<uint32_t>(g * 2 * kStageBoxBytes);
        int sbuf = 0;
        const uint32_t even_tempty0 = map_to_rank(tempty_bar(0), 0);
        const uint32_t odd_tfull0 = map_to_rank(tfull_bar(0), 1);
        // the accumulator of the unit at MMA position idx (buffer idx & 1) is
        // complete: wait for it and forward the news to the odd CTA
        auto wait_full = [&](int idx) -> bool {
            const int acc = idx & 1;
            const bool ready = mbar_wait(tfull_bar(acc), static_cast<uint32_t>(idx >> 1) & 1u, abort_flag, p.timeout_ns);
            if (!__all_sync(0xffffffffu, ready)) {
                *abort_flag = 1;
                if (lane == 0) atomicExch(p.err, kDevAbortGemmEpilogue);
                return false;
            }
            if (even && warp == 2 && lane == 0) mbar_arrive_cluster(odd_tfull0 + 8u * acc);
            tc_fence_after_sync();
            return true;
        };
        auto t_row_of = [&](int idx) {
            return tmem_base + (static_cast<uint32_t>(g * 32) << 16) + static_cast<uint32_t>((idx & 1) * kPairN);
        };
        // bias, conversion and the store of accumulator columns [c_begin, c_end)
        auto store_c = [&](const PairWork &u, int idx, int c_begin, int c_end, bool reduce) {
            int64_t tm, tn;
            tile_raster(num_m_pairs, num_n_pairs, kGroupM, u.tile, tm, tn);
            const int m0 = static_cast<int>(tm) * 2 * kBlockM + static_cast<int>(rank) * kBlockM;
            const int n0 = static_cast<int>(tn) * kPairN;
            const uint32_t t_row = t_row_of(idx);
            if (p.staged) {
                store_tile_staged<kPairN>(p, cmaps, t_row, m0 + g * 32, n0, staging, sbuf, lane, c_begin, c_end,
                                          reduce);
            } else {
                const int row = m0 + g * 32 + lane;
#pragma unroll 1
                for (int c = c_begin / 32; c < c_end / 32; ++c) {
                    const int col0 = n0 + c * 32;
                    if (col0 >= p.n) break;
                    uint32_t r[32];
                    tmem_load_32(t_row + c * 32, r);
                    tmem_load_wait();
                    if (p.bias != nullptr) add_bias_chunk(p, col0, lane, r);
                    if (row < p.m) store_row_chunk(p, row, col0, r);
                }
            }
        };
        auto release = [&](int idx) {
            tc_fence_before_sync();
            __syncwarp();
            if (lane == 0) {
                if (even) mbar_arrive(tempty_bar(idx & 1));
                else mbar_arrive_cluster(even_tempty0 + 8u * (idx & 1));
            }
        };
        // whole tiles in MMA order; a split tile's unit first publishes the
        // columns the tile's other units own (no waiting) and keeps its
        // accumulator.  Split units are the pair's last (at most two), so
        // once all have published, every MMA of the pair is complete and the
        // operand ring is free to land the other units' columns of its own.
        PairUnits units;
        units.init(sched, pair);
        PairWork w;
        PairWork split_u0{}, split_u1{};
        int n_split = 0, idx = 0;
        bool ok = true;
        for (; ok && units.next(sched, w); ++idx) {
            if (!wait_full(idx)) {
                ok = false;
                break;
            }
            if (w.kind != kUnitWhole && p.sk_l2add == 2) {  // ordered L2 fold (see above)
                const SplitTile t = split_tile(p, sched, w);
                int *flag = sk_flag(p, sk_slot(sched, t.q0, t.rel), rank, g);
                if (t.j == 0) {
                    store_c(w, idx, 0, kPairN, false);
                    if (lane == 0) {
                        bulk_wait_group_all();  // this warp's rows of the tile are in C
                        fence_proxy_async_global();
                        red_release_gpu_add(flag, t.n - 1);
                    }
                    __syncwarp();
                } else {
                    bool up = true;
                    if (lane == 0) {
                        const uint64_t t0 = global_timer_ns();
                        while (ld_acquire_gpu(flag) < 1) {
                            if (*abort_flag != 0 || global_timer_ns() - t0 > p.timeout_ns) {
                                up = false;
                                break;
                            }
                        }
                        if (up) {
                            fence_proxy_async_global();  // the acquire comes before the reduce-adds
                            atomicSub(flag, 1);
                        }
                    }
                    if (!__shfl_sync(0xffffffffu, up, 0)) {
                        *abort_flag = 1;
                        if (lane == 0) atomicExch(p.err, kDevAbortGemmStreamK);
                        ok = false;
                        break;
                    }
                    store_c(w, idx, 0, kPairN, true);
                }
                release(idx);
                continue;
            }
            if (w.kind == kUnitWhole || p.sk_l2add) {  // a split unit adds its partial onto C in L2
                store_c(w, idx, 0, kPairN, w.kind != kUnitWhole);
                release(idx);
                continue;
            }
            sk_publish(p, sched, split_tile(p, sched, w), rank, g, lane, t_row_of(idx), staging, sbuf);
            if (n_split == 0) split_u0 = w;
            else split_u1 = w;
            ++n_split;
        }
        if (ok && n_split > 0) {
            SplitTile st[2];
            uint32_t rows[2];
            for (int i = 0; i < n_split; ++i) {
                st[i] = split_tile(p, sched, i == 0 ? split_u0 : split_u1);
                rows[i] = t_row_of(idx - n_split + i);
            }
            uint32_t land_phase = 0;
            const uint32_t land = smem_addr(smem) + static_cast<uint32_t>(g * kLandBoxes * kStageBoxBytes);
            // both units' boxes in one round when they fit the landing slice
            const bool one_round = n_split == 1 || sk_land_boxes(st[0]) + sk_land_boxes(st[1]) <= kLandBoxes;
            bool folded = sk_wait_others(p, sched, st, n_split, rank, g, lane, abort_flag);
            if (folded && one_round) {
                folded = sk_land_and_add(p, sched, st, rows, 0, n_split, rank, g, lane, land, fold_bar(g), land_phase,
                                         abort_flag);
            } else {
                for (int i = 0; folded && i < n_split; ++i)
                    folded = sk_land_and_add(p, sched, st, rows, i, i + 1, rank, g, lane, land, fold_bar(g),
                                             land_phase, abort_flag);
            }
            if (!folded) {
                *abort_flag = 1;
                if (lane == 0) atomicExch(p.err, kDevAbortGemmStreamK);
            } else {
                sk_release_reads(p, sched, st, n_split, rank, g, lane);
                for (int i = 0; i < n_split; ++i) {
                    store_c(i == 0 ? split_u0 : split_u1, idx - n_split + i, st[i].c_begin, st[i].c_end, false);
                    release(idx - n_split + i);
                }
            }
        }
        if (p.staged && lane == 0) bulk_wait_group_all();  // every TMA store of C has landed
    }

    publish_peer_writes(p);
    tc_fence_before_sync();
    cluster_sync();  // all MMAs retired, all TMEM reads done, no remote access pending
    if (warp == 1) {
        __syncwarp();
        tc_fence_after_sync();
        tmem_dealloc_pair(tmem_base, Cfg::kTmemCols);
    }
}

// ---------------------------------------------------------------- fp32 via 3xTF32, split in shared memory
// fp32 A and B come in by TMA untouched; a converter warpgroup splits every
// staged element x into tf32 hi = tf32(x) (written back in place) and
// lo = tf32(x - hi) (written to a twin buffer with the same swizzled
// layout), and the MMA warp issues hi*hi, hi*lo and lo*hi per K step of 8.
// The split is elementwise, so the 128-byte swizzle of the staged tiles
// needs no special handling; a proxy fence hands the converted bytes to the
// tensor core.  Compared with packing the operands in global memory first,
// HBM/L2 traffic drops from 3x to 1x of A and B and two launches disappear.
constexpr int kX3SplitWarps = 8;
constexpr int kX3SplitThreads = 32 * kX3SplitWarps;
constexpr int kX3Threads = 192 + kX3SplitThreads;  // warps: 0 TMA, 1 MMA, 2-5 epilogue, 6.. split

template <int BN, bool B_MN>
struct X3Cfg {
    static constexpr int kABytes = kBlockM * kRowBytes;  // 128 rows x 32 fp32
    static constexpr int kBBytes = BN * kRowBytes;       // BN x 32 fp32
    // per stage: A (hi in place), A lo, B hi, B lo, and for an N-contiguous B
    // the raw tile (transposed into B hi / B lo by the split warps)
    static constexpr int kStageBytes = 2 * kABytes + 2 * kBBytes + (B_MN ? kBBytes : 0);
    static constexpr int kStages = (232448 - 1280) / kStageBytes > 4 ? 4 : (232448 - 1280) / kStageBytes;
    static constexpr int kTmemCols = 2 * BN;
    static constexpr int kSmemBytes = kStages * kStageBytes + 256 + 1024;
    static_assert(kStages >= 3, "too few pipeline stages");
};

__device__ __forceinline__ uint32_t tf32_bits(float x) {
    uint32_t u = __float_as_uint(x);
    if ((u & 0x7f800000u) == 0x7f800000u) return u;
    u += 0x0fffu + ((u >> 13) & 1u);
    return u & 0xffffe000u;
}

template <bool B_MN, int BN>
__global__ void __launch_bounds__(kX3Threads, 1)
    gemm_tf32x3_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                       const KParams p) {
    using Cfg = X3Cfg<BN, B_MN>;
    constexpr int kBK = 32;          // fp32 elements per stage row (128 bytes)
    constexpr int kMmaK = 8;         // K per tcgen05.mma kind::tf32
    constexpr int kKSteps = kBK / kMmaK;
    // tf32 operands are always handed to the MMA K-major: an N-contiguous
    // tf32 B read by the tensor core comes back as zeros on sm_100a, so an
    // N-contiguous B is transposed by the split warps
    constexpr uint32_t kIdesc = mma_idesc(2, false, false, kBlockM, BN);

    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + Cfg::kStages * Cfg::kStageBytes);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 3 * Cfg::kStages + 5);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t bar0 = smem_addr(bars);
    auto full_bar = [&](int s) { return bar0 + 8u * s; };
    auto split_bar = [&](int s) { return bar0 + 8u * (Cfg::kStages + s); };
    auto empty_bar = [&](int s) { return bar0 + 8u * (2 * Cfg::kStages + s); };
    auto tfull_bar = [&](int a) { return bar0 + 8u * (3 * Cfg::kStages + a); };
    auto tempty_bar = [&](int a) { return bar0 + 8u * (3 * Cfg::kStages + 2 + a); };
    const uint32_t drain_bar = bar0 + 8u * (3 * Cfg::kStages + 4);
    // stage s: [A | A lo | B | B lo]
    auto a_of = [&](int s) { return smem + s * Cfg::kStageBytes; };
    auto alo_of = [&](int s) { return smem + s * Cfg::kStageBytes + Cfg::kABytes; };
    auto b_of = [&](int s) { return smem + s * Cfg::kStageBytes + 2 * Cfg::kABytes; };
    auto blo_of = [&](int s) { return smem + s * Cfg::kStageBytes + 2 * Cfg::kABytes + Cfg::kBBytes; };
    auto braw_of = [&](int s) { return smem + s * Cfg::kStageBytes + 2 * Cfg::kABytes + 2 * Cfg::kBBytes; };

    if (threadIdx.x == 0) {
        for (int s = 0; s < Cfg::kStages; ++s) {
            mbar_init(full_bar(s), 1);
            mbar_init(split_bar(s), kX3SplitWarps);
            mbar_init(empty_bar(s), 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(tfull_bar(a), 1);
            mbar_init(tempty_bar(a), kEpilogueWarps);
        }
        mbar_init(drain_bar, 1);
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_map(&tmap_a);
        tma_prefetch_map(&tmap_b);
    }
    if (warp == 1) {
        tmem_alloc(smem_addr(tmem_slot), Cfg::kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before_sync();
    __syncthreads();
    tc_fence_after_sync();
    const uint32_t tmem_base = *tmem_slot;
    pdl_begin();  // nothing above touches global memory

    if (warp == 0) {
        // ------------------------------------------------ TMA producer
        if (lane == 0) {
            const uint64_t pol = l2_policy_evict_last();
            int s = 0;
            uint32_t ph = 0;
            bool ok = true;
            for (int t = blockIdx.x; ok && t < p.total_tiles; t += gridDim.x) {
                int64_t tm, tn;
                tile_raster(p.num_m_tiles, p.num_n_tiles, kGroupM, t, tm, tn);
                const int m0 = static_cast<int>(tm) * kBlockM;
                const int n0 = static_cast<int>(tn) * BN;
                for (int kb = 0; kb < p.num_k_blocks; ++kb) {
                    if (!mbar_wait(empty_bar(s), ph ^ 1u, abort_flag, p.timeout_ns)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(full_bar(s), Cfg::kABytes + Cfg::kBBytes);
                    tma_load_2d(smem_addr(a_of(s)), &tmap_a, full_bar(s), kb * kBK, m0, pol);
                    if constexpr (B_MN) {
                        // raw N-contiguous chunks of 32 columns x 32 K rows
                        const uint32_t sraw = smem_addr(braw_of(s));
#pragma unroll
                        for (int j = 0; j < BN / 32; ++j)
                            tma_load_2d(sraw + j * (kBK * 128), &tmap_b, full_bar(s), n0 + 32 * j, kb * kBK, pol);
                    } else {
                        tma_load_2d(smem_addr(b_of(s)), &tmap_b, full_bar(s), kb * kBK, n0, pol);
                    }
                    if (++s == Cfg::kStages) {
                        s = 0;
                        ph ^= 1u;
                    }
                }
            }
            if (!ok) {
                *abort_flag = 1;
                atomicExch(p.err, kDevAbortGemmProducer);
            }
        }
    } else if (warp >= 6) {
        // ------------------------------------------------ split warps: x -> (hi, lo)
        // Each thread first issues all its shared-memory loads of the stage,
        // then converts, then stores, so the loads overlap.
        const int tid = threadIdx.x - 6 * 32;
        constexpr int kAVec = Cfg::kABytes / 16 / kX3SplitThreads;  // float4 of A per thread
        constexpr int kBVec = Cfg::kBBytes / 16 / kX3SplitThreads;  // K-groups of B per thread
        static_assert(kAVec * 16 * kX3SplitThreads == Cfg::kABytes, "A split must divide evenly");
        static_assert(kBVec * 16 * kX3SplitThreads == Cfg::kBBytes, "B split must divide evenly");
        int s = 0;
        uint32_t ph = 0;
        bool ok = true;
        for (int t = blockIdx.x; ok && t < p.total_tiles; t += gridDim.x) {
            for (int kb = 0; kb < p.num_k_blocks; ++kb) {
                const bool ready = mbar_wait(full_bar(s), ph, abort_flag, p.timeout_ns);
                if (!__all_sync(0xffffffffu, ready)) {
                    ok = false;
                    break;
                }
                float4 *a = reinterpret_cast<float4 *>(a_of(s));
                float4 *alo = reinterpret_cast<float4 *>(alo_of(s));
                float4 xa[kAVec];
#pragma unroll
                for (int q = 0; q < kAVec; ++q) xa[q] = a[tid + q * kX3SplitThreads];
                float xb[kBVec][4];
                if constexpr (B_MN) {
                    // raw element (n, k) sits in 32-column chunk n/32, K row k, 16-byte
                    // group (n%32)/4 swizzled with k%8
                    const uint8_t *raw = braw_of(s);
#pragma unroll
                    for (int q = 0; q < kBVec; ++q) {
                        const int idx = tid + q * kX3SplitThreads;
                        const int n = idx % BN, kq = idx / BN, nl = n & 31;
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            const int k = kq * 4 + i;
                            xb[q][i] = *reinterpret_cast<const float *>(
                                raw + (n >> 5) * (kBK * 128) + k * 128 + (((nl >> 2) ^ (k & 7)) << 4) + ((nl & 3) << 2));
                        }
                    }
                } else {
                    const float4 *b = reinterpret_cast<const float4 *>(b_of(s));
#pragma unroll
                    for (int q = 0; q < kBVec; ++q) {
                        const float4 v = b[tid + q * kX3SplitThreads];
                        xb[q][0] = v.x;
                        xb[q][1] = v.y;
                        xb[q][2] = v.z;
                        xb[q][3] = v.w;
                    }
                }
#pragma unroll
                for (int q = 0; q < kAVec; ++q) {
                    float4 h, l;
                    h.x = __uint_as_float(tf32_bits(xa[q].x));
                    h.y = __uint_as_float(tf32_bits(xa[q].y));
                    h.z = __uint_as_float(tf32_bits(xa[q].z));
                    h.w = __uint_as_float(tf32_bits(xa[q].w));
                    l.x = __uint_as_float(tf32_bits(xa[q].x - h.x));
                    l.y = __uint_as_float(tf32_bits(xa[q].y - h.y));
                    l.z = __uint_as_float(tf32_bits(xa[q].z - h.z));
                    l.w = __uint_as_float(tf32_bits(xa[q].w - h.w));
                    a[tid + q * kX3SplitThreads] = h;
                    alo[tid + q * kX3SplitThreads] = l;
                }
#pragma unroll
                for (int q = 0; q < kBVec; ++q) {
                    float4 h, l;
                    h.x = __uint_as_float(tf32_bits(xb[q][0]));
                    h.y = __uint_as_float(tf32_bits(xb[q][1]));
                    h.z = __uint_as_float(tf32_bits(xb[q][2]));
                    h.w = __uint_as_float(tf32_bits(xb[q][3]));
                    l.x = __uint_as_float(tf32_bits(xb[q][0] - h.x));
                    l.y = __uint_as_float(tf32_bits(xb[q][1] - h.y));
                    l.z = __uint_as_float(tf32_bits(xb[q][2] - h.z));
                    l.w = __uint_as_float(tf32_bits(xb[q][3] - h.w));
                    int off;
                    if constexpr (B_MN) {
                        // K-major home of (n, 4 kq .. 4 kq + 3): row n, 16-byte group kq ^ (n % 8)
                        const int idx = tid + q * kX3SplitThreads;
                        const int n = idx % BN, kq = idx / BN;
                        off = n * 128 + ((kq ^ (n & 7)) << 4);
                    } else {
                        off = (tid + q * kX3SplitThreads) * 16;
                    }
                    *reinterpret_cast<float4 *>(b_of(s) + off) = h;
                    *reinterpret_cast<float4 *>(blo_of(s) + off) = l;
                }
                fence_proxy_async_smem();  // generic-proxy writes -> tensor-core reads
                __syncwarp();
                if (lane == 0) mbar_arrive(split_bar(s));
                if (++s == Cfg::kStages) {
                    s = 0;
                    ph ^= 1u;
                }
            }
        }
        if (!ok) *abort_flag = 1;
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer
        if (lane == 0) {
            int s = 0;
            uint32_t ph = 0;
            int iter = 0;
            bool ok = true;
            for (int t = blockIdx.x; ok && t < p.total_tiles; t += gridDim.x, ++iter) {
                const int acc = iter & 1;
                const uint32_t acc_ph = static_cast<uint32_t>(iter >> 1) & 1u;
                if (!mbar_wait(tempty_bar(acc), acc_ph ^ 1u, abort_flag, p.timeout_ns)) {
                    ok = false;
                    break;
                }
                tc_fence_after_sync();
                const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
                for (int kb = 0; kb < p.num_k_blocks; ++kb) {
                    if (!mbar_wait(split_bar(s), ph, abort_flag, p.timeout_ns)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after_sync();
                    const uint32_t sa = smem_addr(a_of(s)), salo = smem_addr(alo_of(s));
                    const uint32_t sb = smem_addr(b_of(s)), sblo = smem_addr(blo_of(s));
#pragma unroll
                    for (int ks = 0; ks < kKSteps; ++ks) {
                        const uint64_t ahi = smem_desc_sw128(sa + ks * 32, 16, 1024);
                        const uint64_t alo = smem_desc_sw128(salo + ks * 32, 16, 1024);
                        const uint64_t bhi = smem_desc_sw128(sb + ks * 32, 16, 1024);
                        const uint64_t blo = smem_desc_sw128(sblo + ks * 32, 16, 1024);
                        // small terms first, then the leading product
                        tc_mma<true>(d_tmem, alo, bhi, kIdesc, (kb | ks) != 0 ? 1u : 0u);
                        tc_mma<true>(d_tmem, ahi, blo, kIdesc, 1u);
                        tc_mma<true>(d_tmem, ahi, bhi, kIdesc, 1u);
                    }
                    tc_commit(empty_bar(s));
                    if (++s == Cfg::kStages) {
                        s = 0;
                        ph ^= 1u;
                    }
                }
                if (!ok) break;
                tc_commit(tfull_bar(acc));
            }
            if (!ok) {
                *abort_flag = 1;
                atomicExch(p.err, kDevAbortGemmMma);
            }
            tc_commit(drain_bar);
            (void)mbar_wait(drain_bar, 0, abort_flag, p.timeout_ns);
        }
    } else {
        // ------------------------------------------------ epilogue (warps 2..5)
        const int g = warp & 3;
        int iter = 0;
        for (int t = blockIdx.x; t < p.total_tiles; t += gridDim.x, ++iter) {
            const int acc = iter & 1;
            const uint32_t acc_ph = static_cast<uint32_t>(iter >> 1) & 1u;
            int64_t tm, tn;
            tile_raster(p.num_m_tiles, p.num_n_tiles, kGroupM, t, tm, tn);
            const int m0 = static_cast<int>(tm) * kBlockM;
            const int n0 = static_cast<int>(tn) * BN;
            const bool ready = mbar_wait(tfull_bar(acc), acc_ph, abort_flag, p.timeout_ns);
            if (!__all_sync(0xffffffffu, ready)) {
                *abort_flag = 1;
                if (lane == 0) atomicExch(p.err, kDevAbortGemmEpilogue);
                break;
            }
            tc_fence_after_sync();
            const int row = m0 + g * 32 + lane;
            const uint32_t t_row = tmem_base + (static_cast<uint32_t>(g * 32) << 16) + static_cast<uint32_t>(acc * BN);
#pragma unroll 1
            for (int c = 0; c < BN / 32; ++c) {
                const int col0 = n0 + c * 32;
                if (col0 >= p.n) break;
                uint32_t r[32];
                tmem_load_32(t_row + c * 32, r);
                tmem_load_wait();
                if (p.bias != nullptr) add_bias_chunk(p, col0, lane, r);
                if (row < p.m) store_row_chunk(p, row, col0, r);
            }
            tc_fence_before_sync();
            __syncwarp();
            if (lane == 0) mbar_arrive(tempty_bar(acc));
        }
    }

    publish_peer_writes(p);
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after_sync();
        tmem_dealloc(tmem_base, Cfg::kTmemCols);
    }
}

// ---------------------------------------------------------------- host side
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    });
    return fn;
}

int make_map(CUtensorMap *map, CUtensorMapDataType dt, const void *base, uint64_t inner, uint64_t outer,
             uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer) {
    auto fn = encode_fn();
    if (!fn) return fail(ST_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    cuuint64_t dims[2] = {inner, outer};
    cuuint64_t strides[1] = {row_bytes};
    cuuint32_t box[2] = {box_inner, box_outer};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, dt, 2, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return fail(ST_ERR_INVALID_ARGUMENT, "cuTensorMapEncodeTiled rejected an operand (error " +
                                                 std::to_string(static_cast<int>(r)) + ")");
    return ST_OK;
}

template <int FMT, bool B_MN, int BN>
int launch_instance(const CUtensorMap &ma, const CUtensorMap &mb, const KParams &kp, const CStoreMaps &cm, int ctas,
                    cudaStream_t stream) {
    using Cfg = TileCfg<BN>;
    auto kern = gemm_tc_kernel<FMT, B_MN, BN>;
    static uint64_t attr_set = 0;  // one bit per device ordinal
    int dev = 0;
    ST_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64 || !(attr_set & (1ull << dev))) {
        ST_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes));
        if (dev >= 0 && dev < 64) attr_set |= 1ull << dev;
    }
    ST_CUDA_TRY(launch_kernel(kern, ctas, kThreads, Cfg::kSmemBytes, stream, ma, mb, kp, cm));
    note_launch();
    const cudaError_t e = cudaPeekAtLastError();
    return e == cudaSuccess ? ST_OK : cuda_fail(cudaGetLastError(), "gemm_tc_kernel launch");
}

template <int FMT, bool B_MN>
int dispatch_bn(int bn, const CUtensorMap &ma, const CUtensorMap &mb, const KParams &kp, const CStoreMaps &cm,
                int ctas, cudaStream_t stream) {
    switch (bn) {
    case 256: return launch_instance<FMT, B_MN, 256>(ma, mb, kp, cm, ctas, stream);
    case 128: return launch_instance<FMT, B_MN, 128>(ma, mb, kp, cm, ctas, stream);
    case 64: return launch_instance<FMT, B_MN, 64>(ma, mb, kp, cm, ctas, stream);
    default: return fail(ST_ERR_UNSUPPORTED, "unsupported block_n");
    }
}

// C = 0 + bias (0 without a bias) on tiles [first, total) of the CTA-pair
// raster only: the split tiles of an L2-add launch whose whole-tile waves
// store their tiles outright.  Block b covers rows [32 (b % 8), +32) of
// split tile b / 8; C's rows start 16-byte aligned (the staged-C rule).
__global__ void __launch_bounds__(256) c_init_tiles_f32_kernel(float *c, long long ldc, const void *bias,
                                                               int bias_dtype, int m, int n, int num_m_pairs,
                                                               int num_n_pairs, int first, int total) {
    pdl_wait();
    const int blocks = (total - first) * 8;
    for (int b = blockIdx.x; b < blocks; b += gridDim.x) {
        int64_t tm, tn;
        tile_raster(num_m_pairs, num_n_pairs, kGroupM, first + b / 8, tm, tn);
        const int r0 = static_cast<int>(tm) * 2 * kBlockM + (b % 8) * 32;
        const int q0 = static_cast<int>(tn) * kPairN;
        for (int i = threadIdx.x; i < 32 * (kPairN / 4); i += blockDim.x) {
            const int r = r0 + i / (kPairN / 4), q = q0 + 4 * (i % (kPairN / 4));
            if (r >= m) break;  // rows grow with i
            if (q >= n) continue;
            float *dst = c + static_cast<long long>(r) * ldc + q;
            if (q + 4 <= n) {
                float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                if (bias != nullptr) {
                    v.x = 0.0f + load_bias(bias, bias_dtype, q);
                    v.y = 0.0f + load_bias(bias, bias_dtype, q + 1);
                    v.z = 0.0f + load_bias(bias, bias_dtype, q + 2);
                    v.w = 0.0f + load_bias(bias, bias_dtype, q + 3);
                }
                *reinterpret_cast<float4 *>(dst) = v;
            } else {
                for (int j = 0; q + j < n; ++j) dst[j] = bias != nullptr ? 0.0f + load_bias(bias, bias_dtype, q + j) : 0.0f;
            }
        }
    }
    pdl_trigger();
}

// The preset an L2-add CTA-pair launch of `pairs` pairs needs: the split
// the kernel will derive from that grid decides which tiles are split; all
// of C when every tile is, only the tail tiles after whole-tile waves.
int launch_c_preset_f32(const GemmArgs &g, const KParams &kp, int pairs, int sm_count, cudaStream_t stream) {
    const int num_m_pairs = (kp.m + 2 * kBlockM - 1) / (2 * kBlockM);
    const int num_n_pairs = (kp.n + kPairN - 1) / kPairN;
    const int total = num_m_pairs * num_n_pairs;
    int dp = 0, skp = 0;
    long long ski = 0;
    stream_k_split(total, pairs, kp.num_k_blocks, kp.sk_mode, dp, skp, ski);
    if (skp == 0) return ST_OK;  // nothing split: every tile is stored whole
    if (dp == 0) return launch_c_init_f32(g, sm_count, stream);
    const int blocks = (total - dp) * 8;
    const int grid = blocks < 8 * sm_count ? blocks : 8 * sm_count;
    ST_CUDA_TRY(launch_kernel(c_init_tiles_f32_kernel, static_cast<unsigned>(grid), 256, 0, stream,
                              static_cast<float *>(g.c), static_cast<long long>(g.ldc), g.bias, g.bias_dtype, kp.m,
                              kp.n, num_m_pairs, num_n_pairs, dp, total));
    note_launch();
    const cudaError_t e = cudaPeekAtLastError();
    return e == cudaSuccess ? ST_OK : cuda_fail(cudaGetLastError(), "c_init_tiles_f32_kernel launch");
}

// preset: for an L2-add launch whose C is not preset yet, the call whose
// split tiles get C = 0 + bias first (on the pair count actually launched)
template <int FMT, bool B_MN, bool X3 = false>
int launch_pair(const CUtensorMap &ma, const CUtensorMap &mb, const KParams &kp, const CStoreMaps &cm,
                int pairs_wanted, const GemmArgs *preset, int sm_count, cudaStream_t stream) {
    using Cfg = std::conditional_t<X3, X3PairCfg, PairCfg>;
    auto kern = gemm_tc_pair_kernel<FMT, B_MN, X3>;
    static uint64_t attr_set = 0;
    static int max_clusters[64] = {0};
    int dev = 0;
    ST_CUDA_TRY(cudaGetDevice(&dev));
    const bool cached = dev >= 0 && dev < 64 && (attr_set & (1ull << dev));
    int clusters = cached ? max_clusters[dev] : 0;
    if (!cached) {
        ST_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes));
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(2 * pairs_wanted, 1, 1);
        cfg.blockDim = dim3(Cfg::kThreadCount, 1, 1);
        cfg.dynamicSmemBytes = Cfg::kSmemBytes;
        cudaLaunchAttribute attr;
        attr.id = cudaLaunchAttributeClusterDimension;
        attr.val.clusterDim.x = 2;
        attr.val.clusterDim.y = 1;
        attr.val.clusterDim.z = 1;
        cfg.attrs = &attr;
        cfg.numAttrs = 1;
        if (cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg) != cudaSuccess || clusters <= 0) {
            cudaGetLastError();
            clusters = pairs_wanted;
        }
        if (dev >= 0 && dev < 64) {
            max_clusters[dev] = clusters;
            attr_set |= 1ull << dev;
        }
    }
    const int pairs = pairs_wanted < clusters ? pairs_wanted : clusters;
    if (preset != nullptr) ST_TRY(launch_c_preset_f32(*preset, kp, pairs, sm_count, stream));
    if (std::getenv("SPTILES_B200_DEBUG"))
        std::fprintf(stderr, "[sptiles_b200] pair gemm: %d pairs (wanted %d, co-resident clusters %d), smem %d\n",
                     pairs, pairs_wanted, clusters, Cfg::kSmemBytes);
    ST_CUDA_TRY(launch_kernel(kern, 2 * pairs, Cfg::kThreadCount, Cfg::kSmemBytes, stream, ma, mb, kp, cm));
    note_launch();
    const cudaError_t e = cudaPeekAtLastError();
    return e == cudaSuccess ? ST_OK : cuda_fail(cudaGetLastError(), "gemm_tc_pair_kernel launch");
}

template <bool B_MN, int BN>
int launch_x3_instance(const CUtensorMap &ma, const CUtensorMap &mb, const KParams &kp, int ctas,
                       cudaStream_t stream) {
    using Cfg = X3Cfg<BN, B_MN>;
    auto kern = gemm_tf32x3_kernel<B_MN, BN>;
    static uint64_t attr_set = 0;
    int dev = 0;
    ST_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64 || !(attr_set & (1ull << dev))) {
        ST_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes));
        if (dev >= 0 && dev < 64) attr_set |= 1ull << dev;
    }
    ST_CUDA_TRY(launch_kernel(kern, ctas, kX3Threads, Cfg::kSmemBytes, stream, ma, mb, kp));
    note_launch();
    const cudaError_t e = cudaPeekAtLastError();
    return e == cudaSuccess ? ST_OK : cuda_fail(cudaGetLastError(), "gemm_tf32x3_kernel launch");
}

}  // namespace

int plan_gemm_x3(int64_t m, int64_t n, bool b_n_contiguous, int sm_count, GemmPlan *plan) {
    if (m <= 0 || n <= 0) return fail(ST_ERR_INVALID_ARGUMENT, "matmul extents must be positive");
    if (sm_count <= 0) sm_count = 148;
    GemmPlan best;
    double best_score = -1.0;
    const int cand[2] = {128, 64};
    const double mma_eff[2] = {1.0, 0.88};
    // an N-contiguous B needs a raw staging buffer: only block_n 64 keeps 4 stages
    for (int i = b_n_contiguous ? 1 : 0; i < 2; ++i) {
        const int bn = cand[i];
        const int64_t tiles = cdiv(m, kBlockM) * cdiv(n, bn);
        const int64_t waves = cdiv(tiles, sm_count);
        const double fill = static_cast<double>(tiles) / static_cast<double>(waves * sm_count);
        const double ncov = static_cast<double>(n) / static_cast<double>(cdiv(n, bn) * bn);
        const double score = fill * ncov * mma_eff[i];
        if (score > best_score + 1e-9) {
            best_score = score;
            best.block_n = bn;
            best.tiles = static_cast<int>(tiles);
        }
    }
    best.pair = false;
    best.block_m = kBlockM;
    best.block_k = 32;
    best.stages = b_n_contiguous ? X3Cfg<64, true>::kStages
                                 : (best.block_n == 128 ? X3Cfg<128, false>::kStages : X3Cfg<64, false>::kStages);
    best.ctas = best.tiles < sm_count ? best.tiles : sm_count;
    *plan = best;
    return ST_OK;
}

int launch_gemm_3xtf32(const GemmArgs &g, int sm_count, int *dev_err, uint64_t timeout_ns, cudaStream_t stream) {
    GemmPlan plan;
    ST_TRY(plan_gemm_x3(g.m, g.n, !g.b_k_major, sm_count, &plan));
    for (const void *ptr : {g.a, g.b})
        if (reinterpret_cast<uintptr_t>(ptr) % 16 != 0)
            return fail(ST_ERR_INVALID_ARGUMENT, "tensor-core operands must be 16-byte aligned");
    if ((g.lda * 4) % 16 != 0 || (g.ldb * 4) % 16 != 0)
        return fail(ST_ERR_INVALID_ARGUMENT, "tensor-core operand row strides must be multiples of 16 bytes");
    CUtensorMap ma, mb;
    ST_TRY(make_map(&ma, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, g.a, static_cast<uint64_t>(g.k), static_cast<uint64_t>(g.m),
                    static_cast<uint64_t>(g.lda) * 4, 32, kBlockM));
    if (g.b_k_major) {
        ST_TRY(make_map(&mb, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, g.b, static_cast<uint64_t>(g.k),
                        static_cast<uint64_t>(g.n), static_cast<uint64_t>(g.ldb) * 4, 32, plan.block_n));
    } else {
        ST_TRY(make_map(&mb, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, g.b, static_cast<uint64_t>(g.n),
                        static_cast<uint64_t>(g.k), static_cast<uint64_t>(g.ldb) * 4, 32, 32));
    }
    KParams kp;
    kp.m = static_cast<int>(g.m);
    kp.n = static_cast<int>(g.n);
    kp.k = static_cast<int>(g.k);
    kp.num_m_tiles = static_cast<int>(cdiv(g.m, kBlockM));
    kp.num_n_tiles = static_cast<int>(cdiv(g.n, plan.block_n));
    kp.num_k_blocks = static_cast<int>(cdiv(g.k, 32));
    kp.total_tiles = kp.num_m_tiles * kp.num_n_tiles;
    kp.c = g.c;
    kp.sk_ws = nullptr;
    kp.sk_flags = nullptr;
    kp.sk_mode = 0;
    kp.sk_l2add = 0;
    kp.k_snake = 0;
    kp.staged = 0;  // direct stores
    kp.n_peers = g.peers.n;
    for (int i = 0; i < kMaxPeers; ++i) kp.c_peers[i] = i < g.peers.n ? g.peers.base[i] : nullptr;
    kp.ldc = g.ldc;
    kp.c_dtype = g.c_dtype;
    kp.bias = g.bias;
    kp.bias_dtype = g.bias_dtype;
    kp.err = dev_err;
    kp.timeout_ns = timeout_ns;
    if (!g.b_k_major) return launch_x3_instance<true, 64>(ma, mb, kp, plan.ctas, stream);
    if (plan.block_n == 128) return launch_x3_instance<false, 128>(ma, mb, kp, plan.ctas, stream);
    return launch_x3_instance<false, 64>(ma, mb, kp, plan.ctas, stream);
}

// Stream-K mode of the CTA-pair kernel (stream_k_split) set by
// SPTILES_B200_STREAM_K: 0 whole tiles only, 1 only problems with fewer
// tiles than pairs, 2 also partial last waves; -1 when unset.
int stream_k_env() {
    const char *v = std::getenv("SPTILES_B200_STREAM_K");
    if (v != nullptr && v[0] == '0') return 0;
    if (v != nullptr && v[0] == '1') return 1;
    if (v != nullptr && v[0] == '2') return 2;
    return -1;
}

// The mode plan_gemm scores with when it knows nothing about C.
int stream_k_mode() {
    const int env = stream_k_env();
    return env >= 0 ? env : 1;
}

// two slots per pair (a stream-K range covers at most two tiles), each with
// both CTAs' 128 x 256 fp32 and a flag per epilogue warp and CTA
size_t stream_k_flag_offset(int sm_count) {
    const int pairs = (sm_count > 0 ? sm_count : 148) / 2;
    return static_cast<size_t>(pairs) * 2 * 2 * kPairN * kBlockM * sizeof(float);
}

size_t stream_k_workspace_bytes(int sm_count) {
    const int pairs = (sm_count > 0 ? sm_count : 148) / 2;
    return stream_k_flag_offset(sm_count) + static_cast<size_t>(pairs) * 2 * 2 * kEpilogueWarps * sizeof(int);
}

int plan_gemm(int in_dtype, int64_t m, int64_t n, int64_t k, int sm_count, GemmPlan *plan, int sk_mode,
              bool force_pair) {
    if (sk_mode < 0) sk_mode = stream_k_mode();
    if (m <= 0 || n <= 0 || k <= 0) return fail(ST_ERR_INVALID_ARGUMENT, "matmul extents must be positive");
    if (sm_count <= 0) sm_count = 148;
    // SPTILES_B200_GEMM_KERNEL=pair|single pins the kernel family (tests use it
    // to cover both on every shape); unset, the scores below decide
    const char *force = std::getenv("SPTILES_B200_GEMM_KERNEL");
    const bool only_pair = force_pair || (force && std::strcmp(force, "pair") == 0);
    const bool only_single = !force_pair && force && std::strcmp(force, "single") == 0;
    GemmPlan best;
    double best_score = -1.0;
    // one CTA per SM: block 128 x {256, 128, 64}; relative tensor-pipe
    // efficiency of narrower MMA shapes (wider N reuses A more)
    const int cand[3] = {256, 128, 64};
    const double mma_eff[3] = {1.0, 0.93, 0.80};
    const double mcov1 = static_cast<double>(m) / static_cast<double>(cdiv(m, kBlockM) * kBlockM);
    for (int i = 0; i < 3; ++i) {
        const int bn = cand[i];
        const int64_t tiles = cdiv(m, kBlockM) * cdiv(n, bn);
        const int64_t waves = cdiv(tiles, sm_count);
        const double fill = static_cast<double>(tiles) / static_cast<double>(waves * sm_count);
        const double ncov = static_cast<double>(n) / static_cast<double>(cdiv(n, bn) * bn);
        const double score = fill * ncov * mcov1 * mma_eff[i];
        if (!only_pair && score > best_score + 1e-9) {
            best_score = score;
            best.pair = false;
            best.block_m = kBlockM;
            best.block_n = bn;
            best.tiles = static_cast<int>(tiles);
        }
    }
    // CTA pairs: 256 x 256 per pair, half the staged B bytes per SM; a
    // partial last wave goes out as a stream-K tail (whole-tile fill otherwise)
    {
        const int pairs = sm_count / 2;
        const int64_t tiles = cdiv(m, 2 * kBlockM) * cdiv(n, kPairN);
        const int64_t waves = cdiv(tiles, pairs);
        double fill = static_cast<double>(tiles) / static_cast<double>(waves * pairs);
        const int kb = static_cast<int>(cdiv(k, in_dtype == ST_F32 ? 32 : 64));
        int dp_tiles = 0, sk_pairs = 0;
        long long sk_iters = 0;
        if (tiles < (int64_t(1) << 30))
            stream_k_split(static_cast<int>(tiles), pairs, kb, sk_mode, dp_tiles, sk_pairs, sk_iters);
        if (sk_pairs > 0) {
            // per pair: whole tiles, its tail range, ~6 K blocks of partial store / fold
            const double work = static_cast<double>(dp_tiles / pairs) * kb +
                                static_cast<double>((sk_iters + sk_pairs - 1) / sk_pairs) + 6.0;
            const double ideal = static_cast<double>(tiles) * kb / pairs;
            fill = ideal / work < 1.0 ? ideal / work : 1.0;
        }
        const double ncov = static_cast<double>(n) / static_cast<double>(cdiv(n, kPairN) * kPairN);
        const double mcov = static_cast<double>(m) / static_cast<double>(cdiv(m, 2 * kBlockM) * 2 * kBlockM);
        const double score = fill * ncov * mcov * 1.10;
        if (!only_single && (only_pair || score > best_score + 1e-9)) {
            best_score = score;
            best.pair = true;
            best.block_m = 2 * kBlockM;
            best.block_n = kPairN;
            best.tiles = static_cast<int>(tiles);
        }
    }
    best.block_k = in_dtype == ST_F32 ? 32 : 64;
    if (best.pair) {
        best.stages = PairCfg::kStages;
        // every pair with whole tiles or a stream-K range; with fewer tiles
        // than pairs and a split, exactly the split's pairs (the kernel
        // derives the same split from that grid)
        int pairs = best.tiles < sm_count / 2 ? best.tiles : sm_count / 2;
        int dp_tiles = 0, sk_pairs = 0;
        long long sk_iters = 0;
        stream_k_split(best.tiles, sm_count / 2, static_cast<int>(cdiv(k, best.block_k)), sk_mode, dp_tiles,
                       sk_pairs, sk_iters);
        if (sk_pairs > 0) pairs = dp_tiles > 0 ? sm_count / 2 : sk_pairs;
        best.ctas = 2 * pairs;
    } else {
        best.stages = best.block_n == 256 ? TileCfg<256>::kStages
                                          : (best.block_n == 128 ? TileCfg<128>::kStages : TileCfg<64>::kStages);
        best.ctas = best.tiles < sm_count ? best.tiles : sm_count;
    }
    *plan = best;
    return ST_OK;
}

// The TMA-store epilogue needs every C destination 16-byte aligned with a
// row stride of a multiple of 16 bytes; other C views take the per-lane
// direct stores.  Peer copies always go by TMA store (one asynchronous bulk
// store per box and destination instead of per-lane stores across NVLink);
// a local C does unless SPTILES_B200_C_STORE=direct (or =tma) overrides it.
bool c_store_staged(const GemmArgs &g) {
    const int ces = dtype_size(g.c_dtype);
    if ((g.ldc * ces) % 16 != 0) return false;
    if (reinterpret_cast<uintptr_t>(g.c) % 16 != 0) return false;
    for (int d = 0; d < g.peers.n; ++d)
        if (reinterpret_cast<uintptr_t>(g.peers.base[d]) % 16 != 0) return false;
    if (g.peers.n > 0) return true;
    const char *v = std::getenv("SPTILES_B200_C_STORE");
    if (v != nullptr && std::strcmp(v, "direct") == 0) return false;
    if (v != nullptr && std::strcmp(v, "tma") == 0) return true;
    return ST_C_STORE_DEFAULT != 0;
}

// Whether split tiles of a CTA-pair launch can fold by L2 reduce-add: C is
// fp32, staged and on this GPU only, and the caller accepts sums whose last
// bit depends on the order in which L2 applies the units' adds (not
// ST_EXEC_DETERMINISTIC, not SPTILES_B200_SK_FOLD=exchange).
bool stream_k_l2add_ok(const GemmArgs &g) {
    const char *v = std::getenv("SPTILES_B200_SK_FOLD");
    const bool exchange = v != nullptr && std::strcmp(v, "exchange") == 0;
    return !exchange && !g.deterministic && g.c_dtype == ST_F32 && g.peers.n == 0 && c_store_staged(g);
}

// Stream-K mode of one launch: SPTILES_B200_STREAM_K when set; otherwise 2
// (a partial last wave after whole-tile waves is split too) where split
// tiles fold by L2 reduce-add -- the tail then costs a preset of its tiles
// and one reduce-add per unit -- and 1 where they would fold by exchange,
// which on a tail measured slower than leaving the last wave partial.
int stream_k_mode_for(const GemmArgs &g) {
    const int env = stream_k_env();
    if (env >= 0) return env;
    return stream_k_l2add_ok(g) ? 2 : 1;
}

// How a CTA-pair launch folds the tiles a stream-K schedule splits:
// kFoldL2Add where stream_k_l2add_ok (units add their partials onto C,
// preset to the bias on the split tiles); kFoldExchange otherwise
// (reduce-scatter through the stream-K workspace, whose sums come out the
// same bit for bit on every run).
int stream_k_fold(const GemmArgs &g, int sm_count) {
    const int mode = stream_k_mode_for(g);
    if (mode <= 0) return kFoldNone;
    GemmPlan plan;
    if (plan_gemm(g.ab_dtype, g.m, g.n, g.k, sm_count, &plan, mode, g.split_fp32) != ST_OK || !plan.pair)
        return kFoldNone;
    if (sm_count <= 0) sm_count = 148;
    int dp = 0, skp = 0;
    long long ski = 0;
    stream_k_split(plan.tiles, sm_count / 2, static_cast<int>(cdiv(g.k, plan.block_k)), mode, dp, skp, ski);
    if (skp == 0) return kFoldNone;
    return stream_k_l2add_ok(g) ? kFoldL2Add : kFoldExchange;
}

// SPTILES_B200_SK_FOLD=preset: the L2 fold presets C even where it would be ordered.
bool sk_ordered_enabled() {
    const char *v = std::getenv("SPTILES_B200_SK_FOLD");
    return !(v != nullptr && std::strcmp(v, "preset") == 0);
}

// The L2 fold of a launch whose split tiles fold by L2 reduce-add (0 when
// they do not): 2, ordered -- a tile's first unit stores, the others add
// after its flags -- when whole-tile waves come before the split tiles, so
// the first units finish long before the last ones and nothing waits; 1,
// every unit adds onto C preset to the bias, when every tile is split: the
// units then finish together, and an ordered fold would put a store, a flag
// and the adds in a row (fp32 1024^3: 27 vs 22 us per call).
int stream_k_l2add_mode(const GemmArgs &g, int sm_count) {
    if (stream_k_fold(g, sm_count) != kFoldL2Add) return 0;
    if (!sk_ordered_enabled()) return 1;
    GemmPlan plan;
    const int mode = stream_k_mode_for(g);
    if (plan_gemm(g.ab_dtype, g.m, g.n, g.k, sm_count, &plan, mode, g.split_fp32) != ST_OK) return 1;
    if (sm_count <= 0) sm_count = 148;
    int dp = 0, skp = 0;
    long long ski = 0;
    stream_k_split(plan.tiles, sm_count / 2, static_cast<int>(cdiv(g.k, plan.block_k)), mode, dp, skp, ski);
    return dp > 0 ? 2 : 1;
}

// Whether launch_gemm uses the stream-K workspace: the exchange folds
// through its partials and flags, the ordered L2 fold through its flags (the
// workspace is only acquired then, so other calls put no event between
// their launches).
bool gemm_uses_stream_k(const GemmArgs &g, int sm_count) {
    const int fold = stream_k_fold(g, sm_count);
    return fold == kFoldExchange || (fold == kFoldL2Add && stream_k_l2add_mode(g, sm_count) == 2);
}

// C[r, q] = 0 + bias[q] (0 without a bias) for r < m, q < n: the value the
// split units of an L2-add stream-K launch add their partial tiles onto.
// Rows start 16-byte aligned (the staged-C rule), so every full group of
// four columns goes out as one 16-byte store.
__global__ void __launch_bounds__(256) c_init_f32_kernel(float *c, long long ldc, const void *bias, int bias_dtype,
                                                         int m, int n) {
    pdl_wait();
    const int n4 = n >> 2;
    for (int r = blockIdx.x; r < m; r += gridDim.x) {
        float *row = c + static_cast<long long>(r) * ldc;
        for (int q = threadIdx.x; q < n4; q += blockDim.x) {
            float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            if (bias != nullptr) {
                v.x = 0.0f + load_bias(bias, bias_dtype, 4 * q);
                v.y = 0.0f + load_bias(bias, bias_dtype, 4 * q + 1);
                v.z = 0.0f + load_bias(bias, bias_dtype, 4 * q + 2);
                v.w = 0.0f + load_bias(bias, bias_dtype, 4 * q + 3);
            }
            reinterpret_cast<float4 *>(row)[q] = v;
        }
        for (int q = 4 * n4 + static_cast<int>(threadIdx.x); q < n; q += blockDim.x)
            row[q] = bias != nullptr ? 0.0f + load_bias(bias, bias_dtype, q) : 0.0f;
    }
    pdl_trigger();
}

int launch_c_init_f32(const GemmArgs &g, int sm_count, cudaStream_t stream) {
    const int64_t blocks = g.m < 8LL * sm_count ? g.m : 8LL * sm_count;
    ST_CUDA_TRY(launch_kernel(c_init_f32_kernel, static_cast<unsigned>(blocks), 256, 0, stream,
                              static_cast<float *>(g.c), static_cast<long long>(g.ldc), g.bias, g.bias_dtype,
                              static_cast<int>(g.m), static_cast<int>(g.n)));
    note_launch();
    const cudaError_t e = cudaPeekAtLastError();
    return e == cudaSuccess ? ST_OK : cuda_fail(cudaGetLastError(), "c_init_f32_kernel launch");
}

int preload_gemm_tf32_kernels() {
    cudaFuncAttributes attr;
    ST_CUDA_TRY(cudaFuncGetAttributes(&attr, gemm_tc_pair_kernel<2, false>));
    ST_CUDA_TRY(cudaFuncGetAttributes(&attr, gemm_tc_kernel<2, false, 256>));
    ST_CUDA_TRY(cudaFuncGetAttributes(&attr, gemm_tc_kernel<2, false, 128>));
    ST_CUDA_TRY(cudaFuncGetAttributes(&attr, gemm_tc_kernel<2, false, 64>));
    ST_CUDA_TRY(cudaFuncGetAttributes(&attr, c_init_f32_kernel));
    ST_CUDA_TRY(cudaFuncGetAttributes(&attr, c_init_tiles_f32_kernel));
    return ST_OK;
}

bool gemm_split_fp32_fits(const GemmArgs &g, int sm_count) {
    // where the packed route (K' = 3 roundup(K, 32)) would run CTA pairs, the
    // same kernel splitting in shared memory does the same MMAs without the pack
    GemmPlan plan;
    if (plan_gemm(ST_F32, g.m, g.n, 3 * tf32_packed_k(g.k), sm_count, &plan, stream_k_mode_for(g)) != ST_OK ||
        !plan.pair)
        return false;
    for (const void *ptr : {g.a, g.b})
        if (reinterpret_cast<uintptr_t>(ptr) % 16 != 0) return false;
    return (g.lda * 4) % 16 == 0 && (g.ldb * 4) % 16 == 0;
}

// SPTILES_B200_K_SNAKE=0 keeps every tile's K order ascending.
bool k_snake_enabled() {
    const char *v = std::getenv("SPTILES_B200_K_SNAKE");
    return !(v != nullptr && v[0] == '0');
}

int launch_gemm(const GemmArgs &g, int sm_count, int *dev_err, uint64_t timeout_ns, cudaStream_t stream) {
    GemmPlan plan;
    // the packed tf32 K already includes the 3x expansion; plan on the product extents
    const int sk_mode = stream_k_mode_for(g);
    ST_TRY(plan_gemm(g.ab_dtype, g.m, g.n, g.k, sm_count, &plan, sk_mode, g.split_fp32));
    const bool tf32 = g.ab_dtype == ST_F32;
    const int elem = tf32 ? 4 : 2;
    const int bk = kRowBytes / elem;
    if (g.split_fp32 && (!tf32 || !plan.pair))
        return fail(ST_ERR_UNSUPPORTED, "the in-kernel 3xTF32 split runs on the CTA-pair kernel only");
    if (g.b_k_major == false && tf32 && !g.split_fp32)
        return fail(ST_ERR_UNSUPPORTED, "tf32 B operand must be K-major");
    for (const void *p : {g.a, g.b})
        if (reinterpret_cast<uintptr_t>(p) % 16 != 0)
            return fail(ST_ERR_INVALID_ARGUMENT, "tensor-core operands must be 16-byte aligned");
    if ((g.lda * elem) % 16 != 0 || (g.ldb * elem) % 16 != 0)
        return fail(ST_ERR_INVALID_ARGUMENT, "tensor-core operand row strides must be multiples of 16 bytes");
    const CUtensorMapDataType dt = tf32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                        : (g.ab_dtype == ST_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                                : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16);
    CUtensorMap ma, mb;
    ST_TRY(make_map(&ma, dt, g.a, static_cast<uint64_t>(g.k), static_cast<uint64_t>(g.m),
                    static_cast<uint64_t>(g.lda) * elem, bk, kBlockM));
    if (g.b_k_major) {
        ST_TRY(make_map(&mb, dt, g.b, static_cast<uint64_t>(g.k), static_cast<uint64_t>(g.n),
                        static_cast<uint64_t>(g.ldb) * elem, bk, plan.pair ? kPairHalfN : plan.block_n));
    } else {
        // N-contiguous B: boxes of 64 16-bit columns, or (raw fp32 for the
        // in-kernel split) 32 columns of 128 bytes x 32 K rows
        ST_TRY(make_map(&mb, dt, g.b, static_cast<uint64_t>(g.n), static_cast<uint64_t>(g.k),
                        static_cast<uint64_t>(g.ldb) * elem, g.split_fp32 ? 32 : 64, bk));
    }
    KParams kp;
    kp.m = static_cast<int>(g.m);
    kp.n = static_cast<int>(g.n);
    kp.k = static_cast<int>(g.k);
    kp.num_m_tiles = static_cast<int>(cdiv(g.m, kBlockM));
    kp.num_n_tiles = static_cast<int>(cdiv(g.n, plan.block_n));
    kp.num_k_blocks = static_cast<int>(cdiv(g.k, bk));
    kp.total_tiles = kp.num_m_tiles * kp.num_n_tiles;
    kp.c = g.c;
    kp.n_peers = g.peers.n;
    for (int i = 0; i < kMaxPeers; ++i) kp.c_peers[i] = i < g.peers.n ? g.peers.base[i] : nullptr;
    kp.ldc = g.ldc;
    kp.c_dtype = g.c_dtype;
    kp.bias = g.bias;
    kp.bias_dtype = g.bias_dtype;
    kp.err = dev_err;
    kp.timeout_ns = timeout_ns;
    const int fold = plan.pair ? stream_k_fold(g, sm_count) : kFoldNone;
    kp.sk_mode = sk_mode;
    // the ordered L2 fold needs the stream-K flags; without them (or with C
    // already preset by the caller) every unit adds onto a preset C
    kp.sk_l2add = 0;
    if (fold == kFoldL2Add)
        kp.sk_l2add = stream_k_l2add_mode(g, sm_count) == 2 && g.sk_flags != nullptr && !g.c_preset ? 2 : 1;
    kp.k_snake = k_snake_enabled() ? 1 : 0;
    kp.sk_ws = fold == kFoldExchange ? g.sk_ws : nullptr;
    kp.sk_flags = fold != kFoldNone ? g.sk_flags : nullptr;
    CStoreMaps cm;
    std::memset(&cm, 0, sizeof(cm));
    kp.staged = 0;
    if (c_store_staged(g)) {
        const CUtensorMapDataType cdt = g.c_dtype == ST_F32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                                            : (g.c_dtype == ST_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                                                   : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16);
        const int ces = dtype_size(g.c_dtype);
        for (int d = 0; d <= g.peers.n; ++d)
            ST_TRY(make_map(&cm.map[d], cdt, d == 0 ? g.c : g.peers.base[d - 1], static_cast<uint64_t>(g.n),
                            static_cast<uint64_t>(g.m), static_cast<uint64_t>(g.ldc) * ces, 128 / ces, 32));
        kp.staged = 1;
    }
    if (plan.pair) {
        const int pairs = plan.ctas / 2;
        const GemmArgs *preset = kp.sk_l2add == 1 && !g.c_preset ? &g : nullptr;
        const int sms = sm_count > 0 ? sm_count : 148;
        if (g.ab_dtype == ST_F16)
            return g.b_k_major ? launch_pair<0, false>(ma, mb, kp, cm, pairs, preset, sms, stream)
                               : launch_pair<0, true>(ma, mb, kp, cm, pairs, preset, sms, stream);
        if (g.ab_dtype == ST_BF16)
            return g.b_k_major ? launch_pair<1, false>(ma, mb, kp, cm, pairs, preset, sms, stream)
                               : launch_pair<1, true>(ma, mb, kp, cm, pairs, preset, sms, stream);
        if (g.split_fp32)
            return g.b_k_major ? launch_pair<2, false, true>(ma, mb, kp, cm, pairs, preset, sms, stream)
                               : launch_pair<2, true, true>(ma, mb, kp, cm, pairs, preset, sms, stream);
        return launch_pair<2, false>(ma, mb, kp, cm, pairs, preset, sms, stream);
    }
    if (g.ab_dtype == ST_F16) {
        return g.b_k_major ? dispatch_bn<0, false>(plan.block_n, ma, mb, kp, cm, plan.ctas, stream)
                           : dispatch_bn<0, true>(plan.block_n, ma, mb, kp, cm, plan.ctas, stream);
    }
    if (g.ab_dtype == ST_BF16) {
        return g.b_k_major ? dispatch_bn<1, false>(plan.block_n, ma, mb, kp, cm, plan.ctas, stream)
                           : dispatch_bn<1, true>(plan.block_n, ma, mb, kp, cm, plan.ctas, stream);
    }
    return dispatch_bn<2, false>(plan.block_n, ma, mb, kp, cm, plan.ctas, stream);
}

}  // namespace st

extern "C" int st_tile_raster(int64_t m, int64_t n, int64_t tm, int64_t tn, int64_t group_m, int64_t bid,
                              int64_t *bid_m, int64_t *bid_n) {
    if (m <= 0 || n <= 0 || tm <= 0 || tn <= 0 || group_m <= 0 || bid < 0 || !bid_m || !bid_n)
        return st::fail(ST_ERR_INVALID_ARGUMENT, "st_tile_raster: extents must be positive");
    const int64_t num_m = st::cdiv(m, tm), num_n = st::cdiv(n, tn);
    if (bid >= num_m * num_n) return st::fail(ST_ERR_INVALID_ARGUMENT, "st_tile_raster: bid out of range");
    st::tile_raster(num_m, num_n, group_m, bid, *bid_m, *bid_n);
    return ST_OK;
}

extern "C" int st_stream_k_split(int32_t tiles, int32_t pairs, int32_t k_blocks, int32_t *dp_tiles,
                                 int32_t *sk_pairs, int64_t *sk_iters) {
    if (tiles < 0 || pairs <= 0 || k_blocks <= 0 || !dp_tiles || !sk_pairs || !sk_iters)
        return st::fail(ST_ERR_INVALID_ARGUMENT, "st_stream_k_split: tiles >= 0, pairs and k_blocks > 0");
    int dp = 0, skp = 0;
    long long ski = 0;
    st::stream_k_split(tiles, pairs, k_blocks, st::stream_k_mode(), dp, skp, ski);
    *dp_tiles = dp;
    *sk_pairs = skp;
    *sk_iters = ski;
    return ST_OK;
}

extern "C" int st_matmul_plan(int32_t in_dtype, int64_t m, int64_t n, int64_t k, int32_t sm_count, int32_t *block_m,
                              int32_t *block_n, int32_t *block_k, int32_t *stages, int32_t *ctas) {
    if (in_dtype != ST_F32 && in_dtype != ST_F16 && in_dtype != ST_BF16)
        return st::fail(ST_ERR_INVALID_ARGUMENT, "st_matmul_plan: in_dtype must be ST_F32, ST_F16 or ST_BF16");
    st::GemmPlan plan;
    const int64_t keff = in_dtype == ST_F32 ? 3 * st::tf32_packed_k(k) : k;
    ST_TRY(st::plan_gemm(in_dtype, m, n, keff, sm_count, &plan));
    if (block_m) *block_m = plan.block_m;
    if (block_n) *block_n = plan.block_n;
    if (block_k) *block_k = plan.block_k;
    if (stages) *stages = plan.stages;
    if (ctas) *ctas = plan.ctas;
    return ST_OK;
}
