// common.h -- shared host-side declarations of the runtime: status helpers,
// the kernel launchers each .cu file provides, and tensor-view utilities.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <string>
#include <utility>

#include "../../include/sptiles_b200.h"

namespace st {

// Record `msg` as the calling thread's last error and return `code`.
int fail(int code, const std::string &msg);
// Map a CUDA error to ST_ERR_CUDA / ST_ERR_OUT_OF_MEMORY with a message.
int cuda_fail(cudaError_t e, const char *what);

#define ST_CUDA_TRY(expr)                                        \
    do {                                                         \
        cudaError_t st_e_ = (expr);                              \
        if (st_e_ != cudaSuccess) return ::st::cuda_fail(st_e_, #expr); \
    } while (0)

#define ST_TRY(expr)                 \
    do {                             \
        int st_rc_ = (expr);         \
        if (st_rc_ != ST_OK) return st_rc_; \
    } while (0)

inline int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }

// ---- programmatic dependent launch
// Every kernel of this library is launched with programmatic stream
// serialisation (launch_kernel) and waits (pdl_wait) until the previous
// kernel on the stream has completed and its memory is visible before it
// touches global memory; only code before that -- barrier set-up, TMEM
// allocation, tensor-map prefetch -- overlaps the predecessor.  pdl_trigger
// lets the next kernel start launching: the GEMMs do it at once (one CTA per
// SM, so a successor's CTAs only take SMs this grid has left), the streaming
// kernels after their loop (their successors' CTAs would otherwise sit
// resident beside them).  SPTILES_B200_PDL=0 launches without the attribute.
#ifdef __CUDACC__
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_begin() {
    pdl_trigger();
    pdl_wait();
}
#endif

bool pdl_enabled();

template <typename... KArgs, typename... Args>
inline cudaError_t launch_kernel(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                                 Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// Process-wide count of kernel launches issued by this library.
void note_launch(uint64_t n = 1);

inline size_t dtype_size(int dtype) {
    switch (dtype) {
    case ST_F32: return 4;
    case ST_F16: return 2;
    case ST_BF16: return 2;
    case ST_I32: return 4;
    default: return 0;
    }
}

// Error word each kernel with bounded waits may set (one int per device).
// Codes written by kernels:
constexpr int kDevAbortGemmProducer = 0x101;
constexpr int kDevAbortGemmMma = 0x102;
constexpr int kDevAbortGemmEpilogue = 0x103;
constexpr int kDevAbortGemmStreamK = 0x104;  // a split tile's partial never arrived
constexpr int kDevAbortWaitCheckBarrier = 0x1f0;  // st_check_device_wait: mbarrier wait ran out
constexpr int kDevAbortWaitCheckFlag = 0x1f1;     // st_check_device_wait: flag poll ran out

// One warp waits (bounded by limit_ns) on an mbarrier nothing arrives on
// (kind 0) or a flag nothing sets (kind 1), then records its abort code in
// dev_err and returns (diag.cu).
int launch_wait_check(int kind, uint64_t limit_ns, int *dev_err, cudaStream_t stream);

// ---- launchers (implemented in vecadd.cu, gemm.cu, pack.cu) ----

// C[i] = A[i] + B[i] for i in [0, n), element strides sa, sb, sc.
int launch_vector_add_1d(const float *a, int64_t sa, const float *b, int64_t sb, float *c, int64_t sc, int64_t n,
                         int sm_count, cudaStream_t stream);
// C[r, q] = A[r, q] + B[r, q] for r < rows, q < cols with 2D element strides.
int launch_vector_add_2d(const float *a, const int64_t sa[2], const float *b, const int64_t sb[2], float *c,
                         const int64_t sc[2], int64_t rows, int64_t cols, int sm_count, cudaStream_t stream);

// C = fma(A, B, D) elementwise (f32), 2D strides; a rank-1 view is one row.
int launch_vector_fma(const float *a, const int64_t sa[2], const float *b, const int64_t sb[2], const float *d,
                      const int64_t sd[2], float *c, const int64_t sc[2], int64_t rows, int64_t cols, int sm_count,
                      cudaStream_t stream);
// C = A converted to C's dtype (ST_F32 / ST_F16 / ST_BF16), 2D strides.
int launch_cast(const void *a, int a_dtype, const int64_t sa[2], void *c, int c_dtype, const int64_t sc[2],
                int64_t rows, int64_t cols, int sm_count, cudaStream_t stream);

// Tensor-core GEMM plan.
struct GemmPlan {
    bool pair = false;  // CTA-pair kernel (cta_group::2): block_m 256, block_n 256
    int block_m = 128;
    int block_n = 256;
    int block_k = 64;  // elements per pipeline stage (128 bytes of K)
    int stages = 4;
    int ctas = 148;
    int tiles = 0;
};

// sk_mode: the stream-K mode to score a partial last wave with (-1: the
// environment's, else 1); force_pair: the CTA-pair plan whatever the scores
int plan_gemm(int in_dtype, int64_t m, int64_t n, int64_t k, int sm_count, GemmPlan *plan, int sk_mode = -1,
              bool force_pair = false);

// D = A' B'^T-style tensor-core GEMM on operands already laid out for TMA:
//   A: [M, K] row-major (K contiguous) of `ab_dtype` (ST_F16 / ST_BF16, or
//      ST_F32 meaning tf32 operands), row stride lda elements.
//   B: if b_k_major, [N, K] row-major (K contiguous), row stride ldb;
//      else [K, N] row-major (N contiguous), row stride ldb.
//   C: [M, N] with row stride ldc, element type c_dtype; bias[N] optional.
// Other GPUs' copies of C (CUDA IPC mappings over NVLink): the epilogue
// writes every finished chunk to each of them at the same offset as locally.
constexpr int kMaxPeers = 7;
struct PeerOutputs {
    void *base[kMaxPeers] = {};  // element (0, 0) of this call's C in each peer's copy
    int n = 0;
};

struct GemmArgs {
    PeerOutputs peers;
    int ab_dtype;
    const void *a;
    int64_t lda;
    const void *b;
    int64_t ldb;
    bool b_k_major;
    void *c;
    int64_t ldc;
    int c_dtype;
    const void *bias;
    int bias_dtype;
    int64_t m, n, k;
    // stream-K tail of the CTA-pair kernel (null: whole tiles only); sized by
    // stream_k_workspace_bytes, flags zero when idle
    float *sk_ws = nullptr;
    int *sk_flags = nullptr;
    // C already holds 0 + bias everywhere (the pack kernel preset it): an
    // L2-add stream-K launch then skips its own preset of the split tiles
    bool c_preset = false;
    // fold split tiles in a fixed order (ST_EXEC_DETERMINISTIC)
    bool deterministic = false;
    // ab_dtype ST_F32 with raw fp32 A [M, K] and B (K-major [N, K] or
    // N-contiguous [K, N]) and the true K: the CTA-pair kernel splits the
    // tiles into tf32 hi / lo itself (3xTF32); only when gemm_split_fp32_fits
    bool split_fp32 = false;
};
// Whether launch_gemm can take these fp32 operands raw (split_fp32): the
// plan picks the CTA-pair kernel and TMA can address A and B in place.
bool gemm_split_fp32_fits(const GemmArgs &args, int sm_count);
// Partial accumulators (one 256 x 256 fp32 tile per CTA pair) and arrival
// flags of the stream-K tail, for up to sm_count / 2 pairs.
size_t stream_k_workspace_bytes(int sm_count);
// True when launch_gemm folds split tiles through that workspace (an fp32 C
// of this GPU alone takes TMA reduce-adds instead and needs none).
bool gemm_uses_stream_k(const GemmArgs &args, int sm_count);
// How launch_gemm folds the tiles a stream-K schedule splits.
enum : int { kFoldNone = 0, kFoldExchange = 1, kFoldL2Add = 2 };
int stream_k_fold(const GemmArgs &args, int sm_count);
// For kFoldL2Add: 2 when split tiles fold ordered (needs the stream-K
// flags), 1 when C must hold 0 + bias first; 0 for other folds.
int stream_k_l2add_mode(const GemmArgs &args, int sm_count);
size_t stream_k_flag_offset(int sm_count);
int launch_gemm(const GemmArgs &args, int sm_count, int *dev_err, uint64_t timeout_ns, cudaStream_t stream);
// fp32 A and B used in place (TMA-addressable): the split into tf32 hi/lo
// happens in shared memory inside the kernel (args.ab_dtype must be ST_F32,
// args.k the true K).
int plan_gemm_x3(int64_t m, int64_t n, bool b_n_contiguous, int sm_count, GemmPlan *plan);
int launch_gemm_3xtf32(const GemmArgs &args, int sm_count, int *dev_err, uint64_t timeout_ns, cudaStream_t stream);

// 3xTF32 operand preparation.  x = hi + lo with hi, lo tf32-exact.
//   A [M, K] (strides sa0, sa1) -> Ap [M, 3*kp] = [hi | hi | lo], kp = round_up(K, 32)
//   B [K, N] (strides sb0, sb1) -> Bp [N, 3*kp] = [hi | lo | hi] (K contiguous)
// so that Ap @ Bp^T = hi*hi + hi*lo + lo*hi.
int64_t tf32_packed_k(int64_t k);
int launch_pack_a_tf32(const float *a, int64_t sa0, int64_t sa1, int64_t m, int64_t k, float *ap, int64_t kp,
                       cudaStream_t stream);
int launch_pack_b_tf32(const float *b, int64_t sb0, int64_t sb1, int64_t k, int64_t n, float *bp, int64_t kp,
                       cudaStream_t stream);
// CUDA places a kernel's code on the device at its first launch (lazy
// loading); these place the 3xTF32 path's packing and GEMM kernels on the
// current device now, for a caller that must make every device allocation
// of the library up front.
int preload_pack_tf32_kernels();
int preload_gemm_tf32_kernels();
// C[r, q] = 0 + bias[q] (or 0) for r < m, q < n, fp32, rows 16-byte aligned:
// the starting value of an L2-add stream-K launch (c == nullptr: nothing)
struct CPreset {
    float *c = nullptr;
    long long ldc = 0;
    const void *bias = nullptr;
    int bias_dtype = ST_F32;
    int m = 0, n = 0;
};
// both in one launch (B's transposing blocks first, then A's rows, whose
// blocks also write `preset`'s C when given)
int launch_pack_ab_tf32(const float *a, int64_t sa0, int64_t sa1, int64_t m, const float *b, int64_t sb0,
                        int64_t sb1, int64_t n, int64_t k, float *ap, float *bp, int64_t kp,
                        const CPreset *preset, cudaStream_t stream);
// Copy a 16-bit [rows, cols] matrix with arbitrary element strides into a
// dense row-major [rows, ld] buffer (ld >= cols, padding columns zeroed).
int launch_repack_16(const uint16_t *src, int64_t s0, int64_t s1, int64_t rows, int64_t cols, uint16_t *dst,
                     int64_t ld, cudaStream_t stream);

}  // namespace st
