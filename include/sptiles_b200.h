/*
 * sptiles_b200.h -- C ABI of the B200 (sm_100a) backend for the two cuda_tile
 * workloads that spTiles compiles: the elementwise tile add (vector_add, 1D
 * and 2D) and the tiled mmaf matmul.
 *
 * Plain C types only: pointers, sizes, int status codes.  No C++ exceptions
 * and no framework types cross this boundary.  Every function returns an
 * ST_* status; st_last_error() gives the message of the calling thread's
 * last failure.  One host thread drives one context.
 *
 * What each group replaces in the reference (paths within the spTiles tree):
 *   context / buffers  src/examples.cpp:133-174 (create_vulkan_context),
 *                      232-269 (create_host_buffer, upload_*, download_*),
 *                      186-230 (destroy_buffer / destroy_vulkan_context)
 *   st_launch          src/examples.cpp:271-448 (run_compute) and
 *                      shaders/spirv_runtime.py:153-174 (run_spirv_kernel):
 *                      a named kernel, a grid and ordered buffer bindings
 *   st_vector_add      shaders/spirv_vector_add.py:44-92 (spirv_vector_add)
 *   st_matmul          shaders/spirv_matmul.py:48-113 (spirv_matmul,
 *                      cutile_matmul_spirv) and shaders/matmul.py:181-253
 *                      (cutile_matmul)
 *   *_host variants    the same calls on host memory, as the reference's
 *                      Python API copies through the CPU (spirv_vector_add.py
 *                      :37,89-92; spirv_runtime.py:162-173)
 */
#ifndef SPTILES_B200_H
#define SPTILES_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes (replace VK_CHECK's std::runtime_error, examples.cpp:12-20) ---- */
#define ST_OK 0
#define ST_ERR_INVALID_ARGUMENT 1 /* bad shape, stride, dtype, size or null pointer */
#define ST_ERR_UNKNOWN_ENTRY 2    /* no kernel registered under that entry name */
#define ST_ERR_UNSUPPORTED 3      /* valid request this backend does not implement */
#define ST_ERR_CUDA 4             /* a CUDA runtime/driver call failed */
#define ST_ERR_NO_DEVICE 5        /* no usable sm_100 device */
#define ST_ERR_OUT_OF_MEMORY 6
#define ST_ERR_TIMEOUT 7          /* a bounded host wait ran out */
#define ST_ERR_DEVICE_ABORT 8     /* a kernel's bounded on-device wait ran out */

/* ---- element types ---- */
#define ST_F32 0
#define ST_F16 1
#define ST_BF16 2
#define ST_I32 3

/* ---- binding kinds of st_param ---- */
#define ST_PARAM_BUFFER 0 /* data pointer of one array (spirv StorageBuffer f32[]) */
#define ST_PARAM_I32 1    /* one i32 scalar: a size, dim, stride or kernel constant */

/* ---- st_exec.flags ---- */
#define ST_EXEC_SYNC 1          /* block (bounded by timeout_ms) until the work is done */
#define ST_EXEC_HOST_BUFFERS 2  /* st_launch only: buffer params are host memory */
#define ST_EXEC_DETERMINISTIC 4 /* matmul: the same inputs give the same bits on every run (split tiles
                                   with fp32 C are folded in a fixed order instead of by L2 adds) */
#define ST_EXEC_ALL_DEVICES 8   /* st_vector_add_host / st_matmul_host, and st_launch with
                                   ST_EXEC_HOST_BUFFERS for the vector_add and matmul entries: the
                                   single-box partitioner in one process -- the call is split over every
                                   device of the context (vector_add by element ranges on 16-byte
                                   boundaries, matmul by 128-row blocks of A and C, B and the bias to
                                   every device), each on the context's own stream (exec->stream NULL,
                                   exec->device -1); returns when all devices are done (bounded by
                                   timeout_ms each).  A split st_launch writes C in place. */

typedef struct st_ctx st_ctx;

/* One binding of the cutile_python_v1 calling convention, in the reference's
 * order: per 1D array (data, size, stride); per 2D array (data, dim0, dim1,
 * stride0, stride1) (spirv_runtime.py:107-128; lower.hpp:197-209, 277-310).
 * Trailing ST_PARAM_I32 entries after the arrays are the kernel's constants
 * (tile sizes), as in ct.launch(..., (A, B, C, tm, tn, tk)) (matmul.py:252). */
typedef struct {
    int32_t kind;   /* ST_PARAM_BUFFER or ST_PARAM_I32 */
    int32_t dtype;  /* buffer element type (ST_F32 / ST_F16 / ST_BF16) */
    void *data;     /* buffer base address */
    uint64_t bytes; /* buffer size in bytes; 0 = not checked */
    int64_t value;  /* ST_PARAM_I32 value */
} st_param;

/* A tensor view: data + shape + strides in elements (rank 1 or 2). */
typedef struct {
    void *data;
    int32_t dtype;
    int32_t rank;
    int64_t shape[2];
    int64_t strides[2];
} st_tensor;

/* A cuda_tile grid: the number of tile blocks along each axis. */
typedef struct {
    uint32_t x, y, z;
} st_grid;

/* Where and how a call runs. */
typedef struct {
    void *stream;                  /* cudaStream_t; NULL = the context's own stream
                                      (pass cudaStreamLegacy, 0x1, for the NULL stream) */
    int32_t device;                /* CUDA ordinal; -1 = the context's first device */
    int32_t flags;                 /* ST_EXEC_* */
    uint32_t timeout_ms;           /* bound for ST_EXEC_SYNC waits; 0 = 60000 */
    const int32_t *output_indices; /* ST_EXEC_HOST_BUFFERS: params copied back */
    int32_t n_outputs;
} st_exec;

/* ---- library ---- */
const char *st_version(void);
const char *st_last_error(void);
/* Number of CUDA devices visible to the process (0 when there is none). */
int st_device_count(int32_t *count);
/* Number of kernels this library has launched in the process so far. */
int st_kernel_launches(uint64_t *count);

/* ---- context: replaces create_vulkan_context / destroy_vulkan_context ---- */
/* devices: CUDA ordinals to use (NULL with n_devices 0 = device 0).  With
 * several devices, peer access between them is enabled (NVLink), so a
 * device's kernels may store into another's memory (st_matmul_allgather
 * with the other devices' copies of C as peers, in one process). */
int st_init(const int32_t *devices, int32_t n_devices, st_ctx **out);
int st_shutdown(st_ctx *ctx);
/* Bounded wait for all work the context issued on `device`; returns
 * ST_ERR_TIMEOUT after timeout_ms, ST_ERR_DEVICE_ABORT if a kernel gave up
 * a bounded wait. */
int st_sync(st_ctx *ctx, int32_t device, uint32_t timeout_ms);
/* The context's stream on `device` (a cudaStream_t). */
int st_stream(st_ctx *ctx, int32_t device, void **stream);

/* ---- device buffers: replace create_host_buffer / upload_* / download_* /
 *      destroy_buffer (examples.cpp:186-269).  The caller owns them. ---- */
int st_alloc(st_ctx *ctx, int32_t device, uint64_t bytes, void **out);
int st_free(st_ctx *ctx, int32_t device, void *ptr);
int st_upload(st_ctx *ctx, int32_t device, void *dst, const void *src, uint64_t bytes);
int st_download(st_ctx *ctx, int32_t device, void *dst, const void *src, uint64_t bytes);

/* ---- launch by entry name: replaces run_compute (examples.cpp:271-448) and
 *      run_spirv_kernel (spirv_runtime.py:153-174).
 * Registered entries (cuda_tile symbol names):
 *   "vector_add"            A,B,C rank 1 f32 (9 params) [+ tile_size]       default tile 1024
 *   "vector_add_2d"         A,B,C rank 2 f32 (15 params) [+ tile_m, tile_n]  default 64 x 64
 *   "matmul_fp32", "matmul_f16", "matmul_bf16"
 *                           A[M,K], B[K,N], C[M,N] rank 2 (15 params) [+ tm, tn, tk]
 *   "matmul_fp32_bias", "matmul_f16_bias", "matmul_bf16_bias"
 *                           as above + bias[N] rank 1 appended (18 params)
 *   "persistent_matmul_fp32", "persistent_matmul_f16", "persistent_matmul_bf16"
 *                           persistent-kernel semantics (matmul.py:106-178):
 *                           any grid >= 1 covers every output tile
 *   "vector_fma"            A,B,D,C rank 1 f32 (12 params) [+ tile_size]: C = fma(A, B, D)
 *   "vector_fma_2d"         A,B,D,C rank 2 f32 (20 params) [+ tile_m, tile_n]
 *   "cast"                  A,C rank 1 (6 params) [+ tile_size]: C = A in C's dtype
 *   "cast_2d"               A,C rank 2 (10 params) [+ tile_m, tile_n]
 * grid counts tile blocks.  A matmul grid must cover every output tile
 * (cdiv(M,tm)*cdiv(N,tn) blocks) unless the entry is persistent; a
 * vector_add grid may cover fewer tiles, and only those are computed. */
int st_launch(st_ctx *ctx, const char *entry_name, const st_grid *grid,
              const st_param *params, int32_t n_params, const st_exec *exec);

/* The reference runners dispatch workgroups of 1024 invocations, one output
 * element each (lower.hpp:277-290; spirv_runtime.py:11).  Convert such a
 * dispatch to the cuda_tile grid of `entry_name` with tile elements
 * `tile_elems`: tiles = cdiv(dx*dy*dz*1024, tile_elems). */
int st_grid_from_dispatch(const char *entry_name, const uint32_t dispatch[3], int64_t tile_elems,
                          st_grid *out);

/* ---- failure path check.  Runs one warp that waits, with the helpers the
 * GEMM kernels' bounded waits use, on something that never completes: an
 * mbarrier nothing arrives on (kind 0) or a GPU-scope flag nothing sets
 * (kind 1).  After limit_us (1 .. 10^7) it gives up, records its abort code
 * in the device's error word and returns; the next bounded host wait
 * (ST_EXEC_SYNC here, or st_sync) reports ST_ERR_DEVICE_ABORT and clears the
 * word, and the context stays usable.  Nothing faults or hangs.  No
 * counterpart in the reference, whose host waits on a fence without a limit
 * (src/examples.cpp:439). */
int st_check_device_wait(st_ctx *ctx, int32_t kind, uint32_t limit_us, const st_exec *exec);

/* ---- cuda_tile modules (TileIR bytecode, .tilebc): entry discovery.
 * Replace the translator's module loading (src/main.cpp:75-104:
 * load_cuda_tile_file, isTileIRBytecode, readBytecode) and its derivation of
 * the launch ABI from each cuda_tile.entry (src/lower.hpp:197-310:
 * replace_entries, convert_entry_type, attach_spirv_abi_attrs -- parameter i
 * is binding i; tile<ptr<T>> is a buffer, tile<i32> an i32 scalar).  Only the
 * entries' symbols and parameter types, their sm_100 hints and the tile
 * shapes of the module's partition views are read; function bodies are
 * skipped, never decoded or run.  Bytecode versions 13.1 to 13.3. */
typedef struct st_module st_module;

#define ST_MODULE_PARAM_BUFFER 0 /* tile<ptr<T>>: the data of an array */
#define ST_MODULE_PARAM_I32 1    /* tile<i32>: a size or stride */
#define ST_MODULE_PARAM_OTHER 2  /* any other parameter type (not launchable here) */

typedef struct {
    const char *name;           /* entry symbol (valid until st_module_free) */
    int32_t n_params;           /* parameters = bindings, in order */
    int32_t n_arrays;           /* cutile_python_v1 array descriptors they form (0: none) */
    int32_t array_rank[8];
    int32_t array_dtype[8];     /* ST_F32 / ST_F16 / ST_BF16, -1 for other element types */
    int32_t n_constants;        /* tile sizes recovered from the module; 0 = not unambiguous */
    int32_t constants[3];       /* vector_add: tile_size (1D) or tile_m, tile_n; matmul: tm, tn, tk */
    int32_t num_cta_in_cga;     /* sm_100 entry hint, 0 when absent */
    int32_t occupancy;          /* sm_100 entry hint, 0 when absent */
    const char *backend_entry;  /* st_launch registry entry serving it; NULL = none */
} st_module_entry_info;

/* Parse a module held in memory (the bytes are not kept). */
int st_module_load(const void *bytes, uint64_t size, st_module **out);
/* Read and parse a .tilebc file (load_cuda_tile_file, main.cpp:87-104; MLIR
 * text input is not accepted). */
int st_module_load_file(const char *path, st_module **out);
int st_module_free(st_module *module);
int st_module_version(const st_module *module, int32_t *major, int32_t *minor, int32_t *tag);
int st_module_entry_count(const st_module *module, int32_t *count);
int st_module_entry(const st_module *module, int32_t index, st_module_entry_info *out);
/* Kind (ST_MODULE_PARAM_*) and element type of one entry parameter. */
int st_module_param(const st_module *module, int32_t entry, int32_t param, int32_t *kind, int32_t *dtype);
/* st_launch of a module entry (run_compute with the module's entry name,
 * examples.cpp:271-448).  entry_name may be NULL for a one-entry module.
 * The bindings must match the entry's parameters in kind and element type;
 * the module's tile sizes are appended unless the caller passes its own as
 * trailing i32 constants (required when n_constants is 0).  The grid counts
 * tile blocks, as for st_launch. */
int st_launch_module(st_ctx *ctx, const st_module *module, const char *entry_name, const st_grid *grid,
                     const st_param *params, int32_t n_params, const st_exec *exec);

/* ---- typed calls (device memory) ---- */
/* C = A + B elementwise over the whole of C (rank 1 or 2, f32, any strides). */
int st_vector_add(st_ctx *ctx, const st_tensor *a, const st_tensor *b, const st_tensor *c,
                  const st_exec *exec);
/* C[M,N] = A[M,K] @ B[K,N] (+ bias[N]); fp32 accumulation.  A and B are
 * both f32 (3xTF32 on the tensor cores), both f16 or both bf16; C is f32,
 * f16 or bf16; bias (may be NULL) is f32 or the input type. */
int st_matmul(st_ctx *ctx, const st_tensor *a, const st_tensor *b, const st_tensor *bias,
              const st_tensor *c, const st_exec *exec);

/* C = fma(A, B, D) elementwise: A*B + D rounded once (f32, rank 1 or 2,
 * any strides) -- the lowering's fma (tileops.hpp:616-623). */
int st_vector_fma(st_ctx *ctx, const st_tensor *a, const st_tensor *b, const st_tensor *d, const st_tensor *c,
                  const st_exec *exec);
/* C = A converted to C's dtype (ST_F32 / ST_F16 / ST_BF16; round to nearest
 * even when narrowing) -- the lowering's ftof (tileops.hpp:257-258). */
int st_cast(st_ctx *ctx, const st_tensor *a, const st_tensor *c, const st_exec *exec);

/* ---- typed calls on host memory: copy in, compute, copy out, all on the
 *      context's stream; returns once C is back in host memory. ---- */
int st_vector_add_host(st_ctx *ctx, const st_tensor *a, const st_tensor *b, const st_tensor *c,
                       const st_exec *exec);
int st_matmul_host(st_ctx *ctx, const st_tensor *a, const st_tensor *b, const st_tensor *bias,
                   const st_tensor *c, const st_exec *exec);

/* ---- one process per GPU: replicated C written by the GEMM epilogue ----
 * The reference runs on one device (examples.cpp:115-131); these calls back
 * the single-box partitioner.  st_ipc_handle exports a device allocation
 * made by st_alloc; st_ipc_open maps another process's allocation on this
 * GPU (over NVLink on the B200 box); st_ipc_close unmaps it.
 * st_matmul_allgather computes C rows [row_offset, row_offset + rows(A)) =
 * A @ B (+ bias) and its epilogue stores every finished chunk both into
 * c_full (this GPU's [M, N] copy) and, over peer memory, into each of the
 * n_peers (<= 7) other copies at the same offset -- the GEMM and the
 * all-gather of C in one kernel (16-bit A/B: TMA stores of 32-row boxes when
 * every copy's base and row stride are 16-byte multiples).  The other ranks'
 * rows arrive in c_full once every rank's call has completed (e.g. after a
 * collective on the same stream); the caller also orders the call after
 * every reader of the previous contents of the other copies.  With K = 0
 * the call returns ST_ERR_UNSUPPORTED. */
int st_ipc_handle(st_ctx *ctx, int32_t device, void *ptr, uint8_t handle[64]);
int st_ipc_open(st_ctx *ctx, int32_t device, const uint8_t handle[64], void **out);
int st_ipc_close(st_ctx *ctx, int32_t device, void *ptr);
int st_matmul_allgather(st_ctx *ctx, const st_tensor *a, const st_tensor *b, const st_tensor *bias,
                        const st_tensor *c_full, void *const *peer_c_full, int32_t n_peers, int64_t row_offset,
                        const st_exec *exec);

/* ---- fp32 matmul that allocates nothing ----
 * No counterpart in the reference.  For callers that must not allocate
 * device memory: a process whose memory pool already holds the GPU's memory,
 * or a latency-critical caller that cannot pay for cudaMalloc / cudaFree
 * (cudaFree waits for the whole device).  Same arithmetic as st_matmul with
 * f32 A and B (3xTF32), but the packed operands live in one fixed
 * ST_STATIC_SCRATCH_BYTES device array inside the library, which every GPU
 * that loads the library holds until the process exits.  Needs no context:
 * exec may be NULL; exec->stream NULL means the legacy default stream.
 *   - (M + N) * 3 * roundup(K, 32) * 4 bytes must fit in the array, else
 *     ST_ERR_INVALID_ARGUMENT; bias, if given, is f32.
 *   - exec->stream, if given, must belong to the call's device.
 *   - The first call on a device is its set-up: CUDA loads modules lazily,
 *     so that call is when the array and the code of the kernels this entry
 *     point launches take their device memory (it places them all at once,
 *     and finds the array's device address).  Later calls allocate nothing.
 *     A caller whose memory pool takes the GPU's memory makes one call per
 *     device before that (any small product), and before any stream capture.
 *   - All calls share the array: calls that overlap on the GPU race.
 *   - A kernel that gives up a bounded wait leaves C incomplete and its code
 *     in this entry point's abort word; the next call made with
 *     ST_EXEC_SYNC returns ST_ERR_DEVICE_ABORT and clears the word (without
 *     ST_EXEC_SYNC nothing is reported until then). */
#define ST_STATIC_SCRATCH_BYTES (32u * 1024u * 1024u)
int st_matmul_static_scratch(const st_tensor *a, const st_tensor *b, const st_tensor *bias, const st_tensor *c,
                             const st_exec *exec);

/* ---- runtime policy, exposed for inspection and tests (no device work) ---- */
/* Tile block (bid_m, bid_n) of tile id `bid` under the GROUP_SIZE_M raster
 * of the cuTile matmul (matmul.py:14-24). */
int st_tile_raster(int64_t m, int64_t n, int64_t tm, int64_t tn, int64_t group_m, int64_t bid,
                   int64_t *bid_m, int64_t *bid_n);
/* The tensor-core tile this runtime picks for a matmul: block_m x block_n x
 * block_k elements, smem pipeline depth, and the CTA count of the persistent
 * launch for a device with `sm_count` SMs. */
int st_matmul_plan(int32_t in_dtype, int64_t m, int64_t n, int64_t k, int32_t sm_count,
                   int32_t *block_m, int32_t *block_n, int32_t *block_k, int32_t *stages,
                   int32_t *ctas);
/* Work split of the CTA-pair matmul kernel for `tiles` 256 x 256 output
 * tiles of `k_blocks` K blocks each on `pairs` CTA pairs: tiles
 * [0, dp_tiles) go out whole (tile t to pair t mod pairs); the remaining
 * tiles' K blocks (sk_iters of them) are split into sk_pairs equal
 * contiguous ranges, range q = [q * sk_iters / sk_pairs, (q + 1) * sk_iters
 * / sk_pairs) on pair pairs - 1 - q (sk_pairs = 0: whole tiles only).  No
 * counterpart in the reference. */
int st_stream_k_split(int32_t tiles, int32_t pairs, int32_t k_blocks, int32_t *dp_tiles, int32_t *sk_pairs,
                      int64_t *sk_iters);
/* Contiguous shard [begin, end) of `total` units for `rank` of `count`
 * ranks, boundaries rounded to multiples of `align` units (vector_add: 4
 * elements = 16 bytes; matmul: M rows). */
int st_shard_range(int64_t total, int32_t count, int32_t rank, int64_t align, int64_t *begin,
                   int64_t *end);

#ifdef __cplusplus
}
#endif

#endif /* SPTILES_B200_H */
