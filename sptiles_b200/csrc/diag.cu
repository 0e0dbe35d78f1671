// diag.cu -- a kernel whose bounded wait cannot complete, for testing the
// device-side failure path without faulting or hanging the GPU.
//
// Every wait in the GEMM kernels is bounded: an mbarrier wait (mbar_wait)
// or a poll of a GPU-scope flag (the stream-K reduce-scatter) gives up after
// a time limit, the giving-up lane records an abort code in the device's
// error word, and the kernel returns; the next bounded host wait reports
// ST_ERR_DEVICE_ABORT and clears the word.  In those kernels the path only
// runs if something has already gone wrong, so this one-warp kernel takes
// it on purpose: it waits, with the same helpers, on an mbarrier that
// nothing arrives on or on a flag that nothing sets.  It holds no TMEM and
// has no copy or MMA in flight when it gives up.
#include <cuda_runtime.h>

#include "common.h"
#include "sm100.cuh"

namespace st {
namespace {

__device__ int g_never_set;  // a flag that no code writes (zero-initialised)

__global__ void __launch_bounds__(32) wait_check_kernel(int kind, uint64_t limit_ns, int *err) {
    __shared__ alignas(8) uint64_t bar;
    __shared__ int abort_flag;
    const int lane = static_cast<int>(threadIdx.x);
    if (lane == 0) {
        abort_flag = 0;
        mbar_init(smem_addr(&bar), 1);  // expects one arrival, which never comes
        fence_barrier_init();
    }
    __syncwarp();
    bool done;
    if (kind == 0) {
        done = mbar_wait(smem_addr(&bar), 0, &abort_flag, limit_ns);
    } else {
        const uint64_t t0 = global_timer_ns();
        for (;;) {
            if (__all_sync(0xffffffffu, ld_acquire_gpu(&g_never_set) >= 1)) {
                done = true;
                break;
            }
            if (__any_sync(0xffffffffu, global_timer_ns() - t0 > limit_ns)) {
                done = false;
                break;
            }
        }
    }
    if (!__all_sync(0xffffffffu, done) && lane == 0) {
        abort_flag = 1;
        atomicExch(err, kind == 0 ? kDevAbortWaitCheckBarrier : kDevAbortWaitCheckFlag);
    }
}

}  // namespace

int launch_wait_check(int kind, uint64_t limit_ns, int *dev_err, cudaStream_t stream) {
    wait_check_kernel<<<1, 32, 0, stream>>>(kind, limit_ns, dev_err);
    note_launch();
    const cudaError_t e = cudaPeekAtLastError();
    return e == cudaSuccess ? ST_OK : cuda_fail(cudaGetLastError(), "wait_check_kernel launch");
}

}  // namespace st
