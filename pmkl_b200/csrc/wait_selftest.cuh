// wait_selftest.cuh -- a diagnostic kernel that makes one bounded mbarrier
// wait run out on purpose, so that the failure path of the tensor-core kernels
// can be tested without a fault: the same mbar_wait, the same abort flag, the
// same early-exit checks of the device error word and the same clean-up order
// (drain issued tcgen05 work, free tensor memory, then report).
#pragma once

#include "common.cuh"
#include "sm100_ptx.cuh"

namespace pmkl_b200 {
namespace diag {

// Per CTA, out[2 * cta] = outcome (0: the wait completed, 1: it ran out,
// 2: the CTA found the device error word set at start and skipped its work,
// as every tensor-core kernel does), out[2 * cta + 1] = nanoseconds spent
// waiting.  Nothing ever arrives on the barrier, so an unskipped CTA always
// gives up after limit_ns (+ at most one suspend period).
__global__ void __launch_bounds__(128, 1) wait_selftest_kernel(unsigned long long limit_ns,
                                                               unsigned long long *out) {
    using namespace ptx;
    __shared__ uint64_t bar_never;  // no thread and no copy arrives on it
    __shared__ uint64_t bar_drain;
    __shared__ uint32_t tmem_slot;
    __shared__ volatile int abort_flag;
    __shared__ int skip;
    const int warp = threadIdx.x >> 5;
    if (threadIdx.x == 0) {
        mbar_init(&bar_never, 1);
        mbar_init(&bar_drain, 1);
        abort_flag = 0;
        skip = (*reinterpret_cast<volatile unsigned int *>(&g_device_error) != 0u) ? 1 : 0;
        fence_mbarrier_init();
    }
    __syncthreads();
    if (skip) {
        if (threadIdx.x == 0) {
            out[2 * blockIdx.x] = 2;
            out[2 * blockIdx.x + 1] = 0;
        }
        return;
    }
    // Hold tensor memory across the wait, as the attention kernels do.
    if (warp == 0) {
        tmem_alloc(&tmem_slot, 32);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;
    if (threadIdx.x == 0) {
        const unsigned long long t0 = globaltimer();
        const bool ok = mbar_wait(&bar_never, 0, &abort_flag, limit_ns);
        out[2 * blockIdx.x] = ok ? 0 : 1;
        out[2 * blockIdx.x + 1] = globaltimer() - t0;
        // Clean-up of an abandoned CTA: every tcgen05 operation this thread
        // issued completes (none here) before tensor memory is released.
        mma_commit(&bar_drain);
        volatile int never = 0;
        mbar_wait(&bar_drain, 0, &never);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, 32);
    }
    if (threadIdx.x == 0 && abort_flag) report_device_error(PMKL_DEVERR_TIMEOUT);
}

}  // namespace diag
}  // namespace pmkl_b200
