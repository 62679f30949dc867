// Diagnostic of the bounded device waits: one CTA holds tensor memory, waits on an mbarrier phase
// that can never complete, and must give up after the given budget, report the expiry in the
// format's status word and free its tensor memory, as the SpMM kernels do on an expired wait. No
// copy and no MMA is issued, so nothing is in flight when the wait gives up.
#include <cuda_runtime.h>

#include "common.cuh"
#include "wait_check.hpp"

namespace vcsrmc {
namespace dev {
namespace {

constexpr uint32_t kCheckTmemCols = 32;  // the smallest tensor-memory allocation

__global__ void __launch_bounds__(128) bounded_wait_check_kernel(uint32_t* status, long long budget,
                                                                  uint32_t* completed) {
    __shared__ uint64_t bar;
    __shared__ uint32_t tmem_base;
    const int warp = threadIdx.x >> 5;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_mbar_init();
    }
    if (warp == 0) {
        tmem_alloc(&tmem_base, kCheckTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (threadIdx.x == 0) {
        // The one arrival is made, but the phase also waits for 1024 bytes of copies that are
        // never issued: it cannot complete.
        mbar_arrive_expect_tx(&bar, 1024u);
        const bool ok = mbar_wait_bounded(&bar, 0u, budget);
        if (!ok) atomicOr(status, kStatusTimeout);
        *completed = ok ? 1u : 0u;
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0) tmem_dealloc(tmem_base, kCheckTmemCols);
}

}  // namespace

cudaError_t bounded_wait_check(uint32_t* status, long long budget_cycles, uint32_t* completed, cudaStream_t st) {
    bounded_wait_check_kernel<<<1, 128, 0, st>>>(status, budget_cycles, completed);
    return cudaGetLastError();
}

}  // namespace dev
}  // namespace vcsrmc
