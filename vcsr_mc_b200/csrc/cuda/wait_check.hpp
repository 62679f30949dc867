// Diagnostic of the bounded device waits (see wait_check.cu).
#pragma once
#include <cuda_runtime.h>

#include <cstdint>

namespace vcsrmc {
namespace dev {

// One CTA allocates tensor memory, waits up to budget_cycles on an mbarrier phase that cannot
// complete, sets kStatusTimeout in *status when the wait expires, frees its tensor memory, and
// writes 1 (the phase completed) or 0 (expired) to *completed (device memory). Asynchronous.
cudaError_t bounded_wait_check(uint32_t* status, long long budget_cycles, uint32_t* completed, cudaStream_t st);

}  // namespace dev
}  // namespace vcsrmc
