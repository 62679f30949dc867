// Launchers of the SpMM kernels (one translation unit each), called by the C ABI.
#pragma once
#include <cuda_runtime.h>

#include "common.cuh"

namespace vcsrmc {
namespace dev {

// FP32 format, fp32 B, CUDA-core FFMA, C += A*B through vector reductions.
cudaError_t spmm_fp32_atomic(const DeviceFormatView& F, const float* B, int64_t ldb, int O, int tileK, float* C,
                             int64_t ldc, cudaStream_t st);

// FP16 format, B fp16 (b_is_f16 = 1, staged by TMA when aligned) or fp32 (converted while
// staging), tcgen05 MMA with fp32 accumulators in tensor memory, C += scale * A*B through
// vector reductions.
cudaError_t spmm_fp16_tc_atomic(const DeviceFormatView& F, const void* B, int b_is_f16, int64_t ldb, int O,
                                int tileK, float* C, int64_t ldc, cudaStream_t st);

// Dense U(-1,1) generator (same stream as the host generator).
cudaError_t gen_dense_device(int64_t rows, int cols, uint64_t seed, int f16, void* out, int64_t ld,
                             cudaStream_t st);

}  // namespace dev
}  // namespace vcsrmc
