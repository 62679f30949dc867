// FP32 VCSR-MC SpMM on CUDA cores (the matched-precision path; B200 has no FP32 tensor core).
//
// Same dataflow and results contract as the reference's vcsr_mc_fp32<NSLAB,SW>
// (src/vcsr_mc.cu:239-329): one CTA per (work item, TK-column slab); the item's B segment
// [seg_base, seg_base + SW) x [k0, k0 + TK) is staged in shared memory once (rows >= N and
// columns >= O read as zero, src/vcsr_mc.cu:279-294); each 16-row group is accumulated in
// fp32 and added into C (C += A * B). Differences: FFMA instead of FP32 MFMA, 128-bit loads
// and stores everywhere, and one 16-byte vector reduction (red.global.add.v4.f32) per
// 4 columns instead of one scalar atomicAdd per column.
//
// Thread layout: TK threads per CTA. Thread t owns group lane row = t / (TK/16) and the
// 16 columns {4*(q + j*TK/16) .. +3 : j < 4}, q = t % (TK/16): a warp covers 4 rows x 32
// consecutive float4 columns, so every shared-memory B read and every C reduction of a warp
// touches whole 128-byte lines.
#include <cuda_runtime.h>

#include "common.cuh"
#include "spmm_launch.hpp"

namespace vcsrmc {
namespace dev {
namespace {

template <int TK, int SW>
__global__ void __launch_bounds__(TK) vcsr_mc_fp32_kernel(DeviceFormatView F, const float* __restrict__ B,
                                                         int64_t ldb, int O, float* __restrict__ C, int64_t ldc,
                                                         int vec_b, int vec_c) {
    constexpr int TPR = TK / 16;  // threads per group row
    extern __shared__ __align__(16) float Bs[];  // SW x TK

    const int item = blockIdx.x;
    const int k0 = blockIdx.y * TK;
    const int2 it = F.items[item];
    const int seg_base = F.gmeta[it.x].z;

    // Stage the B segment (zero outside [0, N) x [0, O)).
    for (int e = threadIdx.x; e < SW * TK / 4; e += TK) {
        const int r = e / (TK / 4), c = (e % (TK / 4)) * 4;
        const int gr = seg_base + r, gc = k0 + c;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (gr < F.N) {
            const float* src = B + int64_t(gr) * ldb + gc;
            if (vec_b && gc + 3 < O) {
                v = __ldg(reinterpret_cast<const float4*>(src));
            } else {
                if (gc < O) v.x = __ldg(src);
                if (gc + 1 < O) v.y = __ldg(src + 1);
                if (gc + 2 < O) v.z = __ldg(src + 2);
                if (gc + 3 < O) v.w = __ldg(src + 3);
            }
        }
        *reinterpret_cast<float4*>(&Bs[r * TK + c]) = v;
    }
    __syncthreads();

    const int row = threadIdx.x / TPR, q = threadIdx.x % TPR;
    const float* __restrict__ val = static_cast<const float*>(F.val);
    for (int g = it.x; g < it.y; ++g) {
        const int4 m = F.gmeta[g];
        float4 acc[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[j] = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int d = 0; d < m.y; ++d) {
            const int s = m.x + d * 16 + row;
            const int lc = F.lcol[s];
            const float a = __ldg(val + s);
            if (unsigned(lc) < unsigned(SW)) {
                const float* brow = Bs + lc * TK;
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const float4 b = *reinterpret_cast<const float4*>(brow + 4 * (q + j * TPR));
                    acc[j].x = fmaf(a, b.x, acc[j].x);
                    acc[j].y = fmaf(a, b.y, acc[j].y);
                    acc[j].z = fmaf(a, b.z, acc[j].z);
                    acc[j].w = fmaf(a, b.w, acc[j].w);
                }
            }
        }
        const int crow = F.grows[g * 16 + row];
        if (crow < 0) continue;
        float* crow_ptr = C + int64_t(crow) * ldc;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int col = k0 + 4 * (q + j * TPR);
            if (vec_c && col + 3 < O) {
                atomicAdd(reinterpret_cast<float4*>(crow_ptr + col), acc[j]);
            } else {
                if (col < O) atomicAdd(crow_ptr + col, acc[j].x);
                if (col + 1 < O) atomicAdd(crow_ptr + col + 1, acc[j].y);
                if (col + 2 < O) atomicAdd(crow_ptr + col + 2, acc[j].z);
                if (col + 3 < O) atomicAdd(crow_ptr + col + 3, acc[j].w);
            }
        }
    }
}

template <int TK, int SW>
cudaError_t launch_fp32(const DeviceFormatView& F, const float* B, int64_t ldb, int O, float* C, int64_t ldc,
                        cudaStream_t st) {
    const size_t smem = size_t(SW) * TK * sizeof(float);
    auto kern = vcsr_mc_fp32_kernel<TK, SW>;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
        if (e != cudaSuccess) return e;
    }
    const int vec_b = ((ldb & 3) == 0 && (reinterpret_cast<uintptr_t>(B) & 15) == 0) ? 1 : 0;
    const int vec_c = ((ldc & 3) == 0 && (reinterpret_cast<uintptr_t>(C) & 15) == 0) ? 1 : 0;
    const dim3 grid(F.num_items, (O + TK - 1) / TK);
    kern<<<grid, TK, smem, st>>>(F, B, ldb, O, C, ldc, vec_b, vec_c);
    return cudaGetLastError();
}

template <int TK>
cudaError_t launch_fp32_sw(const DeviceFormatView& F, const float* B, int64_t ldb, int O, float* C, int64_t ldc,
                           cudaStream_t st) {
    switch (F.segw) {
        case 16: return launch_fp32<TK, 16>(F, B, ldb, O, C, ldc, st);
        case 32: return launch_fp32<TK, 32>(F, B, ldb, O, C, ldc, st);
        case 48: return launch_fp32<TK, 48>(F, B, ldb, O, C, ldc, st);
        case 64: return launch_fp32<TK, 64>(F, B, ldb, O, C, ldc, st);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace

cudaError_t spmm_fp32_atomic(const DeviceFormatView& F, const float* B, int64_t ldb, int O, int tileK, float* C,
                             int64_t ldc, cudaStream_t st) {
    if (F.num_items == 0 || O == 0) return cudaSuccess;
    switch (tileK) {
        case 16: return launch_fp32_sw<16>(F, B, ldb, O, C, ldc, st);
        case 32: return launch_fp32_sw<32>(F, B, ldb, O, C, ldc, st);
        case 64: return launch_fp32_sw<64>(F, B, ldb, O, C, ldc, st);
        case 128: return launch_fp32_sw<128>(F, B, ldb, O, C, ldc, st);
        case 256: return launch_fp32_sw<256>(F, B, ldb, O, C, ldc, st);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace dev
}  // namespace vcsrmc
