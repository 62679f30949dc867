// FP16 VCSR-MC SpMM on the 5th-generation tensor cores (tcgen05, fp32 accumulation in TMEM).
//
// Results contract of the reference's vcsr_mc<NSLAB,SW> (src/vcsr_mc.cu:143-237): per work
// item (a run of <= 32 groups of one segment) and TK-column slab, the item's B segment
// B[seg_base : seg_base+SW, k0 : k0+TK] is staged once, every group's 16 x SW A tile is
// densified from its (lcol, val) slots, multiplied in fp16 with fp32 accumulation, scaled by
// `scale` and added into C (C += A * B). The B200 formulation:
//   * B segment: TMA 2-D boxes of SW rows x 64 columns with 128-byte swizzle (rows >= N and
//     columns >= O are zero-filled by the TMA unit, as the reference's `gr < N` guard does).
//     The boxes are the MMA's B operand as is: MN-major, one 64-column panel per box.
//   * A: eight groups are stacked into one M = 128 tile (thread t densifies lane t%16 of
//     group t/16 across its depth), K-major without swizzle: core matrices of 8 rows x 16 B,
//     K-adjacent core matrices 128 B apart (LBO), M-adjacent 8-row blocks SW*16 B apart (SBO).
//   * One elected thread issues SW/16 tcgen05.mma (M=128, N=TK, K=16) into a 128 x TK fp32
//     accumulator in tensor memory and commits to an mbarrier.
//   * Epilogue: warp w reads TMEM lanes 32w..32w+31 (one tile row per thread) with
//     tcgen05.ld and adds scale*row into C[group_rows[...]] with 16-byte vector reductions.
// Every wait is bounded (common.cuh); on expiry the kernel flags the format's status word,
// stops issuing work, frees its tensor memory and exits.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstring>

#include "common.cuh"
#include "spmm_launch.hpp"
#include "tma_host.hpp"

namespace vcsrmc {
namespace dev {
namespace {

constexpr int kThreads = 128;
constexpr int kTileM = 128;        // 8 groups x 16 rows
constexpr int kGroupsPerTile = 8;
constexpr int kSmemPerSM = 233472;  // 228 KB usable shared memory per SM
constexpr int kSmemReservedPerCTA = 1024;

__device__ __forceinline__ __half to_half(float v) { return __float2half_rn(v); }
__device__ __forceinline__ __half to_half(__half v) { return v; }

template <int TKI, int SW>
struct TcLayout {
    static constexpr int kPanels = TKI / 64;
    static constexpr int kPanelBytes = SW * 128;  // SW rows x 64 fp16
    static constexpr int kBBytes = kPanels * kPanelBytes;
    static constexpr int kABytes = kTileM * SW * 2;
    static constexpr int kBarOffset = kBBytes + kABytes;
    static constexpr int kUsed = kBarOffset + 64;
    static constexpr int kTmemCols = TKI;  // 64, 128 or 256: powers of two >= 32
    // Dynamic shared memory requested per CTA: enough that no more CTAs fit on an SM than its
    // 512 TMEM columns can serve at once, plus 1 KB for aligning the base to 1024 B.
    static constexpr int kMaxResident = 512 / kTmemCols;
    static constexpr int kCap = kSmemPerSM / (kMaxResident + 1) - kSmemReservedPerCTA + 64;
    static constexpr int kRequest = (kUsed > kCap ? kUsed : kCap) + 1024;
};

template <int TKI, int SW, bool kTma, typename BT>
__global__ void __launch_bounds__(kThreads, 1)
    vcsr_mc_fp16_tc_kernel(DeviceFormatView F, const __grid_constant__ CUtensorMap tmap, const BT* __restrict__ B,
                           int64_t ldb, int O, float* __restrict__ C, int64_t ldc, int vec_c) {
    using L = TcLayout<TKI, SW>;
    static_assert(SW % 16 == 0 && TKI % 64 == 0 && TKI <= 256, "unsupported tile");
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_addr = smem_u32(smem_raw);
    uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
    uint8_t* Bs = smem;
    uint8_t* As = smem + L::kBBytes;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBarOffset);  // [0] B staged, [1] MMA done
    uint32_t* tslot = reinterpret_cast<uint32_t*>(smem + L::kBarOffset + 16);
    int* abort_flag = reinterpret_cast<int*>(smem + L::kBarOffset + 20);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int k0 = blockIdx.y * TKI;
    const int2 it = F.items[blockIdx.x];
    const int seg_base = F.gmeta[it.x].z;
    const __half* __restrict__ aval = static_cast<const __half*>(F.val);

    if (warp == 0) {
        tmem_alloc(tslot, L::kTmemCols);
        tmem_relinquish();
    }
    if (tid == 0) {
        mbar_init(&bars[0], 1);
        mbar_init(&bars[1], 1);
        *abort_flag = 0;
        fence_mbar_init();
        if constexpr (kTma) prefetch_tmap(&tmap);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;

    // ---- stage the B segment -----------------------------------------------------------------
    if constexpr (kTma) {
        if (tid == 0) {
            mbar_arrive_expect_tx(&bars[0], uint32_t(L::kBBytes));
#pragma unroll
            for (int p = 0; p < L::kPanels; ++p)
                tma_load_2d(Bs + p * L::kPanelBytes, &tmap, &bars[0], k0 + 64 * p, seg_base);
        }
    } else {
        // Same bytes the TMA path produces: element (r, c) at panel c/64, row r, 16-byte chunk
        // ((c%64)/8) XOR (r%8), as the 128-byte swizzle lays it out.
        for (int e = tid; e < SW * (TKI / 8); e += kThreads) {
            const int r = e / (TKI / 8), c8 = (e % (TKI / 8)) * 8;
            const int gr = seg_base + r, gc = k0 + c8;
            __align__(16) __half h[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                __half v = __float2half_rn(0.f);
                if (gr < F.N && gc + j < O) v = to_half(B[int64_t(gr) * ldb + gc + j]);
                h[j] = v;
            }
            const int chunk = (c8 & 63) >> 3;
            const int off = (c8 >> 6) * L::kPanelBytes + r * 128 + ((chunk ^ (r & 7)) << 4);
            *reinterpret_cast<uint4*>(Bs + off) = *reinterpret_cast<const uint4*>(h);
        }
        fence_proxy_async_smem();
    }

    constexpr uint32_t kIdesc = idesc_f16_f32(kTileM, TKI, true);
    const uint32_t a_base = smem_u32(As), b_base = smem_u32(Bs);
    const int ngroups = it.y - it.x;
    uint32_t mma_parity = 0;
    bool b_ready = !kTma;

    for (int t0 = 0; t0 < ngroups; t0 += kGroupsPerTile) {
        const int gcount = min(kGroupsPerTile, ngroups - t0);
        // Zero the A tile (the previous tile's MMA has completed: its commit was awaited).
        for (int i = tid; i < L::kABytes / 16; i += kThreads)
            reinterpret_cast<uint4*>(As)[i] = make_uint4(0u, 0u, 0u, 0u);
        __syncthreads();
        // Densify: thread t -> group t/16 of the tile, lane t%16, all depth levels.
        const int gi = tid >> 4, ln = tid & 15;
        if (gi < gcount) {
            const int4 m = F.gmeta[it.x + t0 + gi];
            const int row = gi * 16 + ln;
            for (int d = 0; d < m.y; ++d) {
                const int s = m.x + d * 16 + ln;
                const int lc = F.lcol[s];
                if (unsigned(lc) < unsigned(SW)) {
                    const int off = ((row >> 3) * (SW / 8) + (lc >> 3)) * 128 + (row & 7) * 16 + (lc & 7) * 2;
                    *reinterpret_cast<__half*>(As + off) = aval[s];
                }
            }
        }
        fence_proxy_async_smem();
        __syncthreads();

        if (tid == 0) {
            bool good = true;
            if (!b_ready) good = mbar_wait_bounded(&bars[0], 0);
            if (good) {
                tc_fence_after();
#pragma unroll
                for (int kk = 0; kk < SW / 16; ++kk) {
                    const uint64_t adesc = smem_desc(a_base + kk * 256, 128, SW * 16, 0);
                    const uint64_t bdesc = smem_desc(b_base + kk * 2048, L::kPanelBytes, 1024, 2);
                    tc_mma_f16(tmem, adesc, bdesc, kIdesc, kk > 0 ? 1u : 0u);
                }
                tc_commit(&bars[1]);
            } else {
                *abort_flag = 1;
            }
        }
        b_ready = true;
        __syncthreads();
        bool ok = *abort_flag == 0;
        if (ok) ok = mbar_wait_bounded(&bars[1], mma_parity);
        if (__syncthreads_or(!ok)) {
            if (tid == 0) atomicOr(F.status, kStatusTimeout);
            break;
        }
        mma_parity ^= 1u;
        tc_fence_after();

        // ---- epilogue: TMEM -> registers -> C reductions --------------------------------------
        const int row = warp * 32 + lane;
        const int rgi = row >> 4;
        const int crow = rgi < gcount ? F.grows[(it.x + t0 + rgi) * 16 + (row & 15)] : -1;
        float* crow_ptr = C + int64_t(crow < 0 ? 0 : crow) * ldc;
#pragma unroll 1
        for (int c = 0; c < TKI; c += 32) {
            if (k0 + c >= O) break;  // uniform across the CTA
            uint32_t r[32];
            tmem_ld_32x32b_x32(tmem + (uint32_t(warp * 32) << 16) + uint32_t(c), r);
            tmem_wait_ld();
            if (crow >= 0) {
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const int col = k0 + c + 4 * j;
                    const float4 v = make_float4(__uint_as_float(r[4 * j]) * F.scale,
                                                 __uint_as_float(r[4 * j + 1]) * F.scale,
                                                 __uint_as_float(r[4 * j + 2]) * F.scale,
                                                 __uint_as_float(r[4 * j + 3]) * F.scale);
                    if (vec_c && col + 3 < O) {
                        atomicAdd(reinterpret_cast<float4*>(crow_ptr + col), v);
                    } else {
                        if (col < O) atomicAdd(crow_ptr + col, v.x);
                        if (col + 1 < O) atomicAdd(crow_ptr + col + 1, v.y);
                        if (col + 2 < O) atomicAdd(crow_ptr + col + 2, v.z);
                        if (col + 3 < O) atomicAdd(crow_ptr + col + 3, v.w);
                    }
                }
            }
        }
        tc_fence_before();
        __syncthreads();
    }

    // A TMA that was issued but never awaited (empty item) must land before the CTA exits.
    if (kTma && !b_ready && tid == 0) {
        if (!mbar_wait_bounded(&bars[0], 0)) atomicOr(F.status, kStatusTimeout);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, L::kTmemCols);
    }
}

template <int TKI, int SW, bool kTma, typename BT>
cudaError_t launch_tc(const DeviceFormatView& F, const CUtensorMap& tmap, const BT* B, int64_t ldb, int O, float* C,
                      int64_t ldc, cudaStream_t st) {
    using L = TcLayout<TKI, SW>;
    auto kern = vcsr_mc_fp16_tc_kernel<TKI, SW, kTma, BT>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kRequest);
    if (e != cudaSuccess) return e;
    const int vec_c = ((ldc & 3) == 0 && (reinterpret_cast<uintptr_t>(C) & 15) == 0) ? 1 : 0;
    const dim3 grid(F.num_items, (O + TKI - 1) / TKI);
    kern<<<grid, kThreads, L::kRequest, st>>>(F, tmap, B, ldb, O, C, ldc, vec_c);
    return cudaGetLastError();
}

template <int TKI, int SW>
cudaError_t dispatch_b(const DeviceFormatView& F, const void* B, int b_is_f16, int64_t ldb, int O, float* C,
                       int64_t ldc, cudaStream_t st) {
    CUtensorMap tmap;
    if (b_is_f16) {
        const __half* Bh = static_cast<const __half*>(B);
        if (encode_b_tmap_f16(&tmap, B, ldb, O, F.N, SW))
            return launch_tc<TKI, SW, true, __half>(F, tmap, Bh, ldb, O, C, ldc, st);
        return launch_tc<TKI, SW, false, __half>(F, tmap, Bh, ldb, O, C, ldc, st);
    }
    std::memset(&tmap, 0, sizeof(tmap));
    return launch_tc<TKI, SW, false, float>(F, tmap, static_cast<const float*>(B), ldb, O, C, ldc, st);
}

template <int TKI>
cudaError_t dispatch_sw(const DeviceFormatView& F, const void* B, int b_is_f16, int64_t ldb, int O, float* C,
                        int64_t ldc, cudaStream_t st) {
    switch (F.segw) {
        case 16: return dispatch_b<TKI, 16>(F, B, b_is_f16, ldb, O, C, ldc, st);
        case 32: return dispatch_b<TKI, 32>(F, B, b_is_f16, ldb, O, C, ldc, st);
        case 48: return dispatch_b<TKI, 48>(F, B, b_is_f16, ldb, O, C, ldc, st);
        case 64: return dispatch_b<TKI, 64>(F, B, b_is_f16, ldb, O, C, ldc, st);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace

cudaError_t spmm_fp16_tc_atomic(const DeviceFormatView& F, const void* B, int b_is_f16, int64_t ldb, int O,
                                int tileK, float* C, int64_t ldc, cudaStream_t st) {
    if (F.num_items == 0 || O == 0) return cudaSuccess;
    switch (tileK) {
        case 16:
        case 32:
        case 64: return dispatch_sw<64>(F, B, b_is_f16, ldb, O, C, ldc, st);
        case 128: return dispatch_sw<128>(F, B, b_is_f16, ldb, O, C, ldc, st);
        case 256: return dispatch_sw<256>(F, B, b_is_f16, ldb, O, C, ldc, st);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace dev
}  // namespace vcsrmc
