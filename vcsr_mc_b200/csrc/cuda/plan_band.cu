// Row-band execution plan for the FP16 format on the 5th-generation tensor cores: every CTA
// owns a band of 128 consecutive rows of A and a 128-column slab of B and C, accumulates the
// band's product over its column tiles in tensor memory, and writes its C tile once.
//
// The reference's FP16 dataflow (src/vcsr_mc.cu:143-237) multiplies densified 16-row groups of
// one segment by that segment's rows of B and adds every group into C with atomics. Here the
// same tcgen05 tile product (A densified from (column, value) entries in shared memory, B staged
// by TMA with the 128-byte swizzle, fp32 accumulation) runs row-stationary:
//   * a tile = the band's entries in 32 consecutive columns; tiles of a band are visited in
//     ascending column order, each adding a 128 x 32 by 32 x 128 product into one TMEM
//     accumulator (M = 128, N = 128, two K = 16 steps);
//   * 4 shared-memory stages of (B 8 KB, A 8 KB) and 5 warps: producer warp w owns stage w and
//     the tiles w, w + 4, ...: once the MMAs of its previous tile have completed it starts the
//     TMA load of the next B tile, clears its previous entries from the A tile (the positions
//     it remembers, or the whole tile after a large one), writes the new entries and arrives on
//     the stage's barrier; lane 0 of the fifth warp issues the MMAs in tile order. Producers
//     load their next tile's entries and bounds before they wait, so four tiles are being
//     prepared while the tensor cores work;
//   * epilogue: tcgen05.ld (warp w: rows 32w .. 32w+31), scale, one streaming store per C
//     element; C is never read (or read once, for C += A*B).
// B traffic per band is the B rows of its tiles (32 x 256 bytes each), which neighbouring bands
// share in L2; this suits matrices whose rows touch few column windows (stencils, banded or
// reordered matrices). Matrices with scattered columns are served better by the ROWS plan.
// Every wait is bounded; on expiry the kernel drains what it issued, flags the format's status
// word, frees its tensor memory and exits.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <vector>

#include "../capi_internal.hpp"
#include "../host/parallel.hpp"
#include "common.cuh"
#include "plan_band.hpp"
#include "tma_host.hpp"

namespace vcsrmc {
namespace dev {
namespace {

constexpr int kSlab = 128;                       // columns of B and C per CTA = MMA N
constexpr int kStages = 4;
constexpr int kProducers = kStages;              // producer warp w fills stage w: tiles i = w mod kStages
constexpr int kMmaWarp = kProducers;             // + one warp whose lane 0 issues the MMAs
constexpr int kThreads = (kProducers + 1) * 32;
constexpr int kSaved = 4;                        // entries a producer lane keeps per tile (to clear them)
constexpr int kPanelBytes = kBandK * 128;        // 32 rows x 64 fp16, 128-byte swizzle
constexpr int kBBytes = 2 * kPanelBytes;
constexpr int kABytes = kBandRows * kBandK * 2;
constexpr int kStageBytes = kBBytes + kABytes;   // a multiple of 1024: swizzle atoms stay aligned
constexpr int kBarOffset = kStages * kStageBytes;
constexpr int kSmemBytes = kBarOffset + 3 * kStages * 8 + 16 + 1024;  // + barriers, slot, alignment
constexpr uint32_t kTmemCols = kSlab;
static_assert(kStageBytes % 1024 == 0, "stage alignment");

// Byte offset of A element (row r, column c) in the K-major, unswizzled A tile: core matrices of
// 8 rows x 16 bytes, K-adjacent ones 128 B apart (LBO), 8-row blocks kBandK * 16 B apart (SBO).
__device__ __forceinline__ int a_offset(int r, int c) {
    return ((r >> 3) * (kBandK / 8) + (c >> 3)) * 128 + (r & 7) * 16 + (c & 7) * 2;
}
__device__ __forceinline__ int ent_offset(uint32_t e) { return a_offset(int((e >> 5) & 127u), int(e & 31u)); }

__device__ __forceinline__ __half to_half(float v) { return __float2half_rn(v); }
__device__ __forceinline__ __half to_half(__half v) { return v; }

// B rows [kc, kc + 32) x columns [k0, k0 + 128) by one warp's plain loads, in the layout the TMA
// path produces (element (r, c): panel c / 64, row r, 16-byte chunk ((c % 64) / 8) XOR (r % 8));
// rows >= N and columns >= O are zero.
template <typename BT>
__device__ __forceinline__ void stage_b_warp(uint8_t* Bs, const BT* __restrict__ B, int64_t ldb, int N, int O,
                                             int kc, int k0, int lane) {
    for (int e = lane; e < kBandK * (kSlab / 8); e += 32) {
        const int r = e / (kSlab / 8), c8 = (e % (kSlab / 8)) * 8;
        const int gr = kc + r, gc = k0 + c8;
        __align__(16) __half h[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            __half v = __float2half_rn(0.f);
            if (gr < N && gc + j < O) v = to_half(B[int64_t(gr) * ldb + gc + j]);
            h[j] = v;
        }
        const int chunk = (c8 & 63) >> 3;
        const int off = (c8 >> 6) * kPanelBytes + r * 128 + ((chunk ^ (r & 7)) << 4);
        *reinterpret_cast<uint4*>(Bs + off) = *reinterpret_cast<const uint4*>(h);
    }
}

template <bool kTma, bool kAcc, typename BT>
__global__ void __launch_bounds__(kThreads)
    vcsr_band_kernel(BandPlanView P, const __grid_constant__ CUtensorMap tmap, const BT* __restrict__ B,
                     int64_t ldb, int O, float* __restrict__ C, int64_t ldc, int vec_c) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_addr = smem_u32(smem_raw);
    uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
    uint64_t* full_b = reinterpret_cast<uint64_t*>(smem + kBarOffset);  // B tile of a stage landed (TMA)
    uint64_t* full_a = full_b + kStages;                                 // A tile of a stage written
    uint64_t* done = full_a + kStages;                                   // MMAs reading a stage completed
    uint32_t* tslot = reinterpret_cast<uint32_t*>(done + kStages);
    int* abort_flag = reinterpret_cast<int*>(tslot + 1);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int band = blockIdx.x;
    const int k0 = blockIdx.y * kSlab;
    const int ncols = min(kSlab, O - k0);
    const int row0 = band * kBandRows;
    const int t_beg = P.tile_ptr[band];
    const int nt = P.tile_ptr[band + 1] - t_beg;

    if (nt == 0) {  // rows without entries (uniform across the CTA: no barrier or TMEM needed)
        if (!kAcc)
            for (int i = tid; i < kBandRows * ncols; i += kThreads) {
                const int r = row0 + i / ncols;
                if (r < P.M) C[int64_t(r) * ldc + k0 + i % ncols] = 0.f;
            }
        return;
    }

    if (warp == 0) {
        tmem_alloc(tslot, kTmemCols);
        tmem_relinquish();
    }
    if (tid == 0) {
#pragma unroll
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full_b[s], 1);
            mbar_init(&full_a[s], 32);
            mbar_init(&done[s], 1);
        }
        *abort_flag = 0;
        fence_mbar_init();
        if constexpr (kTma) prefetch_tmap(&tmap);
    }
    // A tiles start zeroed; afterwards a producer clears its previous tile's entries.
    for (int i = tid; i < kStages * (kABytes / 16); i += kThreads) {
        const int s = i / (kABytes / 16), j = i % (kABytes / 16);
        reinterpret_cast<uint4*>(smem + s * kStageBytes + kBBytes)[j] = make_uint4(0u, 0u, 0u, 0u);
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;

    if (warp < kProducers) {
        // ---- producer: tiles w, w + 4, ... into stage w -------------------------------------
        const int s = warp;
        uint8_t* Bs = smem + s * kStageBytes;
        uint8_t* As = Bs + kBBytes;
        // The second 64-column panel of B is loaded only where it holds columns < O; past O the
        // accumulator columns are never stored, so the panel's contents do not matter there.
        const int npanels = k0 + 64 < O ? 2 : 1;
        int saved[kSaved];
#pragma unroll
        for (int k = 0; k < kSaved; ++k) saved[k] = -1;
        bool prev_overflow = false;
        int last_use = -1;  // lane 0: the last use of this stage whose B load was issued
        int kc = 0, e0 = 0, e1 = 0;
        if (s < nt) {
            kc = P.tile_col[t_beg + s];
            e0 = P.tile_eptr[t_beg + s];
            e1 = P.tile_eptr[t_beg + s + 1];
        }
        for (int i = s; i < nt; i += kStages) {
            const uint32_t use = uint32_t(i / kStages);
            // this tile's first entries and the next tile's bounds, loaded ahead of the wait
            uint32_t ev[kSaved];
#pragma unroll
            for (int k = 0; k < kSaved; ++k) {
                const int e = e0 + lane + 32 * k;
                ev[k] = e < e1 ? __ldg(P.ents + e) : 0u;
            }
            int nkc = 0, ne0 = 0, ne1 = 0;
            if (i + kStages < nt) {
                nkc = __ldg(P.tile_col + t_beg + i + kStages);
                ne0 = __ldg(P.tile_eptr + t_beg + i + kStages);
                ne1 = __ldg(P.tile_eptr + t_beg + i + kStages + 1);
            }
            // the stage is free once the MMAs of tile i - kStages completed
            if (use > 0 && !__all_sync(0xffffffffu, mbar_wait_bounded(&done[s], (use - 1u) & 1u))) {
                if (lane == 0) { *abort_flag = 1; atomicOr(P.status, kStatusTimeout); }
                break;
            }
            if constexpr (kTma) {
                if (lane == 0) {
                    mbar_arrive_expect_tx(&full_b[s], uint32_t(npanels * kPanelBytes));
                    tma_load_2d(Bs, &tmap, &full_b[s], k0, kc);
                    if (npanels == 2) tma_load_2d(Bs + kPanelBytes, &tmap, &full_b[s], k0 + 64, kc);
                    last_use = int(use);
                }
            } else {
                stage_b_warp<BT>(Bs, B, ldb, P.N, O, kc, k0, lane);
            }
            // clear the previous tile's entries: the remembered ones, or the whole tile
            if (use > 0) {
                if (prev_overflow) {
                    for (int j = lane; j < kABytes / 16; j += 32)
                        reinterpret_cast<uint4*>(As)[j] = make_uint4(0u, 0u, 0u, 0u);
                } else {
#pragma unroll
                    for (int k = 0; k < kSaved; ++k)
                        if (saved[k] >= 0) *reinterpret_cast<uint16_t*>(As + saved[k]) = 0;
                }
                __syncwarp();  // clears land before this tile's entries (positions may coincide)
            }
#pragma unroll
            for (int k = 0; k < kSaved; ++k) {
                const int e = e0 + lane + 32 * k;
                saved[k] = -1;
                if (e < e1) {
                    saved[k] = ent_offset(ev[k]);
                    *reinterpret_cast<uint16_t*>(As + saved[k]) = uint16_t(ev[k] >> 16);
                }
            }
            prev_overflow = e1 - e0 > 32 * kSaved;
            for (int e = e0 + 32 * kSaved + lane; e < e1; e += 32) {
                const uint32_t en = __ldg(P.ents + e);
                *reinterpret_cast<uint16_t*>(As + ent_offset(en)) = uint16_t(en >> 16);
            }
            fence_proxy_async_smem();
            mbar_arrive(&full_a[s]);
            kc = nkc;
            e0 = ne0;
            e1 = ne1;
        }
        __syncwarp();
        // a B load that was issued must land before the CTA exits (normally it has been awaited
        // by the MMA issuer already, and this wait returns at once)
        if (kTma && lane == 0 && last_use >= 0) mbar_wait_bounded(&full_b[s], uint32_t(last_use) & 1u);
    } else if (warp == kMmaWarp && lane == 0) {
        // ---- MMA issuer ----------------------------------------------------------------------
        constexpr uint32_t kIdesc = idesc_f16_f32(kBandRows, kSlab, true);
        int committed = -1;
        for (int i = 0; i < nt; ++i) {
            const int s = i % kStages;
            const uint32_t par = uint32_t(i / kStages) & 1u;
            bool good = mbar_wait_bounded(&full_a[s], par);
            if (kTma && good) good = mbar_wait_bounded(&full_b[s], par);
            if (!good) {
                *abort_flag = 1;
                atomicOr(P.status, kStatusTimeout);
                break;
            }
            tc_fence_after();
            const uint32_t a_addr = smem_u32(smem + s * kStageBytes + kBBytes);
            const uint32_t b_addr = smem_u32(smem + s * kStageBytes);
#pragma unroll
            for (int kk = 0; kk < kBandK / 16; ++kk)
                tc_mma_f16(tmem, smem_desc(a_addr + kk * 256, 128, kBandK * 16, 0),
                           smem_desc(b_addr + kk * 2048, kPanelBytes, 1024, 2), kIdesc, (i > 0 || kk > 0) ? 1u : 0u);
            tc_commit(&done[s]);
            committed = i;
        }
        // the accumulator is complete (or, after a timeout, no MMA is in flight) once the last
        // committed group of MMAs has completed
        if (committed >= 0 && !mbar_wait_bounded(&done[committed % kStages], uint32_t(committed / kStages) & 1u)) {
            *abort_flag = 1;
            atomicOr(P.status, kStatusTimeout);
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();

    // ---- epilogue: warp w < 4 holds rows 32w .. 32w+31 of the accumulator -----------------------
    if (*abort_flag == 0 && warp < 4) {
        const int grow = row0 + warp * 32 + lane;
        float* crow = C + int64_t(grow) * ldc + k0;
#pragma unroll 1
        for (int c = 0; c < kSlab; c += 32) {
            if (c >= ncols) break;  // uniform across the CTA
            uint32_t v[32];
            tmem_ld_32x32b_x32(tmem + (uint32_t(warp * 32) << 16) + uint32_t(c), v);
            tmem_wait_ld();
            if (grow < P.M) {
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const int col = c + 4 * j;
                    float4 x = make_float4(__uint_as_float(v[4 * j]) * P.scale, __uint_as_float(v[4 * j + 1]) * P.scale,
                                           __uint_as_float(v[4 * j + 2]) * P.scale,
                                           __uint_as_float(v[4 * j + 3]) * P.scale);
                    if (vec_c && col + 3 < ncols) {
                        float4* d = reinterpret_cast<float4*>(crow + col);
                        if constexpr (kAcc) {
                            const float4 o = *d;
                            x.x += o.x; x.y += o.y; x.z += o.z; x.w += o.w;
                        }
                        __stcs(d, x);
                    } else {
                        const float xs[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
                        for (int q = 0; q < 4; ++q)
                            if (col + q < ncols) {
                                if constexpr (kAcc) crow[col + q] += xs[q];
                                else crow[col + q] = xs[q];
                            }
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

template <bool kTma, bool kAcc, typename BT>
cudaError_t launch_band_t(const BandPlanView& P, const CUtensorMap& tmap, const BT* B, int64_t ldb, int O, float* C,
                          int64_t ldc, cudaStream_t st) {
    auto kern = vcsr_band_kernel<kTma, kAcc, BT>;
    const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    if (e != cudaSuccess) return e;
    const int vec_c = ((ldc & 3) == 0 && (reinterpret_cast<uintptr_t>(C) & 15) == 0) ? 1 : 0;
    const int slabs = (O + kSlab - 1) / kSlab;
    if (slabs > 65535) return cudaErrorInvalidValue;
    const dim3 grid(unsigned(P.n_bands), unsigned(slabs));
    kern<<<grid, kThreads, kSmemBytes, st>>>(P, tmap, B, ldb, O, C, ldc, vec_c);
    return cudaGetLastError();
}

template <bool kTma, typename BT>
cudaError_t launch_band_b(const BandPlanView& P, const CUtensorMap& tmap, const BT* B, int64_t ldb, int O, float* C,
                          int64_t ldc, bool accumulate, cudaStream_t st) {
    return accumulate ? launch_band_t<kTma, true, BT>(P, tmap, B, ldb, O, C, ldc, st)
                      : launch_band_t<kTma, false, BT>(P, tmap, B, ldb, O, C, ldc, st);
}

}  // namespace

cudaError_t spmm_band(const BandPlanView& P, const void* B, int b_is_f16, int64_t ldb, int O, float* C, int64_t ldc,
                      bool accumulate, cudaStream_t st) {
    if (P.M == 0 || O == 0 || P.n_bands == 0) return cudaSuccess;
    CUtensorMap tmap;
    if (b_is_f16) {
        const __half* Bh = static_cast<const __half*>(B);
        if (encode_b_tmap_f16(&tmap, B, ldb, O, P.N, kBandK))
            return launch_band_b<true, __half>(P, tmap, Bh, ldb, O, C, ldc, accumulate, st);
        return launch_band_b<false, __half>(P, tmap, Bh, ldb, O, C, ldc, accumulate, st);
    }
    std::memset(&tmap, 0, sizeof(tmap));
    return launch_band_b<false, float>(P, tmap, static_cast<const float*>(B), ldb, O, C, ldc, accumulate, st);
}

// ---- host: the band view -----------------------------------------------------------------------
BandViewHost build_band_view(const RowViewHost& rv, int M, int nthreads) {
    BandViewHost h;
    const int nb = (M + kBandRows - 1) / kBandRows;
    const int64_t nnz = M > 0 ? rv.rp[M] : 0;
    // one sort key per entry: tile (column / 32) above (row in band, local column, fp16 value),
    // so a band's sorted keys are its tiles in column order
    std::vector<uint64_t> keys(size_t(std::max<int64_t>(nnz, 0)));
    std::vector<int> ntiles(size_t(nb), 0);
    const int nth = resolve_threads(nthreads);
    parallel_for_dynamic(0, nb, nth, 64, [&](int64_t lo, int64_t hi) {
        for (int64_t b = lo; b < hi; ++b) {
            const int r0 = int(b) * kBandRows, r1 = std::min(M, r0 + kBandRows);
            for (int r = r0; r < r1; ++r)
                for (int p = rv.rp[r]; p < rv.rp[r + 1]; ++p) {
                    const uint32_t col = uint32_t(rv.cols[p]);
                    const __half hv = __float2half_rn(rv.vals[p]);
                    unsigned short bits;
                    std::memcpy(&bits, &hv, sizeof bits);
                    const uint32_t ent = (col & 31u) | (uint32_t(r - r0) << 5) | (uint32_t(bits) << 16);
                    keys[size_t(p)] = (uint64_t(col >> 5) << 32) | ent;
                }
            uint64_t* kb = keys.data() + rv.rp[r0];
            uint64_t* ke = keys.data() + rv.rp[r1];
            std::sort(kb, ke);
            int n = 0;
            for (uint64_t* k = kb; k < ke; ++k)
                if (k == kb || (*k >> 32) != (k[-1] >> 32)) ++n;
            ntiles[size_t(b)] = n;
        }
    });
    h.tile_ptr.assign(size_t(nb) + 1, 0);
    for (int b = 0; b < nb; ++b) h.tile_ptr[size_t(b) + 1] = h.tile_ptr[size_t(b)] + ntiles[size_t(b)];
    const int64_t T = h.tile_ptr[size_t(nb)];
    h.tile_col.resize(size_t(T));
    h.tile_eptr.resize(size_t(T) + 1);
    h.ents.resize(size_t(nnz));
    h.tile_eptr[size_t(T)] = int(nnz);
    parallel_for_dynamic(0, nb, nth, 64, [&](int64_t lo, int64_t hi) {
        for (int64_t b = lo; b < hi; ++b) {
            const int r0 = int(b) * kBandRows, r1 = std::min(M, r0 + kBandRows);
            int t = h.tile_ptr[size_t(b)];
            for (int p = rv.rp[r0]; p < rv.rp[r1]; ++p) {
                const uint64_t k = keys[size_t(p)];
                if (p == rv.rp[r0] || (k >> 32) != (keys[size_t(p) - 1] >> 32)) {
                    h.tile_col[size_t(t)] = int(k >> 32) * kBandK;
                    h.tile_eptr[size_t(t)] = p;
                    ++t;
                }
                h.ents[size_t(p)] = uint32_t(k);
            }
        }
    });
    // Every index the kernel follows stays inside its array: checked once here.
    auto bad = [] { throw StatusError(VCSRMC_INTERNAL, "band view construction is inconsistent"); };
    for (int b = 0; b < nb; ++b) {
        const int t0 = h.tile_ptr[size_t(b)], t1 = h.tile_ptr[size_t(b) + 1];
        if (t1 < t0 || t1 > T) bad();
        const int r0 = b * kBandRows, r1 = std::min(M, r0 + kBandRows);
        if (t1 > t0 && (h.tile_eptr[size_t(t0)] != rv.rp[r0] || h.tile_eptr[size_t(t1)] != rv.rp[r1])) bad();
        for (int t = t0; t < t1; ++t)
            if (h.tile_eptr[size_t(t) + 1] <= h.tile_eptr[size_t(t)] || h.tile_col[size_t(t)] < 0 ||
                h.tile_col[size_t(t)] % kBandK != 0 || (t > t0 && h.tile_col[size_t(t)] <= h.tile_col[size_t(t) - 1]))
                bad();
    }
    return h;
}

}  // namespace dev
}  // namespace vcsrmc
