// Row-band execution plan for the FP16 format on the 5th-generation tensor cores: each band of
// up to 128 consecutive rows of A, times a 128-column slab of B, is accumulated over its column
// tiles in tensor memory and its C tile is written once.
//
// The reference's FP16 dataflow (src/vcsr_mc.cu:143-237) multiplies densified 16-row groups of
// one segment by that segment's rows of B and adds every group into C with atomics. Here the
// same tcgen05 tile product (A densified from (column, value) entries in shared memory, B staged
// by TMA with the 128-byte swizzle, fp32 accumulation) runs row-stationary:
//   * a tile = a band's entries in kBandK (64) consecutive columns starting at the first column
//     not covered by the previous tile; each adds its product into the band's TMEM accumulator,
//     transposed: (128 slab columns x 64) by (64 x NB band rows), NB = 64 for bands of at most 64
//     rows, else 128 (M = 128, N = NB, four K = 16 steps);
//   * persistent CTAs (three per SM for NB = 64, two for NB = 128) walk their work items (band,
//     slab) in a strided order; the tiles of all their items form one sequence through the CTA's
//     shared-memory stages (B 16 KB + A NB x 128 bytes each). Producer warp w owns stage w: once
//     the MMAs of its previous tile have completed it starts the TMA load of its next B tile,
//     clears its previous entries from the A tile (the positions it remembers, or the whole tile
//     after a large one), writes the new entries and arrives on the stage's barrier. Its
//     registers run one position ahead (entries and bounds are loaded two iterations before use);
//   * lane 0 of the MMA warp issues the MMAs in sequence order into one of two TMEM
//     accumulators, so the MMAs of a band overlap the epilogue of the previous one;
//   * four epilogue warps read their TMEM lane quarter (tcgen05.ld: a lane is a column of C, the
//     registers are rows) and store each row's 32 columns as one 128-byte warp store (for
//     C += A*B, one 128-byte warp reduction).
// Several CTAs per SM outrun one CTA with more stages (0.300 against 0.365 ms on a 27-point
// stencil in an earlier form): each CTA's MMA issuer walks its tiles one at a time, and the other
// CTAs fill its waits. 64-column tiles beat 32-column ones by halving the tiles.
// B traffic per band is the B rows of its tiles (64 x 256 bytes each), which neighbouring bands
// share in L2; this suits matrices whose rows touch few column windows (stencils, banded or
// reordered matrices). Matrices with scattered columns are served better by the ROWS plan.
// Every wait is bounded; on expiry the CTA's warps stop, drain what they issued, the format's
// status word is flagged and the tensor memory is freed.
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

// The band product, for bands of at most NB rows (64 or 128): D^T (128 slab columns x NB band rows)
// = B tile^T (M = 128, MN-major: kBandK rows of B x 128 columns in two 64-column panels with the
// 128-byte swizzle, as TMA lands them) x A tile^T (N = NB, K-major: the band's entries scattered
// into NB x kBandK fp16). A TMEM lane holds a column of C, so a warp's store of one row writes 128
// contiguous bytes, and a band of at most 64 rows costs half the tensor-core work of N = 128.
// Per SM, stages in flight decide the speed (each stage waits for its B tile's TMA load after its
// previous MMAs complete): on a 27-point stencil at 62-row bands, 2 CTAs x 3 stages took 0.298 ms,
// 2 x 4 stages 0.278 ms and 3 x 3 stages 0.2665 ms; 128-row bands (2 x 3 stages) 0.289 ms, against
// 0.294 ms for the same product with a row of C per TMEM lane and a transposing epilogue (all with
// an L2 prefetch of each stage's next B tile, since dropped: 3 x 3 stages now 0.246 ms).
constexpr int kSlab = 128;                       // columns of B and C per work item (= MMA M)
constexpr int kSaved = 8;                        // entries a producer lane keeps per tile (to clear them)
constexpr int kAccs = 2;                         // TMEM accumulators: one band's MMAs overlap the previous epilogue
constexpr int kPanelBytes = kBandK * 128;        // kBandK rows x 64 fp16, 128-byte swizzle
constexpr int kBBytes = 2 * kPanelBytes;
constexpr int kSmemPerSm = 233472;
#ifndef VCSRMC_BAND_CTAS64
#define VCSRMC_BAND_CTAS64 3
#endif

template <int NB>
struct BandShape {
    static_assert(NB == 64 || NB == 128, "bands of at most 64 or 128 rows");
    static constexpr int kCtas = NB == 64 ? VCSRMC_BAND_CTAS64 : 2;  // CTAs per SM
    static constexpr int kABytes = NB * kBandK * 2;
    static constexpr int kStageBytes = kBBytes + kABytes;  // a multiple of 1024: swizzle atoms stay aligned
    static constexpr int kFixed = (3 * 8 + 2 * kAccs) * 8 + 16 + 1024;  // barriers, slot, flag, alignment
    static constexpr int kFit = (kSmemPerSm / kCtas - 1024 - kFixed) / kStageBytes;
    static constexpr int kStages = kFit < 6 ? kFit : 6;
    static constexpr int kProducers = kStages;   // warps 0 .. kStages - 1: producer w fills stage w
    static constexpr int kMmaWarp = kProducers;  // next warp: lane 0 issues the MMAs
    static constexpr int kEpiWarp0 = kProducers + 1;  // last 4 warps: epilogue (TMEM lane quarter = warp % 4)
    static constexpr int kThreads = (kEpiWarp0 + 4) * 32;
    static constexpr uint32_t kTmemCols = kAccs * NB;
    static constexpr int kBarOffset = kStages * kStageBytes;
    static constexpr int kNumBars = 3 * kStages + 2 * kAccs;
    static constexpr int kSmemBytes = kBarOffset + kNumBars * 8 + 16 + 1024;
    static constexpr uint32_t kIdesc = idesc_f16_f32(kSlab, NB, false, true);  // A MN-major, B K-major
    static_assert(kStages >= 2 && kStages <= 8, "two to eight stages");
    static_assert(kStageBytes % 1024 == 0, "stage alignment");
    static_assert(kCtas * kTmemCols <= 512, "tensor memory per SM");
    static_assert(kCtas * (kSmemBytes + 1024) <= kSmemPerSm, "shared memory per SM");
};

// Byte offset of A element (row r, column c) in the K-major, unswizzled A tile: core matrices of
// 8 rows x 16 bytes, K-adjacent ones 128 B apart (LBO), 8-row blocks kBandK * 16 B apart (SBO).
__device__ __forceinline__ int a_offset(int r, int c) {
    return ((r >> 3) * (kBandK / 8) + (c >> 3)) * 128 + (r & 7) * 16 + (c & 7) * 2;
}
// An entry's place in an A tile of NB rows (the row masked to the tile, so that no entry can write
// outside it).
template <int NB>
__device__ __forceinline__ int ent_offset(uint32_t e) {
    return a_offset(int((e >> kBandColBits) & uint32_t(NB - 1)), int(e & uint32_t(kBandK - 1)));
}

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

// Bounded wait that also gives up when another warp has flagged an abort (or flags one itself
// when its own budget runs out), so that one expired wait ends the whole CTA promptly.
__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    for (;;) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*abort_flag != 0) return false;
        if (clock64() - t0 > kWaitBudgetCycles) {
            *abort_flag = 1;
            return false;
        }
    }
}

// Work items of a CTA: items blockIdx.x, + gridDim.x, ...; item -> band item % n_bands and
// column slab item / n_bands. The tiles of all its items form one sequence; position q of it
// uses stage q % kStages.
struct ItemRange {
    int t_beg, nt;
};
__device__ __forceinline__ ItemRange item_range(const BandPlanView& P, int item, int n_items) {
    if (item >= n_items) return ItemRange{0, 0};
    const int b = item % P.n_bands;
    const int t0 = __ldg(P.tile_ptr + b);
    return ItemRange{t0, __ldg(P.tile_ptr + b + 1) - t0};
}
// A position in the tile sequence (the next item's range is loaded ahead).
struct TileIter {
    int item, t;
    ItemRange cur, next;
};
__device__ __forceinline__ void iter_advance(TileIter& it, int step, const BandPlanView& P, int n_items) {
    it.t += step;
    while (it.item < n_items && it.t >= it.cur.nt) {
        it.t -= it.cur.nt;
        it.item += gridDim.x;
        it.cur = it.next;
        it.next = item_range(P, it.item + gridDim.x, n_items);
    }
}
__device__ __forceinline__ TileIter iter_begin(const BandPlanView& P, int n_items, int step) {
    TileIter it;
    it.item = blockIdx.x;
    it.t = 0;
    it.cur = item_range(P, it.item, n_items);
    it.next = item_range(P, it.item + gridDim.x, n_items);
    iter_advance(it, step, P, n_items);
    return it;
}

// A producer's registers for one position of the tile sequence.
struct ProducerRegs {
    TileIter it;
    int kc, e0, e1;          // tile's first column and entry range
    uint32_t ev[kSaved];     // its first 32 * kSaved entries, lane-strided
};
__device__ __forceinline__ void load_bounds(ProducerRegs& r, const BandPlanView& P, int n_items) {
    r.kc = 0;
    r.e0 = 0;
    r.e1 = 0;
    if (r.it.item < n_items) {
        const int t = r.it.cur.t_beg + r.it.t;
        r.kc = __ldg(P.tile_col + t);
        r.e0 = __ldg(P.tile_eptr + t);
        r.e1 = __ldg(P.tile_eptr + t + 1);
    }
}
__device__ __forceinline__ void load_entries(ProducerRegs& r, const BandPlanView& P, int lane) {
#pragma unroll
    for (int k = 0; k < kSaved; ++k) {
        const int e = r.e0 + lane + 32 * k;
        r.ev[k] = e < r.e1 ? __ldg(P.ents + e) : 0u;
    }
}

template <bool kTma, bool kAcc, typename BT, int NB>
__global__ void __launch_bounds__(BandShape<NB>::kThreads, BandShape<NB>::kCtas)
    vcsr_band_kernel(BandPlanView P, const __grid_constant__ CUtensorMap tmap, const BT* __restrict__ B,
                     int64_t ldb, int O, float* __restrict__ C, int64_t ldc) {
    using S = BandShape<NB>;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_addr = smem_u32(smem_raw);
    uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
    uint64_t* full_b = reinterpret_cast<uint64_t*>(smem + S::kBarOffset);  // B tile of a stage landed (TMA)
    uint64_t* full_a = full_b + S::kStages;                                 // A tile of a stage written
    uint64_t* done = full_a + S::kStages;                                   // MMAs reading a stage completed
    uint64_t* acc_full = done + S::kStages;                                 // a band's accumulator is complete
    uint64_t* acc_empty = acc_full + kAccs;                              // the epilogue has read it
    uint32_t* tslot = reinterpret_cast<uint32_t*>(acc_empty + kAccs);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tslot + 1);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int n_items = P.n_bands * ((O + kSlab - 1) / kSlab);

    if (warp == 0) {
        tmem_alloc(tslot, S::kTmemCols);
        tmem_relinquish();
    }
    if (tid == 0) {
#pragma unroll
        for (int s = 0; s < S::kStages; ++s) {
            mbar_init(&full_b[s], 1);
            mbar_init(&full_a[s], 1);
            mbar_init(&done[s], 1);
        }
#pragma unroll
        for (int a = 0; a < kAccs; ++a) {
            mbar_init(&acc_full[a], 1);
            mbar_init(&acc_empty[a], 128);
        }
        *abort_flag = 0;
        fence_mbar_init();
        if constexpr (kTma) prefetch_tmap(&tmap);
    }
    // A tiles start zeroed; afterwards a producer clears its previous tile's entries.
    for (int i = tid; i < S::kStages * (S::kABytes / 16); i += S::kThreads) {
        const int s = i / (S::kABytes / 16), j = i % (S::kABytes / 16);
        reinterpret_cast<uint4*>(smem + s * S::kStageBytes + kBBytes)[j] = make_uint4(0u, 0u, 0u, 0u);
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;

    if (warp < S::kProducers) {
        // ---- producer w: positions w, w + S::kStages, ... of the tile sequence, into stage w -----
        const int s = warp;
        uint8_t* Bs = smem + s * S::kStageBytes;
        uint8_t* As = Bs + kBBytes;
        int saved[kSaved];
#pragma unroll
        for (int k = 0; k < kSaved; ++k) saved[k] = -1;
        bool prev_overflow = false;
        int last_use = -1;  // lane 0: the last use of this stage whose B load was issued
        uint32_t use = 0;
        // Three register sets rotate through the roles current (bounds and first entries
        // loaded), next (bounds loaded) and after-next; every iteration issues the loads of the
        // next position's entries and the after-next position's bounds before it waits for its
        // stage, and consumes them two iterations later. The loop is unrolled three times so that
        // no register holding a pending load is ever copied (a copy would wait for the load).
        ProducerRegs X, Y, Z;
        X.it = iter_begin(P, n_items, s);
        load_bounds(X, P, n_items);
        Y.it = X.it;
        iter_advance(Y.it, S::kStages, P, n_items);
        load_bounds(Y, P, n_items);
        load_entries(X, P, lane);
        auto step = [&](ProducerRegs& cur, ProducerRegs& nxt, ProducerRegs& nn) -> bool {
            if (cur.it.item >= n_items) return false;
            load_entries(nxt, P, lane);
            nn.it = nxt.it;
            iter_advance(nn.it, S::kStages, P, n_items);
            load_bounds(nn, P, n_items);
            // the stage is free once the MMAs of its previous tile completed (lane 0 waits; the
            // warp barrier orders the other lanes' writes to the stage after its observation)
            if (use > 0) {
                bool free = true;
                if (lane == 0) free = wait_or_abort(&done[s], (use - 1u) & 1u, abort_flag);
                if (!__shfl_sync(0xffffffffu, free, 0)) return false;
            }
            const int k0 = (cur.it.item / P.n_bands) * kSlab;
            if constexpr (kTma) {
                // (no L2 prefetch of the stage's next B tile: on a 27-point stencil, where 85 % of the
                // B tile reads hit L2 anyway, dropping it took 0.267 -> 0.246 ms)
                if (lane == 0) {
                    // The second 64-column panel is loaded only where it holds columns < O; past O
                    // the accumulator columns are never stored, so its contents do not matter.
                    const int npanels = k0 + 64 < O ? 2 : 1;
                    mbar_arrive_expect_tx(&full_b[s], uint32_t(npanels * kPanelBytes));
                    tma_load_2d(Bs, &tmap, &full_b[s], k0, cur.kc);
                    if (npanels == 2) tma_load_2d(Bs + kPanelBytes, &tmap, &full_b[s], k0 + 64, cur.kc);
                    last_use = int(use);
                }
            } else {
                stage_b_warp<BT>(Bs, B, ldb, P.N, O, cur.kc, k0, lane);
            }
            // clear the previous tile's entries: the remembered ones, or the whole tile
            if (use > 0) {
                if (prev_overflow) {
                    for (int j = lane; j < S::kABytes / 16; j += 32)
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
                const int e = cur.e0 + lane + 32 * k;
                saved[k] = -1;
                if (e < cur.e1) {
                    saved[k] = ent_offset<NB>(cur.ev[k]);
                    *reinterpret_cast<uint16_t*>(As + saved[k]) = uint16_t(cur.ev[k] >> 16);
                }
            }
            prev_overflow = cur.e1 - cur.e0 > 32 * kSaved;
            for (int e = cur.e0 + 32 * kSaved + lane; e < cur.e1; e += 32) {
                const uint32_t en = __ldg(P.ents + e);
                *reinterpret_cast<uint16_t*>(As + ent_offset<NB>(en)) = uint16_t(en >> 16);
            }
            // every lane makes its writes visible to the tensor core's (async) reads, the warp
            // barrier orders them before lane 0's arrival, which releases them to the MMA issuer
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(&full_a[s]);
            ++use;
            return true;
        };
        for (;;) {
            if (!step(X, Y, Z)) break;
            if (!step(Y, Z, X)) break;
            if (!step(Z, X, Y)) break;
        }
        __syncwarp();
        // A B load that was issued must land before the CTA exits (normally the MMA warp has
        // awaited it already and this returns at once).
        if (kTma && lane == 0 && last_use >= 0) mbar_wait_bounded(&full_b[s], uint32_t(last_use) & 1u);
    } else if (warp == S::kMmaWarp) {
        // ---- MMA issuer: the tile sequence in order, one accumulator per band -----------------
        if (lane == 0) {
            uint32_t q = 0, u = 0;  // sequence position; bands with tiles so far
            int last_stage = -1;
            uint32_t last_par = 0;
            bool ok = true;
            ItemRange r = item_range(P, blockIdx.x, n_items);
            for (int item = blockIdx.x; ok && item < n_items; item += gridDim.x) {
                const ItemRange rn = item_range(P, item + gridDim.x, n_items);
                if (r.nt > 0) {
                    const uint32_t acc = u % kAccs;
                    if (u >= kAccs && !wait_or_abort(&acc_empty[acc], ((u / kAccs) - 1u) & 1u, abort_flag)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    for (int t = 0; t < r.nt; ++t, ++q) {
                        const int s = int(q % S::kStages);
                        const uint32_t par = (q / S::kStages) & 1u;
                        if (!wait_or_abort(&full_a[s], par, abort_flag) ||
                            (kTma && !wait_or_abort(&full_b[s], par, abort_flag))) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint32_t a_addr = smem_u32(smem + s * S::kStageBytes + kBBytes);
                        const uint32_t b_addr = smem_u32(smem + s * S::kStageBytes);
#pragma unroll
                        for (int kk = 0; kk < kBandK / 16; ++kk) {
                            // the band's entries: K-major, unswizzled core matrices; the B tile:
                            // MN-major, 128-byte swizzle, 64-column panels kPanelBytes apart
                            const uint64_t da = smem_desc(a_addr + kk * 256, 128, kBandK * 16, 0);
                            const uint64_t db = smem_desc(b_addr + kk * 2048, kPanelBytes, 1024, 2);
                            tc_mma_f16(tmem + acc * NB, db, da, S::kIdesc, (t > 0 || kk > 0) ? 1u : 0u);
                        }
                        tc_commit(&done[s]);
                        last_stage = s;
                        last_par = par;
                    }
                    if (!ok) break;
                    tc_commit(&acc_full[acc]);
                    ++u;
                }
                r = rn;
            }
            // after an abort no MMA may still be reading shared memory or writing TMEM at exit
            if (!ok && last_stage >= 0) mbar_wait_bounded(&done[last_stage], last_par);
        }
        __syncwarp();
    } else {
        // ---- epilogue ---------------------------------------------------------------------------
        const int quarter = warp & 3;
        const uint32_t lane_base = uint32_t(quarter * 32) << 16;
        uint32_t u = 0;
        ItemRange r = item_range(P, blockIdx.x, n_items);
        for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
            const ItemRange rn = item_range(P, item + gridDim.x, n_items);
            const int band = item % P.n_bands;
            const int k0 = (item / P.n_bands) * kSlab;
            const int ncols = min(kSlab, O - k0);
            const int row0 = band * P.band_rows;
            const int row_end = min(P.M, row0 + P.band_rows);
            // columns k0 + 32 q .. k0 + 32 q + 31 of the band's rows: lane = column
            const int col = quarter * 32 + lane;
            const bool col_ok = col < ncols;
            float* ccol = C + k0 + col;
            if (r.nt == 0) {
                if (!kAcc && col_ok)
                    for (int row = row0; row < row_end; ++row) ccol[int64_t(row) * ldc] = 0.f;
            } else {
                const uint32_t acc = u % kAccs;
                if (!__all_sync(0xffffffffu, wait_or_abort(&acc_full[acc], (u / kAccs) & 1u, abort_flag))) break;
                tc_fence_after();
                if (quarter * 32 < ncols) {  // warp-uniform: this quarter holds columns < O
#pragma unroll 1
                    for (int rr = 0; rr < NB && row0 + rr < row_end; rr += 16) {
                        uint32_t v[16];
                        tmem_ld_32x32b_x16(tmem + lane_base + acc * NB + uint32_t(rr), v);
                        tmem_wait_ld();
                        if (col_ok) {
#pragma unroll
                            for (int j = 0; j < 16; ++j) {
                                const int row = row0 + rr + j;
                                if (row < row_end) {
                                    float* dst = ccol + int64_t(row) * ldc;
                                    const float x = __uint_as_float(v[j]) * P.scale;
                                    // C += A*B: a fire-and-forget reduction (red.global.add.f32) into
                                    // a row that only this band writes, instead of a load-add-store
                                    // that waits for the old value row by row (config 3: 1.136 ms
                                    // with the loads, 0.244 ms with the reductions)
                                    if constexpr (kAcc) atomicAdd(dst, x);
                                    else __stcs(dst, x);
                                }
                            }
                        }
                    }
                }
                tc_fence_before();
                mbar_arrive(&acc_empty[acc]);
                ++u;
            }
            r = rn;
        }
    }
    tc_fence_before();
    __syncthreads();
    if (tid == 0 && *abort_flag != 0) atomicOr(P.status, kStatusTimeout);
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, S::kTmemCols);
    }
}

template <bool kTma, bool kAcc, typename BT, int NB>
cudaError_t launch_band_t(const BandPlanView& P, const CUtensorMap& tmap, const BT* B, int64_t ldb, int O, float* C,
                          int64_t ldc, cudaStream_t st) {
    using S = BandShape<NB>;
    auto kern = vcsr_band_kernel<kTma, kAcc, BT, NB>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, S::kSmemBytes);
    if (e != cudaSuccess) return e;
    int dev = 0, sms = 0;
    if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
    if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return e;
    const int64_t items = int64_t(P.n_bands) * ((O + kSlab - 1) / kSlab);
    if (items > 0x7fffffffLL) return cudaErrorInvalidValue;
    // persistent: at most kCtas CTAs per SM, each walking its items in a strided order
    const int grid = int(std::min<int64_t>(items, int64_t(sms) * S::kCtas));
    kern<<<grid, S::kThreads, S::kSmemBytes, st>>>(P, tmap, B, ldb, O, C, ldc);
    return cudaGetLastError();
}

template <bool kTma, typename BT>
cudaError_t launch_band_b(const BandPlanView& P, const CUtensorMap& tmap, const BT* B, int64_t ldb, int O, float* C,
                          int64_t ldc, bool accumulate, cudaStream_t st) {
    if (P.band_rows <= 64)
        return accumulate ? launch_band_t<kTma, true, BT, 64>(P, tmap, B, ldb, O, C, ldc, st)
                          : launch_band_t<kTma, false, BT, 64>(P, tmap, B, ldb, O, C, ldc, st);
    return accumulate ? launch_band_t<kTma, true, BT, 128>(P, tmap, B, ldb, O, C, ldc, st)
                      : launch_band_t<kTma, false, BT, 128>(P, tmap, B, ldb, O, C, ldc, st);
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
namespace {

// Sort key of an entry of a band: column, then row in the band, then the fp16 value bits.
uint64_t band_key(int col, int row_in_band, float v) {
    const __half hv = __float2half_rn(v);
    unsigned short bits;
    std::memcpy(&bits, &hv, sizeof bits);
    return (uint64_t(uint32_t(col)) << 32) | (uint64_t(row_in_band) << 16) | bits;
}

// Greedy tiles over a band's keys sorted by column: a tile starts at the first column not yet
// covered and covers kBandK columns. Returns the number of tiles.
int64_t count_tiles(const uint64_t* kb, const uint64_t* ke) {
    int64_t n = 0;
    int64_t end = -1;  // first column past the current tile
    for (const uint64_t* k = kb; k < ke; ++k) {
        const int64_t c = int64_t(*k >> 32);
        if (c >= end) {
            ++n;
            end = c + kBandK;
        }
    }
    return n;
}

void band_keys(const RowViewHost& rv, int r0, int r1, uint64_t* out) {
    for (int r = r0; r < r1; ++r)
        for (int p = rv.rp[r]; p < rv.rp[r + 1]; ++p) *out++ = band_key(rv.cols[p], r - r0, rv.vals[p]);
}

}  // namespace

BandChoice choose_band_sampled(int M, const BandSampleFetch& fetch) {
    static const int kCandidates[] = {128, 127, 126, 124, 120, 112, 96, 64, 62, 60, 56, 48, 32};
    BandChoice best{kBandRows, 0.0};
    if (M <= 0) return best;
    // Up to 64 bands spread over the matrix, for every candidate height.
    std::vector<std::pair<int, int>> ranges;
    for (const int H : kCandidates) {
        const int nb = (M + H - 1) / H;
        const int samples = std::min(nb, 64);
        for (int k = 0; k < samples; ++k) {
            const int r0 = int(int64_t(k) * nb / samples) * H;
            ranges.emplace_back(r0, std::min(M, r0 + H));
        }
    }
    std::vector<const int*> first(ranges.size()), last(ranges.size());
    fetch(ranges, first, last);
    double best_cost = 0.0;
    std::vector<int> cols;
    size_t i = 0;
    for (const int H : kCandidates) {
        const int samples = std::min((M + H - 1) / H, 64);
        int64_t tiles = 0, rows = 0, ents = 0, dense = 0;
        for (int k = 0; k < samples; ++k, ++i) {
            cols.assign(first[i], last[i]);
            std::sort(cols.begin(), cols.end());
            int64_t end = -1, in_tile = 0;  // greedy tiles, as build_band_view cuts them
            for (const int c : cols) {
                if (c >= end) {
                    if (in_tile >= int64_t(kBandMinEntriesPerTile)) dense += in_tile;
                    ++tiles;
                    end = int64_t(c) + kBandK;
                    in_tile = 0;
                }
                ++in_tile;
            }
            if (in_tile >= int64_t(kBandMinEntriesPerTile)) dense += in_tile;
            rows += ranges[i].second - ranges[i].first;
            ents += int64_t(cols.size());
        }
        // tensor-core time per row: a tile of a band of at most 64 rows (N = 64) takes 1.85 ns on a
        // B200, one of a taller band (N = 128) 2.18 ns; plus about half a tile per band
        const double tile_cost = H <= 64 ? 1.0 : 1.17;
        const double cost = (double(tiles) * tile_cost + 0.5 * samples) / double(std::max<int64_t>(rows, 1));
        if (H == kCandidates[0] || cost < best_cost * 0.995) {
            best_cost = cost;
            best = BandChoice{H, tiles > 0 ? double(ents) / double(tiles) : 0.0,
                              ents > 0 ? double(dense) / double(ents) : 0.0};
        }
    }
    return best;
}

BandChoice choose_band(const RowViewHost& rv, int M) {
    return choose_band_sampled(M, [&](const std::vector<std::pair<int, int>>& ranges, std::vector<const int*>& first,
                                      std::vector<const int*>& last) {
        for (size_t i = 0; i < ranges.size(); ++i) {
            first[i] = rv.cols.data() + rv.rp[size_t(ranges[i].first)];
            last[i] = rv.cols.data() + rv.rp[size_t(ranges[i].second)];
        }
    });
}

void split_dense_tiles(const RowViewHost& rv, const BandViewHost& bv, int M, int min_entries, int nthreads,
                       RowViewHost& dense, RowViewHost& resid) {
    const int H = bv.band_rows;
    const int nb = int(bv.tile_ptr.size()) - 1;
    const int64_t nnz = M > 0 ? rv.rp[M] : 0;
    if (nb != (M + H - 1) / H) throw StatusError(VCSRMC_INTERNAL, "band view does not match the row view");
    std::vector<uint8_t> in_dense(size_t(std::max<int64_t>(nnz, 1)), 0);
    dense.rp.assign(size_t(M) + 1, 0);
    resid.rp.assign(size_t(M) + 1, 0);
    const int nth = resolve_threads(nthreads);
    parallel_for_dynamic(0, nb, nth, 64, [&](int64_t lo, int64_t hi) {
        for (int64_t b = lo; b < hi; ++b) {
            const int t0 = bv.tile_ptr[size_t(b)], t1 = bv.tile_ptr[size_t(b) + 1];
            for (int r = int(b) * H; r < std::min(M, int(b + 1) * H); ++r) {
                int t = t0, nd = 0;
                for (int p = rv.rp[r]; p < rv.rp[r + 1]; ++p) {  // columns ascend, and so do the tiles
                    const int c = rv.cols[size_t(p)];
                    while (t + 1 < t1 && bv.tile_col[size_t(t) + 1] <= c) ++t;
                    if (t >= t1 || c < bv.tile_col[size_t(t)] || c >= bv.tile_col[size_t(t)] + kBandK)
                        throw StatusError(VCSRMC_INTERNAL, "entry outside its band's tiles");
                    const bool d = bv.tile_eptr[size_t(t) + 1] - bv.tile_eptr[size_t(t)] >= min_entries;
                    in_dense[size_t(p)] = d ? 1 : 0;
                    nd += d ? 1 : 0;
                }
                dense.rp[size_t(r) + 1] = nd;
                resid.rp[size_t(r) + 1] = (rv.rp[r + 1] - rv.rp[r]) - nd;
            }
        }
    });
    for (int r = 0; r < M; ++r) {
        dense.rp[size_t(r) + 1] += dense.rp[size_t(r)];
        resid.rp[size_t(r) + 1] += resid.rp[size_t(r)];
    }
    dense.cols.resize(size_t(dense.rp[size_t(M)]));
    dense.vals.resize(dense.cols.size());
    resid.cols.resize(size_t(resid.rp[size_t(M)]));
    resid.vals.resize(resid.cols.size());
    parallel_for(0, M, nth, [&](int64_t lo, int64_t hi) {
        for (int64_t r = lo; r < hi; ++r) {
            int qd = dense.rp[size_t(r)], qr = resid.rp[size_t(r)];
            for (int p = rv.rp[r]; p < rv.rp[r + 1]; ++p) {
                if (in_dense[size_t(p)]) {
                    dense.cols[size_t(qd)] = rv.cols[size_t(p)];
                    dense.vals[size_t(qd++)] = rv.vals[size_t(p)];
                } else {
                    resid.cols[size_t(qr)] = rv.cols[size_t(p)];
                    resid.vals[size_t(qr++)] = rv.vals[size_t(p)];
                }
            }
        }
    });
}

BandViewHost build_band_view(const RowViewHost& rv, int M, int band_rows, int nthreads) {
    if (band_rows < 1 || band_rows > kBandRows) throw StatusError(VCSRMC_INTERNAL, "band height out of range");
    BandViewHost h;
    h.band_rows = band_rows;
    const int H = band_rows;
    const int nb = (M + H - 1) / H;
    const int64_t nnz = M > 0 ? rv.rp[M] : 0;
    std::vector<uint64_t> keys(size_t(std::max<int64_t>(nnz, 0)));
    std::vector<int> ntiles(size_t(nb), 0);
    const int nth = resolve_threads(nthreads);
    parallel_for_dynamic(0, nb, nth, 64, [&](int64_t lo, int64_t hi) {
        for (int64_t b = lo; b < hi; ++b) {
            const int r0 = int(b) * H, r1 = std::min(M, r0 + H);
            uint64_t* kb = keys.data() + rv.rp[r0];
            uint64_t* ke = keys.data() + rv.rp[r1];
            band_keys(rv, r0, r1, kb);
            std::sort(kb, ke);
            ntiles[size_t(b)] = int(count_tiles(kb, ke));
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
            const int r0 = int(b) * H, r1 = std::min(M, r0 + H);
            int t = h.tile_ptr[size_t(b)] - 1;
            int64_t end = -1, start = 0;
            for (int p = rv.rp[r0]; p < rv.rp[r1]; ++p) {
                const uint64_t k = keys[size_t(p)];
                const int64_t c = int64_t(k >> 32);
                if (c >= end) {  // a new tile starts at this column
                    ++t;
                    start = c;
                    end = c + kBandK;
                    h.tile_col[size_t(t)] = int(c);
                    h.tile_eptr[size_t(t)] = p;
                }
                const uint32_t row = uint32_t(k >> 16) & 0x7fu, bits = uint32_t(k & 0xffffu);
                h.ents[size_t(p)] = uint32_t(c - start) | (row << kBandColBits) | (bits << 16);
            }
        }
    });
    // Every index the kernel follows stays inside its array: checked once here.
    auto bad = [] { throw StatusError(VCSRMC_INTERNAL, "band view construction is inconsistent"); };
    for (int b = 0; b < nb; ++b) {
        const int t0 = h.tile_ptr[size_t(b)], t1 = h.tile_ptr[size_t(b) + 1];
        if (t1 < t0 || t1 > T) bad();
        const int r0 = b * H, r1 = std::min(M, r0 + H);
        if (t1 > t0 && (h.tile_eptr[size_t(t0)] != rv.rp[r0] || h.tile_eptr[size_t(t1)] != rv.rp[r1])) bad();
        if (t1 == t0 && rv.rp[r1] != rv.rp[r0]) bad();
        for (int t = t0; t < t1; ++t)
            if (h.tile_eptr[size_t(t) + 1] <= h.tile_eptr[size_t(t)] || h.tile_col[size_t(t)] < 0 ||
                (t > t0 && h.tile_col[size_t(t)] < h.tile_col[size_t(t) - 1] + kBandK))
                bad();
    }
    return h;
}

}  // namespace dev
}  // namespace vcsrmc
