// Row-stationary execution plan for VCSR-MC SpMM (C written once per row, no C reductions
// except for the chunks of rows that are split across warps).
//
// The reference's dataflow (src/vcsr_mc.cu:143-237) walks the format segment by segment and adds
// every 16-row group into C with atomics. At scale that costs 16 rows x O fp32
// read-modify-writes per group: for the 2^24-row R-MAT about 127 GB of reductions for a
// 12 GB job. This plan consumes the same VCSR-MC data transposed at upload time into a row
// view: row r's entries are its (group, lane) slots over all groups in format order, i.e. in
// ascending segment and local column. A lane group owns a unit of work:
//   * a run of up to kUnitRows consecutive light rows with together <= unit_nnz entries, or
//   * one unit_nnz-entry chunk of a heavy row (more than unit_nnz entries);
// unit_nnz (16 .. 1024) is chosen per matrix at upload: small matrices get small units so that
// every SM has enough lane groups in flight.
// each lane gathers 16 bytes of every entry's B row (fp16 B: 16 lanes cover one 256-byte row,
// so a warp runs two units; fp32 B: 32 lanes), accumulates in fp32 registers, and stores a C
// row once, at its last entry (16-byte streaming stores); a heavy-row chunk adds its partial
// row with 16-byte vector reductions instead. The group streams the unit's entries in batches
// regardless of row boundaries: the row of each entry comes from a 4-step shuffle search over
// the unit's row ends and a ballot marks the last entry of every row.
// A values and column indices are streamed (evict-first); B keeps the default caching so hot
// columns stay in L1/L2.
// Hot columns: the row view may number its most used columns by rank (entries hold ~rank, see
// RowHotView). Each call then first copies the B rows of the leading ranks into one compact
// buffer (hot_rows_copy_kernel), optionally under a persisting L2 access-policy window, and an
// entry's B row is read from there. The values read and the order of the FMAs are the same as
// without the copy, so C is bit-identical either way.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <vector>

#include "common.cuh"
#include "plan_rows.hpp"

namespace vcsrmc {
namespace dev {
namespace {

// Build-time shape of vcsr_rows_kernel: warps per block, the minimum resident blocks per SM the
// register budget is sized for (per B element type), B gathers in flight per lane. Gathers in
// flight per SM decide its speed. On the 2^24-row R-MAT with fp16 B: 4-warp blocks whose A values
// are read back from shared memory at their FMA, held to 64 registers (8 blocks = 32 warps per SM),
// run in 9.30 ms, against 10.24 ms for the same blocks holding the 8 A values in registers at 72
// registers (7 blocks), and 10.50 ms for 8-warp blocks at 80 registers; 16 gathers in flight per
// lane at 128 registers (16 warps) took 11.21 ms. With fp32 B the 64-register build lost (16.29
// against 15.21 ms), so fp32 B keeps 7 blocks of 72 registers.
#ifndef VCSRMC_ROWS_WARPS
#define VCSRMC_ROWS_WARPS 4
#endif
#ifndef VCSRMC_ROWS_IN_FLIGHT
#define VCSRMC_ROWS_IN_FLIGHT 8
#endif
constexpr int kWarpsPerBlock = VCSRMC_ROWS_WARPS;
// Resident blocks per SM that the register budget of vcsr_rows_kernel is sized for, and whether
// the staged A values are read back from shared memory at their FMA (instead of held in registers
// while the gathers are in flight), by B element size.
template <typename BT>
struct RowsShape {
    static constexpr int kMinBlocks = sizeof(BT) == 2 ? 8 : 7;
    static constexpr bool kReloadA = sizeof(BT) == 2;
    // vcsr_rows_folded_kernel (8-warp blocks): 4 blocks = 64 registers for fp16 B; 0 = not given
    static constexpr int kFoldedMinBlocks = sizeof(BT) == 2 ? 4 : 0;
};
constexpr int kFoldedWarpsPerBlock = 8;  // vcsr_rows_folded_kernel (narrow B)
constexpr unsigned kFull = 0xffffffffu;

// One lane's share of an entry's B row: 16 bytes = 8 fp16 or 4 fp32 consecutive columns.
template <typename BT>
struct Lane16 {
    static constexpr int kElems = 16 / int(sizeof(BT));  // columns per lane
    static constexpr int kLanes = 128 / kElems;          // lanes per entry (one 128-column slab)
};

template <bool kVec, typename BT>
__device__ __forceinline__ uint4 load16(const BT* p, int nv) {
    if (kVec && nv == Lane16<BT>::kElems) return __ldg(reinterpret_cast<const uint4*>(p));
    // ragged tail of O, or unaligned B: element by element, zero beyond O
    uint32_t w[4] = {0u, 0u, 0u, 0u};
    if constexpr (sizeof(BT) == 2) {
        const unsigned short* q = reinterpret_cast<const unsigned short*>(p);
        for (int i = 0; i < nv; ++i) w[i >> 1] |= uint32_t(q[i]) << ((i & 1) * 16);
    } else {
        const uint32_t* q = reinterpret_cast<const uint32_t*>(p);
        for (int i = 0; i < nv; ++i) w[i] = q[i];
    }
    return make_uint4(w[0], w[1], w[2], w[3]);
}

// Same, for a B row read once in a while: evict-first in L1 and L2 (ld.global.cs), so that it does not
// displace the popular rows.
template <bool kVec, typename BT>
__device__ __forceinline__ uint4 load16_once(const BT* p, int nv) {
    if (kVec && nv == Lane16<BT>::kElems) return __ldcs(reinterpret_cast<const uint4*>(p));
    return load16<false>(p, nv);
}

// acc[i] += a * B_lane[i]. fp16 x fp16 uses the mixed-precision FMA (f16 inputs, f32 accumulate:
// the product of two f16 values is exact in f32, so this equals converting first and FFMA).
__device__ __forceinline__ void fma2_f16(float& d0, float& d1, unsigned short a, uint32_t b2) {
    asm("{\n\t.reg .b16 blo, bhi;\n\t"
        "mov.b32 {blo, bhi}, %3;\n\t"
        "fma.rn.f32.f16 %0, %2, blo, %0;\n\t"
        "fma.rn.f32.f16 %1, %2, bhi, %1;\n\t}"
        : "+f"(d0), "+f"(d1)
        : "h"(a), "r"(b2));
}
// a holds the A value: fp16 bits in the low half (fp16 x fp16) or fp32 bits (otherwise)
template <typename VT, typename BT>
__device__ __forceinline__ void fma_lane(float (&acc)[8], uint32_t a, const uint4& r) {
    if constexpr (sizeof(BT) == 2) {
        const uint32_t w[4] = {r.x, r.y, r.z, r.w};
        if constexpr (sizeof(VT) == 2) {
#pragma unroll
            for (int i = 0; i < 4; ++i) fma2_f16(acc[2 * i], acc[2 * i + 1], (unsigned short)(a & 0xffffu), w[i]);
        } else {
            const float af = __uint_as_float(a);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
                acc[2 * i] = fmaf(af, f.x, acc[2 * i]);
                acc[2 * i + 1] = fmaf(af, f.y, acc[2 * i + 1]);
            }
        }
    } else {
        const float af = __uint_as_float(a);
        acc[0] = fmaf(af, __uint_as_float(r.x), acc[0]);
        acc[1] = fmaf(af, __uint_as_float(r.y), acc[1]);
        acc[2] = fmaf(af, __uint_as_float(r.z), acc[2]);
        acc[3] = fmaf(af, __uint_as_float(r.w), acc[3]);
    }
}

// The A value of an entry as the bits fma_lane expects.
template <typename VT, typename BT>
__device__ __forceinline__ uint32_t a_bits(const VT* p) {
    if constexpr (sizeof(VT) == 2) {
        const unsigned short h = __ldcs(reinterpret_cast<const unsigned short*>(p));
        if constexpr (sizeof(BT) == 2) return h;
        return __float_as_uint(__half2float(__ushort_as_half(h)));
    } else {
        return __float_as_uint(__ldcs(p));
    }
}

// C row segment of this lane: kE columns at dst (nv valid). Overwrite, add, or reduce. A row of C
// belongs to one lane group (or, split into chunks, is reduced by several): adding into it is a
// fire-and-forget vector reduction (red.global.add.v4.f32), one fp32 add of the row's sum to the
// old value as a load-add-store would do, without waiting for the old value at every row end
// (accumulate mode, config 4: 10.15 -> 8.49 ms; config-2 matrix, O = 16-128: 22-31 % faster).
enum class RowOut { kStore, kAdd, kReduce };
template <int kE, bool kVec, RowOut kOut>
__device__ __forceinline__ void write_lane(float* dst, const float (&acc)[8], float scale, int nv) {
    float v[8];
#pragma unroll
    for (int i = 0; i < kE; ++i) v[i] = acc[i] * scale;
    if (kVec && nv == kE) {
#pragma unroll
        for (int i = 0; i < kE; i += 4) {
            float4 x = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
            float4* d4 = reinterpret_cast<float4*>(dst + i);
            if constexpr (kOut == RowOut::kStore) __stcs(d4, x);
            else atomicAdd(d4, x);
        }
    } else {
        for (int i = 0; i < nv; ++i) {
            if constexpr (kOut == RowOut::kStore) dst[i] = v[i];
            else atomicAdd(dst + i, v[i]);
        }
    }
}

// An entry as the gather loop reads it from shared memory: the byte offset of its B row (relative
// to B, or to the compact hot rows through hot_delta) and its A value bits.
struct alignas(16) Staged {
    long long off;
    uint32_t v;
    uint32_t once;  // 1: a row outside the hot set, read with evict-first
};

// Where a row-view entry's B row is: column c >= 0 is row c of B; a hot entry (~rank) below k_copy
// is row `rank` of the compact copy (hot_delta = copy - B, in bytes); other hot ranks are looked up.
__device__ __forceinline__ long long entry_offset(int c, int row_bytes, const int* __restrict__ hot_cols, int k_copy,
                                                 long long hot_delta) {
    if (c >= 0) return (long long)c * row_bytes;
    const int r = ~c;
    if (r < k_copy) return hot_delta + (long long)r * row_bytes;
    return (long long)__ldg(hot_cols + r) * row_bytes;
}

constexpr int kInFlight = VCSRMC_ROWS_IN_FLIGHT;  // B gathers in flight per lane
static_assert(kInFlight == 8 || kInFlight == 16, "a batch of 16 entries in rounds of 8 or 16");

// A lane group (kL lanes: 16 for fp16 B, 32 for fp32 B) owns one work unit and one 128-column
// slab of C; lane sl of the group holds columns c0 .. c0+kE-1 of it. Per batch of kL entries the
// group stages (B row offset, A value) in shared memory (one broadcast read per entry later),
// pads the batch past the unit's end with (column 0, value 0) so no bounds tests are needed,
// and gathers B eight entries at a time; runs of eight entries without a row end skip the
// per-entry row-end test.
template <bool kVec, bool kAccumulate, typename VT, typename BT, bool kRec16>
__global__ void __launch_bounds__(kWarpsPerBlock * 32, RowsShape<BT>::kMinBlocks)
    vcsr_rows_kernel(const int4* __restrict__ units, int64_t n_units, const int* __restrict__ rp,
                     const int* __restrict__ cols, const VT* __restrict__ vals, const BT* __restrict__ B,
                     int row_bytes, int O, float* __restrict__ C, int64_t ldc, float scale,
                     const int* __restrict__ hot_cols, int k_copy, long long hot_delta, int cold_hint) {
    constexpr int kE = Lane16<BT>::kElems;
    constexpr int kL = Lane16<BT>::kLanes;
    constexpr int kGroups = 32 / kL;
    constexpr RowOut kOut = kAccumulate ? RowOut::kAdd : RowOut::kStore;
    __shared__ Staged stage_all[kWarpsPerBlock * 32];
    const int lane = threadIdx.x & 31;
    const int sub = lane / kL, sl = lane % kL;
    const unsigned gmask = kL == 32 ? kFull : (0xffffu << (16 * sub));
    Staged* stage = stage_all + (threadIdx.x >> 5) * 32 + sub * kL;
    // fp32 B: an entry is staged as 8 bytes (its B row's offset in 16-byte units, or its column on
    // the element-wise path; A value bits), entry j of lane group g in slot j * kGroups + g, unless
    // the layout needs the 16-byte records (kRec16: hot columns, or B row offsets past 2^32 16-byte
    // units). Config 4, fp32 B: 14.43 / 14.83 against 14.79 / 15.28 ms with 16-byte records (two
    // boxes). With fp16 B the 64-register build then spills, and the 16-byte records stay faster
    // (8.94-9.07 against 9.31-9.38 ms).
    constexpr bool kCompact = !kRec16 && sizeof(BT) == 4;
    uint2* rec = reinterpret_cast<uint2*>(stage_all + (threadIdx.x >> 5) * 32) + sub;
    const int64_t unit = (int64_t(blockIdx.x) * kWarpsPerBlock + (threadIdx.x >> 5)) * kGroups + sub;
    if (unit >= n_units) return;  // the whole group leaves together
    const int4 u = units[unit];
    const int c0 = blockIdx.y * 128 + kE * sl;
    const int nv = max(0, min(kE, O - c0));
    const char* bbase = reinterpret_cast<const char*>(B) + size_t(c0) * sizeof(BT);
    const bool partial = (u.y & 0x80000000) != 0;
    const int rb = u.x, pb = u.z, pe = u.w;
    const int nrows = partial ? 1 : (u.y & 0x7fffffff) - rb;

    // Row ends of the unit's rows (<= kUnitRows <= kL), one per lane.
    const int my_end = (!partial && sl < nrows) ? rp[rb + sl + 1] : 0x7fffffff;
    if (!partial && !kAccumulate) {
        // rows without entries are written here; the others when their last entry is done
        // (every lane of the group takes part in the shuffle; lane 0's result is replaced)
        const int prev_end = __shfl_up_sync(gmask, my_end, 1, kL);
        const int my_start = sl == 0 ? pb : prev_end;
        unsigned empty = __ballot_sync(gmask, sl < nrows && my_start == my_end);
        if (kL == 16) empty = (empty >> (16 * sub)) & 0xffffu;
        const float zero[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        while (empty) {
            const int i = __ffs(empty) - 1;
            empty &= empty - 1;
            write_lane<kE, kVec, RowOut::kStore>(C + int64_t(rb + i) * ldc + c0, zero, 1.f, nv);
        }
    }

    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    // (column, A value) of the lane's entry in the next batch; (0, 0) past the unit's end
    int mc = 0;
    uint32_t mv = 0;
    if (pb + sl < pe) {
        mc = __ldcs(cols + pb + sl);
        mv = a_bits<VT, BT>(vals + pb + sl);
    }
    for (int q = pb; q < pe; q += kL) {
        const int n = min(kL, pe - q);
        if constexpr (!kCompact)
            stage[sl] = kRec16 ? Staged{entry_offset(mc, row_bytes, hot_cols, k_copy, hot_delta), mv,
                                        uint32_t(cold_hint & (mc >= 0))}
                               : Staged{(long long)mc * row_bytes, mv, 0u};
        else
            rec[sl * kGroups] = make_uint2(kVec ? uint32_t(mc) * uint32_t(row_bytes >> 4) : uint32_t(mc), mv);
        mc = 0;
        mv = 0;
        if (q + kL + sl < pe) {
            mc = __ldcs(cols + q + kL + sl);
            mv = a_bits<VT, BT>(vals + q + kL + sl);
        }
        // local row of this lane's entry (number of unit rows that end at or before it), and
        // whether the entry is the last of its row
        int lo = 0;
        unsigned ends = 0;
        if (!partial) {
            const int e = q + sl;
#pragma unroll
            for (int step = kUnitRows / 2; step >= 1; step >>= 1) {
                const int probe = __shfl_sync(gmask, my_end, (lo + step - 1) & (kL - 1), kL);
                if (probe <= e) lo += step;
            }
            const int row_end = __shfl_sync(gmask, my_end, lo & (kL - 1), kL);
            ends = __ballot_sync(gmask, sl < n && e + 1 == row_end);
            if (kL == 16) ends = (ends >> (16 * sub)) & 0xffffu;
        }
        __syncwarp(gmask);
        for (int j = 0; j < n; j += kInFlight) {
            uint4 raw[kInFlight];
            uint32_t av[kInFlight];  // held only when RowsShape<BT>::kReloadA is false
#pragma unroll
            for (int k = 0; k < kInFlight; ++k) {
                if constexpr (!kCompact) {
                    const Staged e = stage[j + k];
                    if constexpr (!RowsShape<BT>::kReloadA) av[k] = e.v;
                    const BT* p = reinterpret_cast<const BT*>(bbase + e.off);
                    // the evict-first flag is read only where hot columns can set it (config 4,
                    // fp16 B: 9.00 against 9.30-9.38 ms with the flag read for every entry)
                    if constexpr (kRec16) raw[k] = e.once ? load16_once<kVec>(p, nv) : load16<kVec>(p, nv);
                    else raw[k] = load16<kVec>(p, nv);
                } else {
                    const uint32_t c = reinterpret_cast<const uint32_t*>(rec + (j + k) * kGroups)[0];
                    if constexpr (!RowsShape<BT>::kReloadA) av[k] = rec[(j + k) * kGroups].y;
                    const BT* p = reinterpret_cast<const BT*>(kVec ? bbase + size_t(c) * 16u
                                                                   : bbase + (long long)int(c) * row_bytes);
                    raw[k] = load16<kVec>(p, nv);
                }
            }
            // A value of entry j + k at its FMA: from shared memory (8 registers fewer held while the
            // gathers are in flight) or from the registers loaded with the gathers
            auto a_of = [&](int k) -> uint32_t {
                if constexpr (RowsShape<BT>::kReloadA) {
                    if constexpr (!kCompact) return stage[j + k].v;
                    else return rec[(j + k) * kGroups].y;
                } else {
                    return av[k];
                }
            };
            const unsigned eb = (ends >> j) & ((1u << kInFlight) - 1u);
            if (eb == 0) {
#pragma unroll
                for (int k = 0; k < kInFlight; ++k) fma_lane<VT, BT>(acc, a_of(k), raw[k]);
            } else {
#pragma unroll
                for (int k = 0; k < kInFlight; ++k) {
                    fma_lane<VT, BT>(acc, a_of(k), raw[k]);
                    if ((eb >> k) & 1u) {
                        const int row = rb + __shfl_sync(gmask, lo, j + k, kL);
                        write_lane<kE, kVec, kOut>(C + int64_t(row) * ldc + c0, acc, scale, nv);
#pragma unroll
                        for (int i = 0; i < 8; ++i) acc[i] = 0.f;
                    }
                }
            }
        }
        __syncwarp(gmask);
    }
    if (partial) write_lane<kE, kVec, RowOut::kReduce>(C + int64_t(rb) * ldc + c0, acc, scale, nv);
}

// The same plan for narrow B on the element-wise path (O <= kL * kE / 2 columns: 64 fp16, 64 fp32):
// a row slice of B then needs only kW = kL / kF lanes, so each lane group works on kF entries at
// once. Fold f of the group (lanes f * kW .. f * kW + kW - 1) takes entries f, f + kF, f + 2 kF, ...
// of every staged batch. Per step of kF consecutive entries the folds' contributions to the same
// row are summed across folds with shuffles (rows are non-decreasing along the entries, so the
// folds sharing a row are contiguous); a row that continues past a step is carried in every
// lane's accumulator; the fold holding a row's last entry writes the row.
template <int kF, bool kVec, bool kAccumulate, typename VT, typename BT>
__global__ void __launch_bounds__(kFoldedWarpsPerBlock * 32, RowsShape<BT>::kFoldedMinBlocks)
    vcsr_rows_folded_kernel(const int4* __restrict__ units, int64_t n_units, const int* __restrict__ rp,
                            const int* __restrict__ cols, const VT* __restrict__ vals, const BT* __restrict__ B,
                            int row_bytes, int O, float* __restrict__ C, int64_t ldc, float scale,
                            const int* __restrict__ hot_cols, int k_copy, long long hot_delta, int cold_hint) {
    constexpr int kE = Lane16<BT>::kElems;
    constexpr int kL = Lane16<BT>::kLanes;
    constexpr int kW = kL / kF;        // lanes per entry
    constexpr int kSteps = kL / kF;    // steps per staged batch of kL entries
    constexpr int kR = kSteps < kInFlight ? kSteps : kInFlight;
    constexpr int kGroups = 32 / kL;
    constexpr RowOut kOut = kAccumulate ? RowOut::kAdd : RowOut::kStore;
    static_assert(kF == 2 || kF == 4, "fold of 2 or 4 entries");
    __shared__ Staged stage_all[kFoldedWarpsPerBlock * 32];
    const int lane = threadIdx.x & 31;
    const int sub = lane / kL, sl = lane % kL;
    const int fold = sl / kW, cl = sl % kW;
    const unsigned gmask = kL == 32 ? kFull : (0xffffu << (16 * sub));
    Staged* stage = stage_all + (threadIdx.x >> 5) * 32 + sub * kL;
    const int64_t unit = (int64_t(blockIdx.x) * kFoldedWarpsPerBlock + (threadIdx.x >> 5)) * kGroups + sub;
    if (unit >= n_units) return;  // the whole group leaves together
    const int4 u = units[unit];
    const int c0 = kE * cl;  // one slab: O <= kW * kE
    const int nv = max(0, min(kE, O - c0));
    const char* bbase = reinterpret_cast<const char*>(B) + size_t(c0) * sizeof(BT);
    const bool partial = (u.y & 0x80000000) != 0;
    const int rb = u.x, pb = u.z, pe = u.w;
    const int nrows = partial ? 1 : (u.y & 0x7fffffff) - rb;

    const int my_end = (!partial && sl < nrows) ? rp[rb + sl + 1] : 0x7fffffff;
    if (!partial && !kAccumulate) {
        const int prev_end = __shfl_up_sync(gmask, my_end, 1, kL);
        const int my_start = sl == 0 ? pb : prev_end;
        unsigned empty = __ballot_sync(gmask, sl < nrows && my_start == my_end);
        if (kL == 16) empty = (empty >> (16 * sub)) & 0xffffu;
        const float zero[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        while (empty) {
            const int i = __ffs(empty) - 1;
            empty &= empty - 1;
            if (fold == 0) write_lane<kE, kVec, RowOut::kStore>(C + int64_t(rb + i) * ldc + c0, zero, 1.f, nv);
        }
    }

    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};  // the open row's sum (same in every fold)
    int open_row = -1;
    int mc = 0;
    uint32_t mv = 0;
    if (pb + sl < pe) {
        mc = __ldcs(cols + pb + sl);
        mv = a_bits<VT, BT>(vals + pb + sl);
    }
    for (int q = pb; q < pe; q += kL) {
        const int n = min(kL, pe - q);
        stage[sl] = Staged{entry_offset(mc, row_bytes, hot_cols, k_copy, hot_delta), mv, uint32_t(cold_hint & (mc >= 0))};
        mc = 0;
        mv = 0;
        if (q + kL + sl < pe) {
            mc = __ldcs(cols + q + kL + sl);
            mv = a_bits<VT, BT>(vals + q + kL + sl);
        }
        int lo = 0;
        unsigned ends = 0;
        if (!partial) {
            const int e = q + sl;
#pragma unroll
            for (int step = kUnitRows / 2; step >= 1; step >>= 1) {
                const int probe = __shfl_sync(gmask, my_end, (lo + step - 1) & (kL - 1), kL);
                if (probe <= e) lo += step;
            }
            const int row_end = __shfl_sync(gmask, my_end, lo & (kL - 1), kL);
            ends = __ballot_sync(gmask, sl < n && e + 1 == row_end);
            if (kL == 16) ends = (ends >> (16 * sub)) & 0xffffu;
        }
        __syncwarp(gmask);
        for (int t0 = 0; t0 < kSteps; t0 += kR) {
            uint4 raw[kR];
            uint32_t av[kR];  // held only when RowsShape<BT>::kReloadA is false
#pragma unroll
            for (int k = 0; k < kR; ++k) {
                const Staged e = stage[(t0 + k) * kF + fold];
                if constexpr (!RowsShape<BT>::kReloadA) av[k] = e.v;
                const BT* p = reinterpret_cast<const BT*>(bbase + e.off);
                raw[k] = e.once ? load16_once<kVec>(p, nv) : load16<kVec>(p, nv);
            }
            auto a_of = [&](int k) -> uint32_t {
                if constexpr (RowsShape<BT>::kReloadA) return stage[(t0 + k) * kF + fold].v;
                else return av[k];
            };
#pragma unroll
            for (int k = 0; k < kR; ++k) {
                const int j0 = (t0 + k) * kF;  // first entry of this step
                int row[kF];
#pragma unroll
                for (int g = 0; g < kF; ++g) row[g] = __shfl_sync(gmask, lo, j0 + g, kL);
                float c[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
                fma_lane<VT, BT>(c, a_of(k), raw[k]);
                float v[8];
                const bool carry_in = row[fold] == open_row;
#pragma unroll
                for (int i = 0; i < 8; ++i) v[i] = c[i] + (carry_in ? acc[i] : 0.f);
#pragma unroll
                for (int d = 1; d < kF; ++d) {
                    const bool same = fold >= d && row[fold - d] == row[fold];
#pragma unroll
                    for (int i = 0; i < kE; ++i) {
                        const float o = __shfl_up_sync(gmask, c[i], d * kW, kL);
                        if (same) v[i] += o;
                    }
                }
                if ((ends >> (j0 + fold)) & 1u)
                    write_lane<kE, kVec, kOut>(C + int64_t(rb + row[fold]) * ldc + c0, v, scale, nv);
                if ((ends >> (j0 + kF - 1)) & 1u) {
                    open_row = -1;
#pragma unroll
                    for (int i = 0; i < 8; ++i) acc[i] = 0.f;
                } else {
                    open_row = row[kF - 1];
#pragma unroll
                    for (int i = 0; i < kE; ++i) acc[i] = __shfl_sync(gmask, v[i], (kF - 1) * kW + cl, kL);
                }
            }
        }
        __syncwarp(gmask);
    }
    if (partial && fold == 0) write_lane<kE, kVec, RowOut::kReduce>(C + int64_t(rb) * ldc + c0, acc, scale, nv);
}

// Zeroes C's heavy rows (the ones built from several reduced chunks) before an overwrite.
__global__ void zero_rows_kernel(const int* __restrict__ rows, int n_rows, int O, float* __restrict__ C, int64_t ldc) {
    const int i = blockIdx.x;
    if (i >= n_rows) return;
    float* dst = C + int64_t(rows[i]) * ldc;
    for (int c = threadIdx.x; c < O; c += blockDim.x) dst[c] = 0.f;
}

// Copies the B rows of hot ranks 0 .. k-1 into `dst` (row r of dst = B row hot_cols[r], same row
// pitch); only the first copy_bytes of each row (the O columns read) are copied. 16 lanes per row,
// 16 bytes per lane when B's rows are 16-byte aligned, 2 bytes otherwise.
__global__ void hot_rows_copy_kernel(const int* __restrict__ hot_cols, int k, const char* __restrict__ B,
                                     int row_bytes, int copy_bytes, char* __restrict__ dst, int vec) {
    const int64_t tid = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t groups = int64_t(gridDim.x) * blockDim.x / 16;
    const int sl = int(tid & 15);
    const int vec_bytes = vec ? (copy_bytes & ~15) : 0;
    for (int64_t r = tid >> 4; r < k; r += groups) {
        const char* src = B + int64_t(__ldg(hot_cols + r)) * row_bytes;
        char* d = dst + r * row_bytes;
        for (int b = sl * 16; b < vec_bytes; b += 256)
            *reinterpret_cast<uint4*>(d + b) = __ldg(reinterpret_cast<const uint4*>(src + b));
        for (int b = vec_bytes + sl * 2; b < copy_bytes; b += 32)
            *reinterpret_cast<unsigned short*>(d + b) = *reinterpret_cast<const unsigned short*>(src + b);
    }
}

// Launch configuration of the plan's kernels, with the persisting L2 window over the compact hot
// rows when that is asked for.
struct LaunchShape {
    cudaLaunchConfig_t cfg{};
    cudaLaunchAttribute attr[1];
    LaunchShape(dim3 grid, dim3 block, cudaStream_t st, const void* window, int64_t window_bytes) {
        cfg.gridDim = grid;
        cfg.blockDim = block;
        cfg.dynamicSmemBytes = 0;
        cfg.stream = st;
        cfg.attrs = attr;
        cfg.numAttrs = 0;
        if (window && window_bytes > 0) {
            int dev = 0, max_window = 0;
            size_t persisting = 0;
            cudaGetDevice(&dev);
            cudaDeviceGetAttribute(&max_window, cudaDevAttrMaxAccessPolicyWindowSize, dev);
            cudaDeviceGetLimit(&persisting, cudaLimitPersistingL2CacheSize);
            cudaGetLastError();
            const int64_t bytes = std::min<int64_t>(window_bytes, max_window);
            if (bytes > 0 && persisting > 0) {
                attr[0].id = cudaLaunchAttributeAccessPolicyWindow;
                attr[0].val.accessPolicyWindow.base_ptr = const_cast<void*>(window);
                attr[0].val.accessPolicyWindow.num_bytes = size_t(bytes);
                attr[0].val.accessPolicyWindow.hitRatio = float(std::min(1.0, double(persisting) / double(bytes)));
                attr[0].val.accessPolicyWindow.hitProp = cudaAccessPropertyPersisting;
                attr[0].val.accessPolicyWindow.missProp = cudaAccessPropertyStreaming;
                cfg.numAttrs = 1;
            }
        }
    }
};

template <bool kVec, bool kAcc, typename VT, typename BT>
cudaError_t launch_rows_t(const RowPlanView& P, const BT* B, int64_t ldb, int O, float* C, int64_t ldc,
                          cudaStream_t st) {
    constexpr int kL = Lane16<BT>::kLanes, kE = Lane16<BT>::kElems;
    constexpr int kGroupsPerWarp = 32 / kL;
    const int64_t per_block = int64_t(kWarpsPerBlock) * kGroupsPerWarp;
    const int64_t blocks = (P.n_units + per_block - 1) / per_block;
    const int64_t per_fblock = int64_t(kFoldedWarpsPerBlock) * kGroupsPerWarp;
    const int64_t fblocks = (P.n_units + per_fblock - 1) / per_fblock;
    if (blocks > 0x7fffffffLL) return cudaErrorInvalidValue;
    const int row_bytes = int(ldb * int64_t(sizeof(BT)));
    const VT* vals = static_cast<const VT*>(P.vals);
    // hot rows: copy the leading ranks' B rows into the compact buffer first
    const int k_copy = rows_hot_copy_count(P.hot, row_bytes);
    long long hot_delta = 0;
    const void* window = nullptr;
    int64_t window_bytes = 0;
    if (k_copy > 0) {
        int dev = 0, sms = 1;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        const int64_t copy_blocks = std::min<int64_t>((int64_t(k_copy) * 16 + 255) / 256, int64_t(sms) * 8);
        if (P.hot.persist) {
            window = P.hot.buf;
            window_bytes = int64_t(k_copy) * row_bytes;
        }
        const int copy_vec = (reinterpret_cast<uintptr_t>(B) % 16 == 0) && (row_bytes % 16 == 0);
        LaunchShape L(dim3(unsigned(copy_blocks)), dim3(256), st, window, window_bytes);
        const cudaError_t e = cudaLaunchKernelEx(&L.cfg, hot_rows_copy_kernel, P.hot.hot_cols, k_copy,
                                                 reinterpret_cast<const char*>(B), row_bytes,
                                                 int(O * int64_t(sizeof(BT))), static_cast<char*>(P.hot.buf), copy_vec);
        if (e != cudaSuccess) return e;
        hot_delta = static_cast<const char*>(P.hot.buf) - reinterpret_cast<const char*>(B);
    }
    const int* hot_cols = P.hot.hot_cols;
    const int cold_hint = (P.hot.n_hot > 0 && P.hot.cold_hint) ? 1 : 0;
    // Narrow B on the element-wise path (B or C rows not 16-byte aligned): fold 4 or 2 entries into
    // one lane group when a row slice fits a quarter or half of it. With 16-byte loads the main
    // kernel is faster at every width, its idle lanes included (config-2 matrix, O = 8..64, store
    // mode: fp16 B 0.108-0.112 ms against 0.114-0.136 ms folded, fp32 B 0.140-0.151 against
    // 0.153-0.177 ms; accumulate mode with reductions: fp16 B 0.098-0.102 against 0.119-0.148 ms);
    // on the element-wise path folding wins (O = 33: 0.196 against 0.218 ms).
    if (!kVec && O <= kL * kE / 4) {
        LaunchShape L(dim3(unsigned(fblocks)), dim3(kFoldedWarpsPerBlock * 32), st, window, window_bytes);
        return cudaLaunchKernelEx(&L.cfg, vcsr_rows_folded_kernel<4, kVec, kAcc, VT, BT>, P.units, P.n_units, P.rp,
                                  P.cols, vals, B, row_bytes, O, C, ldc, P.scale, hot_cols, k_copy, hot_delta, cold_hint);
    }
    if (!kVec && O <= kL * kE / 2) {
        LaunchShape L(dim3(unsigned(fblocks)), dim3(kFoldedWarpsPerBlock * 32), st, window, window_bytes);
        return cudaLaunchKernelEx(&L.cfg, vcsr_rows_folded_kernel<2, kVec, kAcc, VT, BT>, P.units, P.n_units, P.rp,
                                  P.cols, vals, B, row_bytes, O, C, ldc, P.scale, hot_cols, k_copy, hot_delta, cold_hint);
    }
    LaunchShape L(dim3(unsigned(blocks), unsigned((O + 127) / 128)), dim3(kWarpsPerBlock * 32), st, window,
                  window_bytes);
    // 16-byte records: hot columns (ranked entries), or B too large for 32-bit row offsets in
    // 16-byte units (kVec) or for int32 columns times the pitch (element-wise path)
    const bool rec16 = P.hot.n_hot > 0 || int64_t(P.N) * (kVec ? row_bytes / 16 : 1) > 0xffffffffLL;
    if (rec16)
        return cudaLaunchKernelEx(&L.cfg, vcsr_rows_kernel<kVec, kAcc, VT, BT, true>, P.units, P.n_units, P.rp, P.cols,
                                  vals, B, row_bytes, O, C, ldc, P.scale, hot_cols, k_copy, hot_delta, cold_hint);
    return cudaLaunchKernelEx(&L.cfg, vcsr_rows_kernel<kVec, kAcc, VT, BT, false>, P.units, P.n_units, P.rp, P.cols,
                              vals, B, row_bytes, O, C, ldc, P.scale, hot_cols, k_copy, hot_delta, cold_hint);
}

template <typename VT, typename BT>
cudaError_t launch_rows_b(const RowPlanView& P, const BT* B, int64_t ldb, int O, float* C, int64_t ldc,
                          bool accumulate, cudaStream_t st) {
    if (ldb * int64_t(sizeof(BT)) > 0x7fffffffLL) return cudaErrorInvalidValue;  // row pitch must fit 31 bits
    // 16-byte B loads and C stores need 16-byte aligned rows
    const bool vec = ((ldb * int64_t(sizeof(BT))) % 16 == 0) && (ldc % 4 == 0) &&
                     (reinterpret_cast<uintptr_t>(B) % 16 == 0) && (reinterpret_cast<uintptr_t>(C) % 16 == 0);
    if (vec) {
        return accumulate ? launch_rows_t<true, true, VT, BT>(P, B, ldb, O, C, ldc, st)
                          : launch_rows_t<true, false, VT, BT>(P, B, ldb, O, C, ldc, st);
    }
    return accumulate ? launch_rows_t<false, true, VT, BT>(P, B, ldb, O, C, ldc, st)
                      : launch_rows_t<false, false, VT, BT>(P, B, ldb, O, C, ldc, st);
}

}  // namespace

int rows_hot_copy_count(const RowHotView& H, int64_t row_bytes) {
    if (!H.buf || H.n_hot <= 0 || H.budget_bytes <= 0 || row_bytes <= 0) return 0;
    const int64_t cap = std::min(H.budget_bytes, H.buf_bytes) / row_bytes;
    return int(std::min<int64_t>(H.n_hot, cap));
}

int rows_launch_count(const RowPlanView& P, int64_t ldb, int b_is_f16, int O, bool accumulate) {
    if (P.n_units == 0 || O == 0) return 0;
    const int64_t row_bytes = ldb * (b_is_f16 ? 2 : 4);
    return (!accumulate && P.n_split_rows > 0 ? 1 : 0) + (rows_hot_copy_count(P.hot, row_bytes) > 0 ? 1 : 0) + 1;
}

cudaError_t spmm_rows(const RowPlanView& P, const void* B, int b_is_f16, int64_t ldb, int O, float* C, int64_t ldc,
                      bool accumulate, cudaStream_t st) {
    if (P.n_units == 0 || O == 0) {
        if (!accumulate && P.M > 0 && O > 0)
            return cudaMemset2DAsync(C, size_t(ldc) * 4, 0, size_t(O) * 4, size_t(P.M), st);
        return cudaSuccess;
    }
    if (!accumulate && P.n_split_rows > 0) {
        zero_rows_kernel<<<P.n_split_rows, 128, 0, st>>>(P.split_rows, P.n_split_rows, O, C, ldc);
        const cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    if (P.vals_f16) {
        if (b_is_f16) return launch_rows_b<__half, __half>(P, static_cast<const __half*>(B), ldb, O, C, ldc, accumulate, st);
        return launch_rows_b<__half, float>(P, static_cast<const float*>(B), ldb, O, C, ldc, accumulate, st);
    }
    return launch_rows_b<float, float>(P, static_cast<const float*>(B), ldb, O, C, ldc, accumulate, st);
}

// ---- host: the row view of a VCSR-MC format ------------------------------------------------------
int choose_unit_nnz(int64_t nnz, int sms) {
    const int64_t target_units = int64_t(std::max(sms, 1)) * 48 * 4;
    int u = 256;
    while (u > 16 && nnz / u < target_units) u >>= 1;
    return u;
}

void pack_units(const int* rp, int M, int unit_nnz, std::vector<RowViewHost::Unit>& units,
                std::vector<int>& split_rows, bool skip_empty) {
    units.clear();
    split_rows.clear();
    // heavy-row chunks first, then runs of light rows
    for (int r = 0; r < M; ++r) {
        const int len = rp[r + 1] - rp[r];
        if (len > unit_nnz) {
            split_rows.push_back(r);
            for (int p = rp[r]; p < rp[r + 1]; p += unit_nnz)
                units.push_back({r, int((unsigned(r + 1)) | 0x80000000u), p, std::min(rp[r + 1], p + unit_nnz)});
        }
    }
    int r = 0;
    while (r < M) {
        if (rp[r + 1] - rp[r] > unit_nnz || (skip_empty && rp[r + 1] == rp[r])) { ++r; continue; }
        const int rb = r;
        int n = 0;
        while (r < M && r - rb < kUnitRows) {
            const int len = rp[r + 1] - rp[r];
            if (len > unit_nnz || (r > rb && n + len > unit_nnz)) break;
            n += len;
            ++r;
        }
        units.push_back({rb, r, rp[rb], rp[r]});
    }
}

RowViewHost build_row_view(const VCSRMC& v, int unit_nnz) {
    RowViewHost h;
    const int M = v.M;
    const int64_t G = int64_t(v.group_depth.size());
    h.rp.assign(size_t(M) + 1, 0);
    // entries per row: for every (group, lane) the non-padding slots (they come first)
    auto lane_count = [&](int64_t g, int lane) {
        int c = 0;
        const int base = v.group_ptr[g];
        while (c < v.group_depth[g] && v.lcol[size_t(base) + size_t(c) * 16 + lane] >= 0) ++c;
        return c;
    };
    for (int64_t g = 0; g < G; ++g)
        for (int lane = 0; lane < 16; ++lane) {
            const int row = v.group_rows[size_t(g) * 16 + lane];
            if (row >= 0) h.rp[size_t(row) + 1] += lane_count(g, lane);
        }
    for (int r = 0; r < M; ++r) h.rp[r + 1] += h.rp[r];
    const int64_t nnz = h.rp[M];
    h.cols.resize(nnz);
    h.vals.resize(nnz);
    std::vector<int> cursor(h.rp.begin(), h.rp.end() - 1);
    // groups are in ascending segment order, slots of a lane in ascending local column, so each
    // row's entries come out in ascending column order
    for (int64_t g = 0; g < G; ++g) {
        const int base = v.group_ptr[g], seg = v.group_seg_base[g];
        for (int lane = 0; lane < 16; ++lane) {
            const int row = v.group_rows[size_t(g) * 16 + lane];
            if (row < 0) continue;
            for (int d = 0; d < v.group_depth[g]; ++d) {
                const size_t s = size_t(base) + size_t(d) * 16 + lane;
                if (v.lcol[s] < 0) break;
                const int dst = cursor[row]++;
                h.cols[dst] = seg + v.lcol[s];
                h.vals[dst] = v.val[s];
            }
        }
    }
    pack_units(h.rp.data(), M, unit_nnz, h.units, h.split_rows);
    return h;
}

}  // namespace dev
}  // namespace vcsrmc
