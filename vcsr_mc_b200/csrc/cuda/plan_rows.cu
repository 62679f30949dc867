// Row-stationary execution plan for VCSR-MC SpMM (C written once per row, no C reductions
// except for the chunks of rows that are split across warps).
//
// The reference's dataflow (src/vcsr_mc.cu:143-237) walks the format segment by segment and adds
// every 16-row group into C with atomics. At scale that costs 16 rows x O fp32
// read-modify-writes per group: for the 2^24-row R-MAT about 127 GB of reductions for a
// 12 GB job. This plan consumes the same VCSR-MC data transposed at upload time into a row
// view: row r's entries are its (group, lane) slots over all groups in format order, i.e. in
// ascending segment and local column. One warp owns a unit of work:
//   * a run of up to kUnitRows consecutive light rows with together <= kUnitNnz entries, or
//   * one kUnitNnz-entry chunk of a heavy row (more than kUnitNnz entries);
// lane l accumulates columns 4l..4l+3 of a 128-column slab in fp32 registers, gathering the B
// row of every entry (fp16: one 8-byte load per lane = one 256-byte line per entry) with eight
// loads in flight per warp; then stores the C row once (16-byte streaming stores), or, for a
// heavy-row chunk, adds it with one 16-byte vector reduction per lane.
// A values and column indices are streamed (evict-first); B keeps the default caching so hot
// columns stay in L1/L2.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <vector>

#include "common.cuh"
#include "plan_rows.hpp"

namespace vcsrmc {
namespace dev {
namespace {

constexpr int kWarpsPerBlock = 8;
constexpr unsigned kFull = 0xffffffffu;

__device__ __forceinline__ float to_f(float v) { return v; }
__device__ __forceinline__ float to_f(__half v) { return __half2float(v); }

template <typename T>
__device__ __forceinline__ T ld_stream(const T* p) {
    return __ldcs(p);
}
template <>
__device__ __forceinline__ __half ld_stream<__half>(const __half* p) {
    const unsigned short u = __ldcs(reinterpret_cast<const unsigned short*>(p));
    return __ushort_as_half(u);
}

// Four consecutive B elements (nv of them valid) as fp32.
template <bool kVec>
__device__ __forceinline__ float4 load_b4(const __half* p, int nv) {
    if (kVec && nv == 4) {
        const uint2 raw = __ldg(reinterpret_cast<const uint2*>(p));
        const float2 lo = __half22float2(*reinterpret_cast<const __half2*>(&raw.x));
        const float2 hi = __half22float2(*reinterpret_cast<const __half2*>(&raw.y));
        return make_float4(lo.x, lo.y, hi.x, hi.y);
    }
    float4 r = make_float4(0.f, 0.f, 0.f, 0.f);
    if (nv > 0) r.x = __half2float(p[0]);
    if (nv > 1) r.y = __half2float(p[1]);
    if (nv > 2) r.z = __half2float(p[2]);
    if (nv > 3) r.w = __half2float(p[3]);
    return r;
}
template <bool kVec>
__device__ __forceinline__ float4 load_b4(const float* p, int nv) {
    if (kVec && nv == 4) return __ldg(reinterpret_cast<const float4*>(p));
    float4 r = make_float4(0.f, 0.f, 0.f, 0.f);
    if (nv > 0) r.x = __ldg(p);
    if (nv > 1) r.y = __ldg(p + 1);
    if (nv > 2) r.z = __ldg(p + 2);
    if (nv > 3) r.w = __ldg(p + 3);
    return r;
}

// acc += A[row, entries p0..p1) * B[:, c0..c0+3]
template <bool kVec, typename VT, typename BT>
__device__ __forceinline__ void accumulate_range(float4& acc, int p0, int p1, const int* __restrict__ cols,
                                                 const VT* __restrict__ vals, const BT* __restrict__ B, int64_t ldb,
                                                 int c0, int nv, int lane) {
    constexpr int U = 8;
    for (int p = p0; p < p1; p += 32) {
        const int n = min(32, p1 - p);
        int mc = 0;
        float mv = 0.f;
        if (lane < n) {
            mc = ld_stream(cols + p + lane);
            mv = to_f(ld_stream(vals + p + lane));
        }
        for (int j = 0; j < n; j += U) {
            float4 b[U];
            float v[U];
#pragma unroll
            for (int k = 0; k < U; ++k) {
                const int c = __shfl_sync(kFull, mc, (j + k) & 31);
                v[k] = __shfl_sync(kFull, mv, (j + k) & 31);
                if (j + k < n) {
                    b[k] = load_b4<kVec>(B + int64_t(c) * ldb + c0, nv);
                } else {
                    b[k] = make_float4(0.f, 0.f, 0.f, 0.f);
                    v[k] = 0.f;
                }
            }
#pragma unroll
            for (int k = 0; k < U; ++k) {
                acc.x = fmaf(v[k], b[k].x, acc.x);
                acc.y = fmaf(v[k], b[k].y, acc.y);
                acc.z = fmaf(v[k], b[k].z, acc.z);
                acc.w = fmaf(v[k], b[k].w, acc.w);
            }
        }
    }
}

template <bool kVec, bool kAccumulate, typename VT, typename BT>
__global__ void __launch_bounds__(kWarpsPerBlock * 32)
    vcsr_rows_kernel(const int4* __restrict__ units, int64_t n_units, const int* __restrict__ rp,
                     const int* __restrict__ cols, const VT* __restrict__ vals, const BT* __restrict__ B,
                     int64_t ldb, int O, float* __restrict__ C, int64_t ldc, float scale) {
    const int lane = threadIdx.x & 31;
    const int64_t w = int64_t(blockIdx.x) * kWarpsPerBlock + (threadIdx.x >> 5);
    if (w >= n_units) return;
    const int4 u = units[w];
    const int c0 = blockIdx.y * 128 + 4 * lane;
    const int nv = max(0, min(4, O - c0));
    const bool partial = (u.y & 0x80000000) != 0;
    const int r_end = u.y & 0x7fffffff;
    if (partial) {
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        accumulate_range<kVec>(acc, u.z, u.w, cols, vals, B, ldb, c0, nv, lane);
        float* dst = C + int64_t(u.x) * ldc + c0;
        acc.x *= scale; acc.y *= scale; acc.z *= scale; acc.w *= scale;
        if (kVec && nv == 4) {
            atomicAdd(reinterpret_cast<float4*>(dst), acc);
        } else {
            if (nv > 0) atomicAdd(dst, acc.x);
            if (nv > 1) atomicAdd(dst + 1, acc.y);
            if (nv > 2) atomicAdd(dst + 2, acc.z);
            if (nv > 3) atomicAdd(dst + 3, acc.w);
        }
        return;
    }
    for (int r = u.x; r < r_end; ++r) {
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        accumulate_range<kVec>(acc, rp[r], rp[r + 1], cols, vals, B, ldb, c0, nv, lane);
        acc.x *= scale; acc.y *= scale; acc.z *= scale; acc.w *= scale;
        float* dst = C + int64_t(r) * ldc + c0;
        if (kVec && nv == 4) {
            if (kAccumulate) {
                const float4 old = *reinterpret_cast<const float4*>(dst);
                acc.x += old.x; acc.y += old.y; acc.z += old.z; acc.w += old.w;
            }
            __stcs(reinterpret_cast<float4*>(dst), acc);
        } else {
            const float a[4] = {acc.x, acc.y, acc.z, acc.w};
            for (int i = 0; i < nv; ++i) dst[i] = kAccumulate ? dst[i] + a[i] : a[i];
        }
    }
}

// Zeroes C's heavy rows (the ones built from several reduced chunks) before an overwrite.
__global__ void zero_rows_kernel(const int* __restrict__ rows, int n_rows, int O, float* __restrict__ C, int64_t ldc) {
    const int i = blockIdx.x;
    if (i >= n_rows) return;
    float* dst = C + int64_t(rows[i]) * ldc;
    for (int c = threadIdx.x; c < O; c += blockDim.x) dst[c] = 0.f;
}

template <bool kVec, bool kAcc, typename VT, typename BT>
cudaError_t launch_rows_t(const RowPlanView& P, const BT* B, int64_t ldb, int O, float* C, int64_t ldc,
                          cudaStream_t st) {
    const int64_t blocks = (P.n_units + kWarpsPerBlock - 1) / kWarpsPerBlock;
    if (blocks > 0x7fffffffLL) return cudaErrorInvalidValue;
    const dim3 grid(unsigned(blocks), unsigned((O + 127) / 128));
    vcsr_rows_kernel<kVec, kAcc, VT, BT><<<grid, kWarpsPerBlock * 32, 0, st>>>(
        P.units, P.n_units, P.rp, P.cols, static_cast<const VT*>(P.vals), B, ldb, O, C, ldc, P.scale);
    return cudaGetLastError();
}

template <typename VT, typename BT>
cudaError_t launch_rows_b(const RowPlanView& P, const BT* B, int64_t ldb, int O, float* C, int64_t ldc,
                          bool accumulate, cudaStream_t st) {
    const bool vec = (ldb % 4 == 0) && (ldc % 4 == 0) && (reinterpret_cast<uintptr_t>(B) % 16 == 0) &&
                     (reinterpret_cast<uintptr_t>(C) % 16 == 0);
    if (vec) {
        return accumulate ? launch_rows_t<true, true, VT, BT>(P, B, ldb, O, C, ldc, st)
                          : launch_rows_t<true, false, VT, BT>(P, B, ldb, O, C, ldc, st);
    }
    return accumulate ? launch_rows_t<false, true, VT, BT>(P, B, ldb, O, C, ldc, st)
                      : launch_rows_t<false, false, VT, BT>(P, B, ldb, O, C, ldc, st);
}

}  // namespace

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
RowViewHost build_row_view(const VCSRMC& v) {
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
    // work units: heavy-row chunks first, then runs of light rows
    for (int r = 0; r < M; ++r) {
        const int len = h.rp[r + 1] - h.rp[r];
        if (len > kUnitNnz) {
            h.split_rows.push_back(r);
            for (int p = h.rp[r]; p < h.rp[r + 1]; p += kUnitNnz)
                h.units.push_back({r, int((unsigned(r + 1)) | 0x80000000u), p, std::min(h.rp[r + 1], p + kUnitNnz)});
        }
    }
    int r = 0;
    while (r < M) {
        if (h.rp[r + 1] - h.rp[r] > kUnitNnz) { ++r; continue; }
        const int rb = r;
        int n = 0;
        while (r < M && r - rb < kUnitRows) {
            const int len = h.rp[r + 1] - h.rp[r];
            if (len > kUnitNnz || (r > rb && n + len > kUnitNnz)) break;
            n += len;
            ++r;
        }
        h.units.push_back({rb, r, h.rp[rb], h.rp[r]});
    }
    return h;
}

}  // namespace dev
}  // namespace vcsrmc
