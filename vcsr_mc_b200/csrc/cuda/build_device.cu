// GPU-side VCSR-MC construction: the format of a CSR that is already in device memory, built
// with sorts and scans on the device instead of the host loops of csr_to_vcsr_mc
// (src/vcsr_mc.cu:25-123), and the ROWS plan's row view next to it.
//
// Steps (rows must list strictly ascending columns, as coo_to_csr leaves them):
//   1. pairs: an entry starts a (segment, row) pair when it is the first of its row or its segment
//      (column / segw) differs from the previous entry's; an exclusive scan numbers the pairs in
//      row-major order, and a pair's entry count is the distance to the next pair's first entry;
//   2. row order: a stable radix sort of the pairs by (segment, 127 - count). Pairs enter in
//      ascending row order, so rows with equal counts stay in ascending row order. (The reference
//      orders such rows by its hash map's iteration; group_rows, lcol and val can therefore differ
//      from the host builder's by a permutation inside runs of equal-count rows. Every other array
//      is identical, and all arrays equal the oracle's canonical build.)
//   3. groups: the sorted pairs of a segment are cut into groups of 16 (per-segment pair counts
//      and an exclusive scan give each group's index); depth = the group's first (largest)
//      count; group_ptr = exclusive scan of 16 * depth; slots are filled depth-major, padding
//      (-1, 0);
//   4. items: runs of at most chunk = max(1, min(32, G / 4096)) groups of one segment, then a
//      stable radix sort by slot count, heaviest first.
// The row view needs no reordering: a CSR row with ascending columns already lists its entries
// in the format's order (ascending segment, then local column). Its work units come from row_ptr
// alone, packed on the host by the same rule as the host-built view (pack_units).
#include <cub/cub.cuh>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <climits>
#include <cstring>
#include <string>
#include <vector>

#include "../capi_internal.hpp"
#include "build_device.hpp"
#include "plan_rows.hpp"

namespace vcsrmc {
namespace dev {
namespace {

constexpr int kBundle = 16;

void check(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return;
    // A failed call also leaves its error as the thread's last runtime error, which the next
    // launch check (cudaGetLastError) would report again; clear it (a sticky error stays).
    cudaGetLastError();
    const int s = e == cudaErrorMemoryAllocation ? VCSRMC_OOM : VCSRMC_CUDA_ERR;
    throw StatusError(s, std::string(what) + ": " + cudaGetErrorString(e));
}

// Device buffer freed on scope exit unless released.
template <class T>
struct Buf {
    T* p = nullptr;
    explicit Buf(size_t n) { check(cudaMalloc(&p, sizeof(T) * std::max<size_t>(n, 1)), "cudaMalloc"); }
    ~Buf() { cudaFree(p); }
    Buf(const Buf&) = delete;
    Buf& operator=(const Buf&) = delete;
    T* release() {
        T* q = p;
        p = nullptr;
        return q;
    }
};

template <class T>
T read_one(const T* d, cudaStream_t st) {
    T h{};
    check(cudaMemcpyAsync(&h, d, sizeof(T), cudaMemcpyDeviceToHost, st), "cudaMemcpyAsync");
    check(cudaStreamSynchronize(st), "cudaStreamSynchronize");
    return h;
}

unsigned blocks_for(int64_t n, int threads = 256) {
    return unsigned(std::max<int64_t>(1, std::min<int64_t>((n + threads - 1) / threads, 148LL * 64)));
}

// Row of entry p: the last r with row_ptr[r] <= p.
__device__ __forceinline__ int row_of(const int* __restrict__ rp, int M, int64_t p) {
    int lo = 0, hi = M - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (rp[mid] <= p) lo = mid;
        else hi = mid - 1;
    }
    return lo;
}

__global__ void abs_max_kernel(const float* __restrict__ v, int64_t n, unsigned* out) {
    float m = 0.f;
    for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x)
        m = fmaxf(m, fabsf(v[i]));
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31) == 0) atomicMax(out, __float_as_uint(m));  // non-negative floats order as their bits
}

// row_ptr[0] = 0, non-decreasing, row_ptr[M] = nnz.
__global__ void row_ptr_check_kernel(const int* __restrict__ rp, int M, int64_t nnz, int* bad) {
    for (int64_t r = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; r <= M; r += int64_t(gridDim.x) * blockDim.x) {
        const int v = rp[r];
        if ((r == 0 && v != 0) || (r == M && int64_t(v) != nnz) || (r < M && rp[r + 1] < v)) atomicOr(bad, 1);
    }
}

__global__ void rows_sorted_kernel(const int* __restrict__ rp, const int* __restrict__ col, int M, int N, int64_t nnz,
                                   int* bad) {
    for (int64_t p = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; p < nnz; p += int64_t(gridDim.x) * blockDim.x) {
        const int c = col[p];
        bool ok = c >= 0 && c < N;
        if (ok && p > 0) {
            const int r = row_of(rp, M, p);
            if (p > rp[r] && col[p - 1] >= c) ok = false;
        }
        if (!ok) atomicOr(bad, 1);
    }
}

// 1 where an entry starts a (segment, row) pair.
__global__ void pair_start_kernel(const int* __restrict__ rp, const int* __restrict__ col, int M, int64_t nnz,
                                  int segw, int* __restrict__ start) {
    for (int64_t p = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; p < nnz; p += int64_t(gridDim.x) * blockDim.x) {
        int s = 1;
        if (p > 0) {
            const int r = row_of(rp, M, p);
            if (p > rp[r] && col[p - 1] / segw == col[p] / segw) s = 0;
        }
        start[p] = s;
    }
}

__global__ void pair_first_kernel(const int* __restrict__ start, const int* __restrict__ pid, int64_t nnz,
                                  int* __restrict__ first) {
    for (int64_t p = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; p < nnz; p += int64_t(gridDim.x) * blockDim.x)
        if (start[p]) first[pid[p]] = int(p);
}

// Sort key (segment, 127 - count), the pair's row, and the per-segment pair histogram.
__global__ void pair_key_kernel(const int* __restrict__ rp, const int* __restrict__ col, const int* __restrict__ first,
                                int M, int64_t nnz, int64_t npairs, int segw, uint64_t* __restrict__ key,
                                int* __restrict__ idx, int* __restrict__ prow, int* __restrict__ seg_pairs) {
    for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < npairs;
         i += int64_t(gridDim.x) * blockDim.x) {
        const int f = first[i];
        const int64_t next = i + 1 < npairs ? int64_t(first[i + 1]) : nnz;
        const int count = int(next - f);
        const int sid = col[f] / segw;
        key[i] = (uint64_t(uint32_t(sid)) << 7) | uint64_t(127 - count);
        idx[i] = int(i);
        prow[i] = row_of(rp, M, f);
        atomicAdd(seg_pairs + sid, 1);
    }
}

__global__ void seg_groups_kernel(const int* __restrict__ seg_pairs, int S, int* __restrict__ seg_groups) {
    for (int s = blockIdx.x * blockDim.x + threadIdx.x; s < S; s += gridDim.x * blockDim.x)
        seg_groups[s] = (seg_pairs[s] + kBundle - 1) / kBundle;
}

// Group rows, depth and segment base from the sorted pairs.
__global__ void group_fill_kernel(const uint64_t* __restrict__ skey, const int* __restrict__ sidx,
                                  const int* __restrict__ prow, const int* __restrict__ seg_pair_off,
                                  const int* __restrict__ seg_group_off, int64_t npairs, int segw,
                                  int* __restrict__ grows, int* __restrict__ depth, int* __restrict__ seg_base) {
    for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < npairs;
         i += int64_t(gridDim.x) * blockDim.x) {
        const uint64_t k = skey[i];
        const int sid = int(k >> 7), count = 127 - int(k & 127u);
        const int rank = int(i) - seg_pair_off[sid];
        const int g = seg_group_off[sid] + rank / kBundle, lane = rank % kBundle;
        grows[int64_t(g) * kBundle + lane] = prow[sidx[i]];
        if (lane == 0) {
            depth[g] = count;
            seg_base[g] = sid * segw;
        }
    }
}

__global__ void group_slots_kernel(const int* __restrict__ depth, int64_t G, int64_t* __restrict__ slots) {
    for (int64_t g = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; g < G; g += int64_t(gridDim.x) * blockDim.x)
        slots[g] = int64_t(depth[g]) * kBundle;
}

__global__ void gmeta_kernel(const int64_t* __restrict__ gptr, const int* __restrict__ depth,
                             const int* __restrict__ seg_base, int64_t G, int4* __restrict__ gmeta) {
    for (int64_t g = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; g < G; g += int64_t(gridDim.x) * blockDim.x)
        gmeta[g] = make_int4(int(gptr[g]), depth[g], seg_base[g], 0);
}

template <bool kF32>
__global__ void slot_fill_kernel(const uint64_t* __restrict__ skey, const int* __restrict__ sidx,
                                 const int* __restrict__ first, const int* __restrict__ seg_pair_off,
                                 const int* __restrict__ seg_group_off, const int4* __restrict__ gmeta,
                                 const int* __restrict__ col, const float* __restrict__ val, int64_t npairs, int segw,
                                 float inv_scale, int8_t* __restrict__ lcol, void* __restrict__ sval) {
    for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < npairs;
         i += int64_t(gridDim.x) * blockDim.x) {
        const uint64_t k = skey[i];
        const int sid = int(k >> 7), count = 127 - int(k & 127u);
        const int rank = int(i) - seg_pair_off[sid];
        const int g = seg_group_off[sid] + rank / kBundle, lane = rank % kBundle;
        const int f = first[sidx[i]];
        const int base = gmeta[g].x;
        for (int d = 0; d < count; ++d) {
            const int64_t slot = int64_t(base) + int64_t(d) * kBundle + lane;
            lcol[slot] = int8_t(col[f + d] % segw);
            const float v = val[f + d] * inv_scale;
            if constexpr (kF32) static_cast<float*>(sval)[slot] = v;
            else static_cast<__half*>(sval)[slot] = __float2half_rn(v);
        }
    }
}

__global__ void seg_items_kernel(const int* __restrict__ seg_groups, int S, int chunk, int* __restrict__ seg_items) {
    for (int s = blockIdx.x * blockDim.x + threadIdx.x; s < S; s += gridDim.x * blockDim.x)
        seg_items[s] = (seg_groups[s] + chunk - 1) / chunk;
}

// Items in group order (segment by segment) with their slot counts as sort keys (heaviest first).
__global__ void item_fill_kernel(const int* __restrict__ seg_groups, const int* __restrict__ seg_group_off,
                                 const int* __restrict__ seg_item_off, const int64_t* __restrict__ gptr, int S,
                                 int chunk, uint32_t* __restrict__ key, int* __restrict__ idx, int2* __restrict__ items) {
    for (int s = blockIdx.x * blockDim.x + threadIdx.x; s < S; s += gridDim.x * blockDim.x) {
        const int g0 = seg_group_off[s], g1 = g0 + seg_groups[s];
        int k = seg_item_off[s];
        for (int gb = g0; gb < g1; gb += chunk, ++k) {
            const int ge = min(gb + chunk, g1);
            const int64_t work = gptr[ge] - gptr[gb];
            key[k] = 0xffffffffu - uint32_t(work);
            idx[k] = k;
            items[k] = make_int2(gb, ge);
        }
    }
}

__global__ void item_gather_kernel(const int* __restrict__ order, const int2* __restrict__ items, int64_t n,
                                   int2* __restrict__ out) {
    for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x)
        out[i] = items[order[i]];
}

template <bool kF32>
__global__ void scale_values_kernel(const float* __restrict__ val, int64_t n, float inv_scale, void* __restrict__ out) {
    for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
        const float v = val[i] * inv_scale;
        if constexpr (kF32) static_cast<float*>(out)[i] = v;
        else static_cast<__half*>(out)[i] = __float2half_rn(v);
    }
}

// Invariants the SpMM kernels rely on.
__global__ void validate_segment_kernel(const int4* __restrict__ gmeta, const int* __restrict__ grows,
                                        const int8_t* __restrict__ lcol, const int2* __restrict__ items, int64_t G,
                                        int64_t S, int64_t I, int M, int N, int segw, int* bad) {
    const int64_t stride = int64_t(gridDim.x) * blockDim.x;
    const int64_t t0 = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    for (int64_t g = t0; g < G; g += stride) {
        const int4 m = gmeta[g];
        const int64_t next = g + 1 < G ? int64_t(gmeta[g + 1].x) : S;
        if (m.x < 0 || m.y < 0 || m.y > 64 || next - m.x != int64_t(m.y) * kBundle || m.z < 0 || m.z % segw != 0 ||
            m.z >= N)
            atomicOr(bad, 1);
        for (int l = 0; l < kBundle; ++l) {
            const int r = grows[g * kBundle + l];
            if (r < -1 || r >= M) atomicOr(bad, 2);
        }
        for (int64_t s = m.x; s < next && s < S; ++s) {
            const int c = lcol[s];
            if (c < -1 || c >= segw || (c >= 0 && m.z + c >= N)) atomicOr(bad, 4);
        }
    }
    for (int64_t i = t0; i < I; i += stride) {
        const int2 it = items[i];
        if (it.x < 0 || it.y <= it.x || it.y > G || gmeta[it.x].z != gmeta[it.y - 1].z) atomicOr(bad, 8);
    }
}

__global__ void validate_rows_kernel(const int* __restrict__ rp, const int* __restrict__ cols,
                                     const int4* __restrict__ units, int64_t U, int M, int N, int64_t nnz, int* bad) {
    const int64_t stride = int64_t(gridDim.x) * blockDim.x;
    const int64_t t0 = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    for (int64_t r = t0; r < M; r += stride)
        if (rp[r] > rp[r + 1] || rp[r] < 0 || rp[r + 1] > nnz) atomicOr(bad, 16);
    for (int64_t p = t0; p < nnz; p += stride)
        if (cols[p] < 0 || cols[p] >= N) atomicOr(bad, 32);
    for (int64_t i = t0; i < U; i += stride) {
        const int4 u = units[i];
        const bool heavy = (u.y & 0x80000000) != 0;
        const int rend = heavy ? u.x + 1 : u.y;
        if (u.x < 0 || rend > M || rend <= u.x || (!heavy && rend - u.x > 16) || u.z < 0 || u.w > nnz || u.w < u.z)
            atomicOr(bad, 64);
    }
}

template <class T>
void exclusive_scan(const T* in, T* out, int64_t n, cudaStream_t st) {
    if (n <= 0) return;
    size_t tmp = 0;
    check(cub::DeviceScan::ExclusiveSum(nullptr, tmp, in, out, n, st), "cub scan");
    Buf<uint8_t> t(tmp);
    check(cub::DeviceScan::ExclusiveSum(t.p, tmp, in, out, n, st), "cub scan");
}

}  // namespace

float device_abs_max(const float* val, int64_t nnz, cudaStream_t st) {
    if (nnz <= 0) return 0.f;
    Buf<unsigned> m(1);
    check(cudaMemsetAsync(m.p, 0, sizeof(unsigned), st), "cudaMemsetAsync");
    abs_max_kernel<<<blocks_for(nnz), 256, 0, st>>>(val, nnz, m.p);
    check(cudaGetLastError(), "abs_max_kernel");
    const unsigned bits = read_one(m.p, st);
    float f;
    std::memcpy(&f, &bits, sizeof f);
    return f;
}

// Scratch of device_abs_max_noalloc: one word per device for the whole library, so that call
// allocates nothing (its callers serialise on it).
static __device__ __align__(256) unsigned g_abs_max_scratch[1];

float device_abs_max_noalloc(const float* val, int64_t nnz, cudaStream_t st) {
    if (nnz <= 0) return 0.f;
    void* scratch = nullptr;
    check(cudaGetSymbolAddress(&scratch, g_abs_max_scratch), "cudaGetSymbolAddress");
    check(cudaMemsetAsync(scratch, 0, sizeof(unsigned), st), "cudaMemsetAsync");
    abs_max_kernel<<<blocks_for(nnz), 256, 0, st>>>(val, nnz, static_cast<unsigned*>(scratch));
    check(cudaGetLastError(), "abs_max_kernel");
    const unsigned bits = read_one(static_cast<const unsigned*>(scratch), st);
    float f;
    std::memcpy(&f, &bits, sizeof f);
    return f;
}

bool device_csr_rows_sorted(const int* row_ptr, const int* col, int M, int N, int64_t nnz, cudaStream_t st) {
    Buf<int> bad(1);
    check(cudaMemsetAsync(bad.p, 0, sizeof(int), st), "cudaMemsetAsync");
    row_ptr_check_kernel<<<blocks_for(int64_t(M) + 1), 256, 0, st>>>(row_ptr, M, nnz, bad.p);
    check(cudaGetLastError(), "row_ptr_check_kernel");
    if (read_one(bad.p, st) != 0) return false;  // entries are located through row_ptr below
    if (nnz > 0) {
        rows_sorted_kernel<<<blocks_for(nnz), 256, 0, st>>>(row_ptr, col, M, N, nnz, bad.p);
        check(cudaGetLastError(), "rows_sorted_kernel");
    }
    return read_one(bad.p, st) == 0;
}

SegmentLayout build_segment_layout(const int* row_ptr, const int* col, const float* val, int M, int N, int64_t nnz,
                                   int segw, bool fp32, float scale, cudaStream_t st) {
    SegmentLayout L;
    const int S = (N + segw - 1) / segw;
    L.num_segments = S;
    if (nnz == 0 || M == 0) {
        L.items = Buf<int2>(1).release();
        L.gmeta = Buf<int4>(1).release();
        L.grows = Buf<int>(1).release();
        L.lcol = Buf<int8_t>(1).release();
        L.val = fp32 ? static_cast<void*>(Buf<float>(1).release()) : static_cast<void*>(Buf<__half>(1).release());
        return L;
    }
    // 1. pairs
    Buf<int> start(nnz), pid(nnz);
    pair_start_kernel<<<blocks_for(nnz), 256, 0, st>>>(row_ptr, col, M, nnz, segw, start.p);
    check(cudaGetLastError(), "pair_start_kernel");
    exclusive_scan(start.p, pid.p, nnz, st);
    const int64_t npairs = int64_t(read_one(pid.p + nnz - 1, st)) + read_one(start.p + nnz - 1, st);
    Buf<int> first(npairs);
    pair_first_kernel<<<blocks_for(nnz), 256, 0, st>>>(start.p, pid.p, nnz, first.p);
    check(cudaGetLastError(), "pair_first_kernel");
    // 2. row order inside segments (stable: ties keep ascending row order)
    Buf<uint64_t> key(npairs), skey(npairs);
    Buf<int> idx(npairs), sidx(npairs), prow(npairs);
    Buf<int> seg_pairs(size_t(S) + 1);
    check(cudaMemsetAsync(seg_pairs.p, 0, sizeof(int) * (size_t(S) + 1), st), "cudaMemsetAsync");
    pair_key_kernel<<<blocks_for(npairs), 256, 0, st>>>(row_ptr, col, first.p, M, nnz, npairs, segw, key.p, idx.p,
                                                         prow.p, seg_pairs.p);
    check(cudaGetLastError(), "pair_key_kernel");
    int end_bit = 7;
    while (end_bit < 64 && (uint64_t(S) << 7) >> end_bit) ++end_bit;
    {
        size_t tmp = 0;
        check(cub::DeviceRadixSort::SortPairs(nullptr, tmp, key.p, skey.p, idx.p, sidx.p, npairs, 0, end_bit, st),
              "cub sort");
        Buf<uint8_t> t(tmp);
        check(cub::DeviceRadixSort::SortPairs(t.p, tmp, key.p, skey.p, idx.p, sidx.p, npairs, 0, end_bit, st),
              "cub sort");
    }
    // 3. groups
    Buf<int> seg_pair_off(size_t(S) + 1), seg_groups(size_t(S) + 1), seg_group_off(size_t(S) + 1);
    exclusive_scan(seg_pairs.p, seg_pair_off.p, int64_t(S) + 1, st);
    check(cudaMemsetAsync(seg_groups.p + S, 0, sizeof(int), st), "cudaMemsetAsync");
    seg_groups_kernel<<<blocks_for(S), 256, 0, st>>>(seg_pairs.p, S, seg_groups.p);
    check(cudaGetLastError(), "seg_groups_kernel");
    exclusive_scan(seg_groups.p, seg_group_off.p, int64_t(S) + 1, st);
    const int64_t G = read_one(seg_group_off.p + S, st);
    if (G * kBundle > INT_MAX) throw StatusError(VCSRMC_INVALID_ARG, "VCSR group count exceeds the format's 32-bit offsets");
    Buf<int> grows(size_t(G) * kBundle), depth(G), seg_base(G);
    check(cudaMemsetAsync(grows.p, 0xff, sizeof(int) * size_t(G) * kBundle, st), "cudaMemsetAsync");
    group_fill_kernel<<<blocks_for(npairs), 256, 0, st>>>(skey.p, sidx.p, prow.p, seg_pair_off.p, seg_group_off.p,
                                                           npairs, segw, grows.p, depth.p, seg_base.p);
    check(cudaGetLastError(), "group_fill_kernel");
    Buf<int64_t> gslots(size_t(G) + 1), gptr(size_t(G) + 1);
    check(cudaMemsetAsync(gslots.p + G, 0, sizeof(int64_t), st), "cudaMemsetAsync");
    group_slots_kernel<<<blocks_for(G), 256, 0, st>>>(depth.p, G, gslots.p);
    check(cudaGetLastError(), "group_slots_kernel");
    exclusive_scan(gslots.p, gptr.p, G + 1, st);
    const int64_t total_slots = read_one(gptr.p + G, st);
    if (total_slots > INT_MAX) throw StatusError(VCSRMC_INVALID_ARG, "VCSR slot count exceeds the format's 32-bit offsets");
    Buf<int4> gmeta(G);
    gmeta_kernel<<<blocks_for(G), 256, 0, st>>>(gptr.p, depth.p, seg_base.p, G, gmeta.p);
    check(cudaGetLastError(), "gmeta_kernel");
    Buf<int8_t> lcol(total_slots);
    check(cudaMemsetAsync(lcol.p, 0xff, size_t(total_slots), st), "cudaMemsetAsync");
    const size_t vbytes = size_t(total_slots) * (fp32 ? 4 : 2);
    Buf<uint8_t> sval(vbytes);
    check(cudaMemsetAsync(sval.p, 0, vbytes, st), "cudaMemsetAsync");
    const float inv_scale = 1.0f / scale;
    if (fp32)
        slot_fill_kernel<true><<<blocks_for(npairs), 256, 0, st>>>(skey.p, sidx.p, first.p, seg_pair_off.p,
                                                                   seg_group_off.p, gmeta.p, col, val, npairs, segw,
                                                                   inv_scale, lcol.p, sval.p);
    else
        slot_fill_kernel<false><<<blocks_for(npairs), 256, 0, st>>>(skey.p, sidx.p, first.p, seg_pair_off.p,
                                                                    seg_group_off.p, gmeta.p, col, val, npairs, segw,
                                                                    inv_scale, lcol.p, sval.p);
    check(cudaGetLastError(), "slot_fill_kernel");
    // 4. items, heaviest first (stable)
    const int chunk = std::max(1, std::min(32, int(G) / 4096));
    Buf<int> seg_items(size_t(S) + 1), seg_item_off(size_t(S) + 1);
    check(cudaMemsetAsync(seg_items.p + S, 0, sizeof(int), st), "cudaMemsetAsync");
    seg_items_kernel<<<blocks_for(S), 256, 0, st>>>(seg_groups.p, S, chunk, seg_items.p);
    check(cudaGetLastError(), "seg_items_kernel");
    exclusive_scan(seg_items.p, seg_item_off.p, int64_t(S) + 1, st);
    const int64_t I = read_one(seg_item_off.p + S, st);
    Buf<uint32_t> ikey(I), sikey(I);
    Buf<int> iidx(I), siidx(I);
    Buf<int2> items(I), sitems(I);
    item_fill_kernel<<<blocks_for(S), 256, 0, st>>>(seg_groups.p, seg_group_off.p, seg_item_off.p, gptr.p, S, chunk,
                                                     ikey.p, iidx.p, items.p);
    check(cudaGetLastError(), "item_fill_kernel");
    {
        size_t tmp = 0;
        check(cub::DeviceRadixSort::SortPairs(nullptr, tmp, ikey.p, sikey.p, iidx.p, siidx.p, I, 0, 32, st), "cub sort");
        Buf<uint8_t> t(tmp);
        check(cub::DeviceRadixSort::SortPairs(t.p, tmp, ikey.p, sikey.p, iidx.p, siidx.p, I, 0, 32, st), "cub sort");
    }
    item_gather_kernel<<<blocks_for(I), 256, 0, st>>>(siidx.p, items.p, I, sitems.p);
    check(cudaGetLastError(), "item_gather_kernel");
    check(cudaStreamSynchronize(st), "cudaStreamSynchronize");
    L.items = sitems.release();
    L.gmeta = gmeta.release();
    L.grows = grows.release();
    L.lcol = lcol.release();
    L.val = sval.release();
    L.n_groups = G;
    L.n_slots = total_slots;
    L.n_items = I;
    return L;
}

RowsLayout build_rows_layout(const int* row_ptr, const int* col, const float* val, int M, int64_t nnz, bool fp32,
                             float scale, int unit_nnz, cudaStream_t st) {
    RowsLayout R;
    Buf<int> rp(size_t(M) + 1), cols(nnz);
    check(cudaMemcpyAsync(rp.p, row_ptr, sizeof(int) * (size_t(M) + 1), cudaMemcpyDeviceToDevice, st), "cudaMemcpyAsync");
    if (nnz) check(cudaMemcpyAsync(cols.p, col, sizeof(int) * size_t(nnz), cudaMemcpyDeviceToDevice, st), "cudaMemcpyAsync");
    Buf<uint8_t> vals(size_t(nnz) * (fp32 ? 4 : 2));
    if (nnz) {
        if (fp32) scale_values_kernel<true><<<blocks_for(nnz), 256, 0, st>>>(val, nnz, 1.0f / scale, vals.p);
        else scale_values_kernel<false><<<blocks_for(nnz), 256, 0, st>>>(val, nnz, 1.0f / scale, vals.p);
        check(cudaGetLastError(), "scale_values_kernel");
    }
    // Work units are packed on the host from row_ptr alone (M + 1 integers; the entries stay on
    // the device) with the same greedy rule as the host-built row view.
    std::vector<int> hrp(size_t(M) + 1);
    check(cudaMemcpyAsync(hrp.data(), row_ptr, sizeof(int) * (size_t(M) + 1), cudaMemcpyDeviceToHost, st),
          "cudaMemcpyAsync");
    check(cudaStreamSynchronize(st), "cudaStreamSynchronize");
    std::vector<RowViewHost::Unit> hunits;
    std::vector<int> hsplit;
    pack_units(hrp.data(), M, unit_nnz, hunits, hsplit);
    static_assert(sizeof(RowViewHost::Unit) == sizeof(int4), "unit layout");
    Buf<int4> units(hunits.size());
    Buf<int> split(hsplit.size());
    if (!hunits.empty())
        check(cudaMemcpyAsync(units.p, hunits.data(), sizeof(int4) * hunits.size(), cudaMemcpyHostToDevice, st),
              "cudaMemcpyAsync");
    if (!hsplit.empty())
        check(cudaMemcpyAsync(split.p, hsplit.data(), sizeof(int) * hsplit.size(), cudaMemcpyHostToDevice, st),
              "cudaMemcpyAsync");
    const int64_t n_units = int64_t(hunits.size()), n_split = int64_t(hsplit.size());
    check(cudaStreamSynchronize(st), "cudaStreamSynchronize");
    R.rp = rp.release();
    R.cols = cols.release();
    R.vals = vals.release();
    R.units = units.release();
    R.n_units = n_units;
    R.split_rows = split.release();
    R.n_split_rows = int(n_split);
    return R;
}

bool device_validate(const SegmentLayout* seg, const RowsLayout* rows, int M, int N, int segw, cudaStream_t st) {
    Buf<int> bad(1);
    check(cudaMemsetAsync(bad.p, 0, sizeof(int), st), "cudaMemsetAsync");
    if (seg && (seg->n_groups > 0 || seg->n_items > 0)) {
        const int64_t n = std::max(seg->n_groups, seg->n_items);
        validate_segment_kernel<<<blocks_for(n), 256, 0, st>>>(seg->gmeta, seg->grows, seg->lcol, seg->items,
                                                               seg->n_groups, seg->n_slots, seg->n_items, M, N, segw,
                                                               bad.p);
        check(cudaGetLastError(), "validate_segment_kernel");
    }
    if (rows) {
        const int64_t nnz = M > 0 ? read_one(rows->rp + M, st) : 0;
        const int64_t n = std::max<int64_t>(std::max<int64_t>(M, nnz), rows->n_units);
        if (n > 0) {
            validate_rows_kernel<<<blocks_for(n), 256, 0, st>>>(rows->rp, rows->cols, rows->units, rows->n_units, M, N,
                                                                nnz, bad.p);
            check(cudaGetLastError(), "validate_rows_kernel");
        }
    }
    return read_one(bad.p, st) == 0;
}

}  // namespace dev
}  // namespace vcsrmc
