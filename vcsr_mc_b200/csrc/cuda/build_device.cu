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
// alone, packed on the host by the same rule as the host-built view (pack_units). The BAND view
// (build_band_layout) sorts each band's entries by column and cuts its tiles with one warp per band.
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

// SMs of the calling thread's current device (the builder's kernels run there).
int current_sm_count() {
    int dev = 0, sms = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) {
        cudaGetLastError();
        return 1;
    }
    return sms;
}

// Grid-stride launches: enough blocks to fill every SM 64 times over (8 resident 256-thread
// blocks per SM, eight waves), fewer for small inputs.
unsigned blocks_for(int64_t n, int threads = 256) {
    const int64_t cap = int64_t(current_sm_count()) * 64;
    return unsigned(std::max<int64_t>(1, std::min<int64_t>((n + threads - 1) / threads, cap)));
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

// ---- BAND view ----------------------------------------------------------------------------------

__global__ void gather_int_kernel(const int* __restrict__ src, const int* __restrict__ idx, int n, int* __restrict__ out) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) out[i] = src[idx[i]];
}

// Band b's entries are [row_ptr[b * H], row_ptr[min(M, (b + 1) * H)]).
__global__ void band_offsets_kernel(const int* __restrict__ rp, int M, int H, int nb, int* __restrict__ boff) {
    for (int b = blockIdx.x * blockDim.x + threadIdx.x; b <= nb; b += gridDim.x * blockDim.x)
        boff[b] = rp[int64_t(b) * H < M ? int64_t(b) * H : int64_t(M)];
}

// An entry's view word without its local column: row within the band (the 7 bits above the local
// column's) and the fp16 bits of value / scale (bits 16-31). One warp per row.
__global__ void band_payload_kernel(const int* __restrict__ rp, const float* __restrict__ val, int M, int H,
                                    float inv_scale, uint32_t* __restrict__ payload) {
    const int lane = threadIdx.x & 31;
    const int64_t nwarps = int64_t(gridDim.x) * (blockDim.x >> 5);
    for (int64_t r = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; r < M; r += nwarps) {
        const uint32_t row = uint32_t(r % H) << kBandColBits;
        for (int p = rp[r] + lane; p < rp[r + 1]; p += 32)
            payload[p] = row | (uint32_t(__half_as_ushort(__float2half_rn(val[p] * inv_scale))) << 16);
    }
}

// Greedy kBandK-column tiles over a band's entries sorted by column: a tile starts at the first
// column at or past the end of the previous tile. One warp per band walks its entries 32 at a
// time; inside a chunk, the next start is the first lane (ballot) whose column reaches the current
// end, repeated while one does. kWrite = false counts the tiles; kWrite = true writes tile_col,
// tile_eptr and each entry's local column into ents.
template <bool kWrite>
__global__ void band_tiles_kernel(const int* __restrict__ boff, const int* __restrict__ scol, int nb,
                                  int* __restrict__ ntiles, const int* __restrict__ tile_ptr,
                                  int* __restrict__ tile_col, int* __restrict__ tile_eptr, uint32_t* __restrict__ ents) {
    const int lane = threadIdx.x & 31;
    const int64_t nwarps = int64_t(gridDim.x) * (blockDim.x >> 5);
    for (int64_t b = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; b < nb; b += nwarps) {
        const int e0 = boff[b], e1 = boff[b + 1];
        int t = kWrite ? tile_ptr[b] : 0;
        int64_t end = -1;  // first column past the current tile
        int start = 0;     // the current tile's first column
        for (int base = e0; base < e1; base += 32) {
            const int i = base + lane;
            const bool valid = i < e1;
            const int c = valid ? scol[i] : 0;
            int mine = start;  // the start of the tile this lane's entry falls in
            unsigned pend = __ballot_sync(0xffffffffu, valid && c >= end);
            while (pend) {
                const int L = __ffs(pend) - 1;
                const int s = __shfl_sync(0xffffffffu, c, L);
                if (kWrite && lane == 0) {
                    tile_col[t] = s;
                    tile_eptr[t] = base + L;
                }
                ++t;
                if (lane >= L) mine = s;
                start = s;
                end = int64_t(s) + kBandK;
                pend = __ballot_sync(0xffffffffu, valid && c >= end);
            }
            if (kWrite && valid) ents[i] |= uint32_t(c - mine);
        }
        if (!kWrite && lane == 0) ntiles[b] = t;
    }
}

// The checks build_band_view makes on the host: per band, tiles in range, covering exactly the
// band's entries, each non-empty, starts ascending by at least kBandK columns.
__global__ void validate_band_kernel(const int* __restrict__ boff, const int* __restrict__ tile_ptr,
                                     const int* __restrict__ tile_col, const int* __restrict__ tile_eptr, int nb,
                                     int64_t T, int* bad) {
    for (int64_t b = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; b < nb; b += int64_t(gridDim.x) * blockDim.x) {
        const int t0 = tile_ptr[b], t1 = tile_ptr[b + 1];
        const int e0 = boff[b], e1 = boff[b + 1];
        if (t0 < 0 || t1 < t0 || t1 > T) {
            atomicOr(bad, 1);
            continue;
        }
        if ((t1 > t0 && (tile_eptr[t0] != e0 || tile_eptr[t1] != e1)) || (t1 == t0 && e1 != e0)) atomicOr(bad, 2);
        for (int t = t0; t < t1; ++t) {
            if (tile_eptr[t + 1] <= tile_eptr[t] || tile_col[t] < 0 ||
                (t > t0 && int64_t(tile_col[t]) < int64_t(tile_col[t - 1]) + kBandK))
                atomicOr(bad, 4);
        }
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

BandChoice choose_band_device(const int* row_ptr, const int* col, int M, cudaStream_t st) {
    // The sampled ranges of all candidate heights overlap (every height samples row 0): the union
    // of their rows is copied once, as merged intervals.
    std::vector<int> store, bound;
    return choose_band_sampled(M, [&](const std::vector<std::pair<int, int>>& ranges, std::vector<const int*>& first,
                                      std::vector<const int*>& last) {
        const size_t n = ranges.size();
        std::vector<size_t> order(n);
        for (size_t i = 0; i < n; ++i) order[i] = i;
        std::sort(order.begin(), order.end(), [&](size_t a, size_t b) { return ranges[a] < ranges[b]; });
        std::vector<std::pair<int, int>> merged;
        std::vector<size_t> owner(n);
        for (const size_t i : order) {
            if (merged.empty() || ranges[i].first > merged.back().second) merged.push_back(ranges[i]);
            else merged.back().second = std::max(merged.back().second, ranges[i].second);
            owner[i] = merged.size() - 1;
        }
        // row_ptr at every range's ends and every interval's ends
        std::vector<int> rows;
        for (const auto& r : ranges) rows.insert(rows.end(), {r.first, r.second});
        for (const auto& m : merged) rows.insert(rows.end(), {m.first, m.second});
        const int nr = int(rows.size());
        Buf<int> drows(rows.size()), dvals(rows.size());
        check(cudaMemcpyAsync(drows.p, rows.data(), sizeof(int) * rows.size(), cudaMemcpyHostToDevice, st),
              "cudaMemcpyAsync");
        gather_int_kernel<<<blocks_for(nr), 256, 0, st>>>(row_ptr, drows.p, nr, dvals.p);
        check(cudaGetLastError(), "gather_int_kernel");
        bound.resize(rows.size());
        check(cudaMemcpyAsync(bound.data(), dvals.p, sizeof(int) * rows.size(), cudaMemcpyDeviceToHost, st),
              "cudaMemcpyAsync");
        check(cudaStreamSynchronize(st), "cudaStreamSynchronize");
        const int* mb = bound.data() + 2 * n;
        std::vector<int64_t> moff(merged.size() + 1, 0);
        for (size_t m = 0; m < merged.size(); ++m) moff[m + 1] = moff[m] + (mb[2 * m + 1] - mb[2 * m]);
        store.resize(size_t(moff.back()));
        for (size_t m = 0; m < merged.size(); ++m)
            if (moff[m + 1] > moff[m])
                check(cudaMemcpyAsync(store.data() + moff[m], col + mb[2 * m], sizeof(int) * size_t(moff[m + 1] - moff[m]),
                                      cudaMemcpyDeviceToHost, st),
                      "cudaMemcpyAsync");
        check(cudaStreamSynchronize(st), "cudaStreamSynchronize");
        for (size_t i = 0; i < n; ++i) {
            const size_t m = owner[i];
            first[i] = store.data() + moff[m] + (bound[2 * i] - mb[2 * m]);
            last[i] = first[i] + (bound[2 * i + 1] - bound[2 * i]);
        }
    });
}

BandLayout build_band_layout(const int* row_ptr, const int* col, const float* val, int M, int64_t nnz, float scale,
                             int band_rows, cudaStream_t st) {
    if (band_rows < 1 || band_rows > kBandRows) throw StatusError(VCSRMC_INTERNAL, "band height out of range");
    const int H = band_rows;
    const int nb = int((int64_t(M) + H - 1) / H);
    Buf<int> boff(size_t(nb) + 1), ntiles(size_t(nb) + 1), tile_ptr(size_t(nb) + 1);
    band_offsets_kernel<<<blocks_for(int64_t(nb) + 1), 256, 0, st>>>(row_ptr, M, H, nb, boff.p);
    check(cudaGetLastError(), "band_offsets_kernel");
    Buf<int> scol(static_cast<size_t>(nnz));
    Buf<uint32_t> ents(static_cast<size_t>(nnz));
    if (nnz) {
        Buf<uint32_t> payload(static_cast<size_t>(nnz));
        band_payload_kernel<<<blocks_for(int64_t(M) * 32), 256, 0, st>>>(row_ptr, val, M, H, 1.0f / scale, payload.p);
        check(cudaGetLastError(), "band_payload_kernel");
        // Rows enter a band in ascending order, so a stable sort by column gives (column, row).
        size_t tmp = 0;
        check(cub::DeviceSegmentedSort::StableSortPairs(nullptr, tmp, col, scol.p, payload.p, ents.p, int(nnz), nb,
                                                         boff.p, boff.p + 1, st),
              "cub segmented sort");
        Buf<uint8_t> t(tmp);
        check(cub::DeviceSegmentedSort::StableSortPairs(t.p, tmp, col, scol.p, payload.p, ents.p, int(nnz), nb, boff.p,
                                                         boff.p + 1, st),
              "cub segmented sort");
        check(cudaStreamSynchronize(st), "cudaStreamSynchronize");
    }
    check(cudaMemsetAsync(ntiles.p, 0, sizeof(int) * (size_t(nb) + 1), st), "cudaMemsetAsync");
    if (nb > 0) {
        band_tiles_kernel<false><<<blocks_for(int64_t(nb) * 32), 256, 0, st>>>(boff.p, scol.p, nb, ntiles.p, nullptr,
                                                                            nullptr, nullptr, nullptr);
        check(cudaGetLastError(), "band_tiles_kernel");
    }
    exclusive_scan(ntiles.p, tile_ptr.p, int64_t(nb) + 1, st);
    const int64_t T = read_one(tile_ptr.p + nb, st);
    if (T < 0 || T > nnz) throw StatusError(VCSRMC_INTERNAL, "band view construction is inconsistent");
    Buf<int> tile_col(static_cast<size_t>(T)), tile_eptr(size_t(T) + 1);
    const int nnz32 = int(nnz);
    check(cudaMemcpyAsync(tile_eptr.p + T, &nnz32, sizeof(int), cudaMemcpyHostToDevice, st), "cudaMemcpyAsync");
    if (nb > 0) {
        band_tiles_kernel<true><<<blocks_for(int64_t(nb) * 32), 256, 0, st>>>(boff.p, scol.p, nb, nullptr, tile_ptr.p,
                                                                           tile_col.p, tile_eptr.p, ents.p);
        check(cudaGetLastError(), "band_tiles_kernel");
    }
    Buf<int> bad(1);
    check(cudaMemsetAsync(bad.p, 0, sizeof(int), st), "cudaMemsetAsync");
    if (nb > 0) {
        validate_band_kernel<<<blocks_for(nb), 256, 0, st>>>(boff.p, tile_ptr.p, tile_col.p, tile_eptr.p, nb, T, bad.p);
        check(cudaGetLastError(), "validate_band_kernel");
    }
    if (read_one(bad.p, st) != 0) throw StatusError(VCSRMC_INTERNAL, "band view construction is inconsistent");
    BandLayout L;
    L.band_rows = H;
    L.n_bands = nb;
    L.n_tiles = T;
    L.tile_ptr = tile_ptr.release();
    L.tile_col = tile_col.release();
    L.tile_eptr = tile_eptr.release();
    L.ents = ents.release();
    return L;
}

// ---- HYBRID plan: dense band tiles and the residual row view ------------------------------------
namespace {

// Per tile: dense (>= min entries) or not; per entry: the same flag and its tile; per tile: its band.
__global__ void hybrid_tile_kernel(const int* __restrict__ tile_ptr, const int* __restrict__ tile_eptr, int nb,
                                   int min_entries, int* __restrict__ tile_dense, int* __restrict__ tile_band,
                                   int* __restrict__ ent_dense, int* __restrict__ ent_tile) {
    for (int64_t b = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; b < nb; b += int64_t(gridDim.x) * blockDim.x) {
        for (int t = tile_ptr[b]; t < tile_ptr[b + 1]; ++t) {
            const int e0 = tile_eptr[t], e1 = tile_eptr[t + 1];
            const int d = e1 - e0 >= min_entries ? 1 : 0;
            tile_dense[t] = d;
            tile_band[t] = int(b);
            for (int e = e0; e < e1; ++e) {
                ent_dense[e] = d;
                ent_tile[e] = t;
            }
        }
    }
}

// The dense layout: tile t -> tpos[t], entry e -> epos[e]; band b's tiles start at tpos[tile_ptr[b]].
__global__ void hybrid_dense_kernel(const int* __restrict__ tile_ptr, const int* __restrict__ tile_col,
                                    const int* __restrict__ tile_eptr, const int* __restrict__ tile_dense,
                                    const int* __restrict__ tpos, const int* __restrict__ epos, int nb, int64_t T,
                                    int* __restrict__ d_tile_ptr, int* __restrict__ d_tile_col,
                                    int* __restrict__ d_tile_eptr) {
    const int64_t stride = int64_t(gridDim.x) * blockDim.x;
    for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i <= nb; i += stride)
        d_tile_ptr[i] = tpos[tile_ptr[i]];
    for (int64_t t = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; t < T; t += stride)
        if (tile_dense[t]) {
            d_tile_col[tpos[t]] = tile_col[t];
            d_tile_eptr[tpos[t]] = epos[tile_eptr[t]];
        }
}

// Dense entries to their compacted place; the others as (row << 32 | column) keys with fp16 values.
__global__ void hybrid_entries_kernel(const uint32_t* __restrict__ ents, const int* __restrict__ ent_dense,
                                      const int* __restrict__ ent_tile, const int* __restrict__ epos,
                                      const int* __restrict__ tile_band, const int* __restrict__ tile_col, int H,
                                      int64_t nnz, uint32_t* __restrict__ d_ents, uint64_t* __restrict__ r_key,
                                      unsigned short* __restrict__ r_val) {
    for (int64_t e = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; e < nnz; e += int64_t(gridDim.x) * blockDim.x) {
        const uint32_t w = ents[e];
        if (ent_dense[e]) {
            d_ents[epos[e]] = w;
        } else {
            const int t = ent_tile[e];
            const int64_t r = e - epos[e];  // residual entries before e
            const int row = tile_band[t] * H + int((w >> kBandColBits) & 127u);
            const int col = tile_col[t] + int(w & uint32_t(kBandK - 1));
            r_key[r] = (uint64_t(uint32_t(row)) << 32) | uint32_t(col);
            r_val[r] = static_cast<unsigned short>(w >> 16);
        }
    }
}

// Residual row view from its sorted keys: columns, and the count of each row.
__global__ void hybrid_resid_kernel(const uint64_t* __restrict__ key, int64_t n, int* __restrict__ cols,
                                    int* __restrict__ row_count) {
    for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
        const uint64_t k = key[i];
        cols[i] = int(uint32_t(k));
        atomicAdd(row_count + int(k >> 32), 1);
    }
}

// The dense layout's own invariants: band tile ranges inside [0, T), entry ranges increasing from 0
// to D, tiles of a band in ascending, non-overlapping column order.
__global__ void validate_dense_band_kernel(const int* __restrict__ tile_ptr, const int* __restrict__ tile_col,
                                           const int* __restrict__ tile_eptr, int nb, int64_t T, int64_t D, int* bad) {
    for (int64_t b = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; b < nb; b += int64_t(gridDim.x) * blockDim.x) {
        const int t0 = tile_ptr[b], t1 = tile_ptr[b + 1];
        if (t0 < 0 || t1 < t0 || t1 > T) {
            atomicOr(bad, 1);
            continue;
        }
        for (int t = t0; t < t1; ++t)
            if (tile_eptr[t] < 0 || tile_eptr[t + 1] <= tile_eptr[t] || tile_eptr[t + 1] > D || tile_col[t] < 0 ||
                (t > t0 && int64_t(tile_col[t]) < int64_t(tile_col[t - 1]) + kBandK))
                atomicOr(bad, 2);
    }
}

}  // namespace

HybridLayout build_hybrid_layout(const BandLayout& full, int M, int N, int64_t nnz, int min_entries, int unit_nnz,
                                 cudaStream_t st) {
    const int nb = full.n_bands, H = full.band_rows;
    const int64_t T = full.n_tiles;
    Buf<int> tile_dense(size_t(T) + 1), tile_band(size_t(std::max<int64_t>(T, 1))), tpos(size_t(T) + 1);
    Buf<int> ent_dense(size_t(nnz) + 1), ent_tile(size_t(std::max<int64_t>(nnz, 1))), epos(size_t(nnz) + 1);
    check(cudaMemsetAsync(tile_dense.p, 0, sizeof(int) * (size_t(T) + 1), st), "cudaMemsetAsync");
    check(cudaMemsetAsync(ent_dense.p, 0, sizeof(int) * (size_t(nnz) + 1), st), "cudaMemsetAsync");
    if (nb > 0) {
        hybrid_tile_kernel<<<blocks_for(nb), 256, 0, st>>>(full.tile_ptr, full.tile_eptr, nb, min_entries, tile_dense.p,
                                                           tile_band.p, ent_dense.p, ent_tile.p);
        check(cudaGetLastError(), "hybrid_tile_kernel");
    }
    exclusive_scan(tile_dense.p, tpos.p, T + 1, st);
    exclusive_scan(ent_dense.p, epos.p, nnz + 1, st);
    const int64_t TD = read_one(tpos.p + T, st), D = read_one(epos.p + nnz, st), R = nnz - D;
    if (TD < 0 || TD > T || D < 0 || D > nnz) throw StatusError(VCSRMC_INTERNAL, "hybrid split is inconsistent");
    HybridLayout out;
    out.dense_nnz = D;
    out.resid_nnz = R;
    // dense part
    Buf<int> d_tile_ptr(size_t(nb) + 1), d_tile_col(size_t(std::max<int64_t>(TD, 1))), d_tile_eptr(size_t(TD) + 1);
    Buf<uint32_t> d_ents(size_t(std::max<int64_t>(D, 1)));
    const int D32 = int(D);
    check(cudaMemcpyAsync(d_tile_eptr.p + TD, &D32, sizeof(int), cudaMemcpyHostToDevice, st), "cudaMemcpyAsync");
    hybrid_dense_kernel<<<blocks_for(std::max<int64_t>(T, int64_t(nb) + 1)), 256, 0, st>>>(
        full.tile_ptr, full.tile_col, full.tile_eptr, tile_dense.p, tpos.p, epos.p, nb, T, d_tile_ptr.p, d_tile_col.p,
        d_tile_eptr.p);
    check(cudaGetLastError(), "hybrid_dense_kernel");
    // residual part
    Buf<uint64_t> r_key(size_t(std::max<int64_t>(R, 1))), r_skey(size_t(std::max<int64_t>(R, 1)));
    Buf<unsigned short> r_val(size_t(std::max<int64_t>(R, 1))), r_sval(size_t(std::max<int64_t>(R, 1)));
    if (nnz > 0) {
        hybrid_entries_kernel<<<blocks_for(nnz), 256, 0, st>>>(full.ents, ent_dense.p, ent_tile.p, epos.p, tile_band.p,
                                                               full.tile_col, H, nnz, d_ents.p, r_key.p, r_val.p);
        check(cudaGetLastError(), "hybrid_entries_kernel");
    }
    Buf<int> bad(1);
    check(cudaMemsetAsync(bad.p, 0, sizeof(int), st), "cudaMemsetAsync");
    if (nb > 0) {
        validate_dense_band_kernel<<<blocks_for(nb), 256, 0, st>>>(d_tile_ptr.p, d_tile_col.p, d_tile_eptr.p, nb, TD,
                                                                   D, bad.p);
        check(cudaGetLastError(), "validate_dense_band_kernel");
    }
    if (read_one(bad.p, st) != 0) throw StatusError(VCSRMC_INTERNAL, "hybrid dense band layout is inconsistent");
    Buf<int> rp(size_t(M) + 1), rcols(size_t(std::max<int64_t>(R, 1))), row_count(size_t(M) + 1);
    check(cudaMemsetAsync(row_count.p, 0, sizeof(int) * (size_t(M) + 1), st), "cudaMemsetAsync");
    if (R > 0) {
        int end_bit = 33;
        while (end_bit < 64 && (uint64_t(uint32_t(M)) << 32) >> end_bit) ++end_bit;
        size_t tmp = 0;
        check(cub::DeviceRadixSort::SortPairs(nullptr, tmp, r_key.p, r_skey.p, r_val.p, r_sval.p, R, 0, end_bit, st),
              "cub sort");
        Buf<uint8_t> t(tmp);
        check(cub::DeviceRadixSort::SortPairs(t.p, tmp, r_key.p, r_skey.p, r_val.p, r_sval.p, R, 0, end_bit, st),
              "cub sort");
        hybrid_resid_kernel<<<blocks_for(R), 256, 0, st>>>(r_skey.p, R, rcols.p, row_count.p);
        check(cudaGetLastError(), "hybrid_resid_kernel");
    }
    exclusive_scan(row_count.p, rp.p, int64_t(M) + 1, st);
    // work units over the non-empty rows, packed on the host from row_ptr alone
    std::vector<int> hrp(size_t(M) + 1);
    check(cudaMemcpyAsync(hrp.data(), rp.p, sizeof(int) * (size_t(M) + 1), cudaMemcpyDeviceToHost, st),
          "cudaMemcpyAsync");
    check(cudaStreamSynchronize(st), "cudaStreamSynchronize");
    if (hrp[size_t(M)] != R) throw StatusError(VCSRMC_INTERNAL, "hybrid residual rows are inconsistent");
    std::vector<RowViewHost::Unit> hunits;
    std::vector<int> hsplit;
    pack_units(hrp.data(), M, unit_nnz, hunits, hsplit, true);
    Buf<int4> units(hunits.size());
    Buf<int> split(hsplit.size());
    if (!hunits.empty())
        check(cudaMemcpyAsync(units.p, hunits.data(), sizeof(int4) * hunits.size(), cudaMemcpyHostToDevice, st),
              "cudaMemcpyAsync");
    if (!hsplit.empty())
        check(cudaMemcpyAsync(split.p, hsplit.data(), sizeof(int) * hsplit.size(), cudaMemcpyHostToDevice, st),
              "cudaMemcpyAsync");
    RowsLayout rl;
    rl.rp = rp.p;
    rl.cols = rcols.p;
    rl.units = units.p;
    rl.n_units = int64_t(hunits.size());
    if (!device_validate(nullptr, &rl, M, N, 16, st))
        throw StatusError(VCSRMC_INTERNAL, "hybrid residual rows failed their index checks");
    out.dense.band_rows = H;
    out.dense.n_bands = nb;
    out.dense.n_tiles = TD;
    out.dense.tile_ptr = d_tile_ptr.release();
    out.dense.tile_col = d_tile_col.release();
    out.dense.tile_eptr = d_tile_eptr.release();
    out.dense.ents = d_ents.release();
    out.resid.rp = rp.release();
    out.resid.cols = rcols.release();
    out.resid.vals = r_sval.release();
    out.resid.units = units.release();
    out.resid.n_units = int64_t(hunits.size());
    out.resid.split_rows = split.release();
    out.resid.n_split_rows = int(hsplit.size());
    return out;
}

// ---- hot columns of the ROWS plan ------------------------------------------------------------
namespace {

__global__ void column_count_kernel(const int* __restrict__ cols, int64_t nnz, unsigned* __restrict__ count) {
    for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < nnz; i += int64_t(gridDim.x) * blockDim.x)
        atomicAdd(count + cols[i], 1u);
}

// key = ~count, so that an ascending sort orders columns by descending count; counts the columns
// used at all and those used at least twice.
__global__ void column_key_kernel(const unsigned* __restrict__ count, int N, unsigned* __restrict__ key,
                                  int* __restrict__ id, unsigned long long* __restrict__ used) {
    for (int64_t c = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; c < N; c += int64_t(gridDim.x) * blockDim.x) {
        const unsigned n = count[c];
        key[c] = ~n;
        id[c] = int(c);
        if (n >= 1) atomicAdd(used, 1ull);
        if (n >= 2) atomicAdd(used + 1, 1ull);
    }
}

// rank_of[col] = rank for the first k columns of the sorted order.
__global__ void hot_rank_kernel(const int* __restrict__ sorted_id, int k, int* __restrict__ rank_of) {
    for (int64_t r = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; r < k; r += int64_t(gridDim.x) * blockDim.x)
        rank_of[sorted_id[r]] = int(r);
}

__global__ void hot_rewrite_kernel(int* __restrict__ cols, int64_t nnz, const int* __restrict__ rank_of) {
    for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < nnz; i += int64_t(gridDim.x) * blockDim.x) {
        const int r = rank_of[cols[i]];
        if (r >= 0) cols[i] = ~r;
    }
}

}  // namespace

int* build_hot_columns(int* cols, int64_t nnz, int N, int max_hot, int* n_hot, cudaStream_t st) {
    *n_hot = 0;
    if (max_hot <= 0 || nnz <= 0 || N <= 0) return nullptr;
    const size_t n = static_cast<size_t>(N);
    Buf<unsigned> count(n), key(n), skey(n);
    Buf<int> id(n), sid(n);
    Buf<unsigned long long> tally(2);
    check(cudaMemsetAsync(count.p, 0, sizeof(unsigned) * n, st), "cudaMemsetAsync");
    check(cudaMemsetAsync(tally.p, 0, sizeof(unsigned long long) * 2, st), "cudaMemsetAsync");
    column_count_kernel<<<blocks_for(nnz), 256, 0, st>>>(cols, nnz, count.p);
    check(cudaGetLastError(), "column_count_kernel");
    column_key_kernel<<<blocks_for(N), 256, 0, st>>>(count.p, N, key.p, id.p, tally.p);
    check(cudaGetLastError(), "column_key_kernel");
    {
        size_t tmp = 0;
        check(cub::DeviceRadixSort::SortPairs(nullptr, tmp, key.p, skey.p, id.p, sid.p, N, 0, 32, st), "cub sort");
        Buf<uint8_t> t(tmp);
        check(cub::DeviceRadixSort::SortPairs(t.p, tmp, key.p, skey.p, id.p, sid.p, N, 0, 32, st), "cub sort");
    }
    unsigned long long used[2] = {0, 0};
    check(cudaMemcpyAsync(used, tally.p, sizeof used, cudaMemcpyDeviceToHost, st), "cudaMemcpyAsync");
    check(cudaStreamSynchronize(st), "cudaStreamSynchronize");
    const int k = int(std::min<unsigned long long>(used[1], (unsigned long long)max_hot));
    if (k <= 0) return nullptr;
    Buf<int> rank_of(n);
    check(cudaMemsetAsync(rank_of.p, 0xff, sizeof(int) * n, st), "cudaMemsetAsync");
    hot_rank_kernel<<<blocks_for(k), 256, 0, st>>>(sid.p, k, rank_of.p);
    check(cudaGetLastError(), "hot_rank_kernel");
    hot_rewrite_kernel<<<blocks_for(nnz), 256, 0, st>>>(cols, nnz, rank_of.p);
    check(cudaGetLastError(), "hot_rewrite_kernel");
    Buf<int> hot(static_cast<size_t>(k));
    check(cudaMemcpyAsync(hot.p, sid.p, sizeof(int) * static_cast<size_t>(k), cudaMemcpyDeviceToDevice, st),
          "cudaMemcpyAsync");
    check(cudaStreamSynchronize(st), "cudaStreamSynchronize");
    *n_hot = k;
    return hot.release();
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
