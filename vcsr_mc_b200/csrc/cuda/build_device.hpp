// GPU-side construction of the VCSR-MC format and of the ROWS plan's row view from a CSR that is
// already in device memory (see build_device.cu).
#pragma once
#include <cuda_runtime.h>

#include <cstdint>

#include "plan_band.hpp"

namespace vcsrmc {
namespace dev {

// Device arrays of the SEGMENT plan, in the layout device_api.cu uploads (the caller owns them).
struct SegmentLayout {
    int2* items = nullptr;   // {gbeg, gend}
    int4* gmeta = nullptr;   // {slot_begin, depth, seg_base, 0}
    int* grows = nullptr;    // 16 per group, -1 = padding
    int8_t* lcol = nullptr;  // per slot, -1 = padding
    void* val = nullptr;     // per slot: __half (FP16 format) or float (FP32 format)
    int64_t n_groups = 0, n_slots = 0, n_items = 0;
    int num_segments = 0;
};

// Device arrays of the ROWS plan (the caller owns them).
struct RowsLayout {
    int* rp = nullptr;
    int* cols = nullptr;
    void* vals = nullptr;  // __half (FP16 format) or float
    int4* units = nullptr;
    int64_t n_units = 0;
    int* split_rows = nullptr;
    int n_split_rows = 0;
};

// Device arrays of the BAND plan, in the host-built view's layout (plan_band.hpp; the caller
// owns them).
struct BandLayout {
    int* tile_ptr = nullptr;   // n_bands + 1
    int* tile_col = nullptr;   // n_tiles
    int* tile_eptr = nullptr;  // n_tiles + 1
    uint32_t* ents = nullptr;  // nnz
    int band_rows = 0, n_bands = 0;
    int64_t n_tiles = 0;
};

// Largest |val| (exact); the FP16 scale follows from it as in half_scale.
float device_abs_max(const float* val, int64_t nnz, cudaStream_t st);

// Same, without allocating: the scratch word is a file-scope device array (one per device), so
// calls must not overlap (the C ABI serialises them).
float device_abs_max_noalloc(const float* val, int64_t nnz, cudaStream_t st);

// Checks row_ptr (0 first, non-decreasing, nnz last) and that every row's columns are strictly
// ascending and inside [0, N). Returns false otherwise (blocking).
bool device_csr_rows_sorted(const int* row_ptr, const int* col, int M, int N, int64_t nnz, cudaStream_t st);

// The VCSR-MC arrays of csr_to_vcsr_mc (src/vcsr_mc.cu:25-123) with equal-count rows of a
// segment in ascending row order. Throws StatusError on failure (nothing is leaked).
SegmentLayout build_segment_layout(const int* row_ptr, const int* col, const float* val, int M, int N, int64_t nnz,
                                   int segw, bool fp32, float scale, cudaStream_t st);

// The row view: the CSR itself (rows sorted by column are already in the format's entry order),
// values divided by the scale, and the work units of the host-built view (packed on the host from
// row_ptr).
RowsLayout build_rows_layout(const int* row_ptr, const int* col, const float* val, int M, int64_t nnz, bool fp32,
                             float scale, int unit_nnz, cudaStream_t st);

// The band height and entries per tile that choose_band gives for the same CSR, from the sampled
// bands' columns copied to the host (at most the entries of 512 bands of <= 128 rows).
BandChoice choose_band_device(const int* row_ptr, const int* col, int M, cudaStream_t st);

// The BAND plan's view, bit for bit the one build_band_view makes on the host: a stable segmented
// sort of each band's entries by column, then one warp per band cuts the greedy kBandK-column tiles.
// Checks the view before returning; throws StatusError on failure (nothing is leaked).
BandLayout build_band_layout(const int* row_ptr, const int* col, const float* val, int M, int64_t nnz, float scale,
                             int band_rows, cudaStream_t st);

// HYBRID plan from a full band layout `full` of the matrix (build_band_layout): the tiles with at
// least min_entries entries as a band layout of their own (tiles and entries compacted in order, so
// it equals the band view the host builds from the dense entries), and every other entry as a row
// view (rows ascending, columns ascending in a row, fp16 values; units packed over non-empty rows
// for accumulate-only use). `full` is left as it is. Throws StatusError on failure (nothing leaked).
struct HybridLayout {
    BandLayout dense;
    RowsLayout resid;
    int64_t dense_nnz = 0, resid_nnz = 0;
};
HybridLayout build_hybrid_layout(const BandLayout& full, int M, int N, int64_t nnz, int min_entries, int unit_nnz,
                                 cudaStream_t st);

// Checks the invariants the SpMM kernels rely on (index ranges, offsets, item ranges). Blocking.
bool device_validate(const SegmentLayout* seg, const RowsLayout* rows, int M, int N, int segw, cudaStream_t st);

}  // namespace dev
}  // namespace vcsrmc
