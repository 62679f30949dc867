// Row-band SpMM plan on the tensor cores (FP16 format): C written once per band of rows.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>
#include <functional>
#include <utility>
#include <vector>

#include "plan_rows.hpp"

namespace vcsrmc {
namespace dev {

#ifndef VCSRMC_BAND_K
#define VCSRMC_BAND_K 64
#endif
constexpr int kBandRows = 128;          // rows per band at most = the largest MMA N
constexpr int kBandK = VCSRMC_BAND_K;   // columns of A (= rows of B) per tile: kBandK / 16 MMA K steps
constexpr int kBandColBits = kBandK == 64 ? 6 : 5;  // bits of an entry's column within its tile
static_assert(kBandK == 32 || kBandK == 64, "tiles of 32 or 64 columns");
// Below this many entries per tile the ROWS plan is faster (measured on a B200: about 2.3 ns of
// tensor-core pipeline per 64-column tile, 1.3 ns per 32-column one, against 0.025-0.045 ns per
// gathered entry for ROWS).
constexpr double kBandMinEntriesPerTile = kBandK == 64 ? 64.0 : 40.0;

// Host-side band view. Band b covers rows [b * band_rows, (b + 1) * band_rows). Its tiles are
// [tile_ptr[b], tile_ptr[b+1]) in ascending column order; tile t covers columns
// [tile_col[t], tile_col[t] + kBandK) and holds entries [tile_eptr[t], tile_eptr[t+1]). A tile
// starts at the first column of the band not covered by the previous tile, so a window of w
// consecutive occupied columns takes ceil(w / kBandK) tiles wherever it starts. An entry packs
// the local column (bits 0 .. kBandColBits - 1), the row within the band (the next 7 bits) and
// the fp16 value (bits 16-31).
struct BandViewHost {
    int band_rows = kBandRows;
    std::vector<int> tile_ptr, tile_col, tile_eptr;
    std::vector<uint32_t> ents;
};

// The band height (<= 128) that minimises the tensor-core time per row (tiles per row, weighted by
// the MMA size: N = 64 for bands of at most 64 rows, else 128; plus a per-band cost), estimated on a
// sample of bands, the mean entries per tile it gives, and the fraction of the sampled entries in
// tiles holding at least kBandMinEntriesPerTile entries (the HYBRID plan's dense part).
struct BandChoice {
    int band_rows;
    double entries_per_tile;
    double dense_fraction = 0.0;
};
// The default layouts add HYBRID (FP16 format, upload only) where BAND alone does not pay but at
// least this fraction of the entries sits in dense tiles.
constexpr double kHybridMinDenseFraction = 0.5;
BandChoice choose_band(const RowViewHost& rv, int M);

// The same choice from any source of the sampled bands: fetch(ranges, first, last) makes
// [first[i], last[i]) the columns (any order) of the entries of rows [ranges[i].first,
// ranges[i].second), in host memory that stays valid until the chooser returns.
using BandSampleFetch = std::function<void(const std::vector<std::pair<int, int>>& ranges,
                                           std::vector<const int*>& first, std::vector<const int*>& last)>;
BandChoice choose_band_sampled(int M, const BandSampleFetch& fetch);

// From the row view (rows' entries in ascending column order, values already divided by the
// format's scale). nthreads <= 0: all host threads.
BandViewHost build_band_view(const RowViewHost& rv, int M, int band_rows, int nthreads);

// Hybrid plan: tiles of the band view `bv` (built from `rv` at its band height) that hold at least
// min_entries entries are "dense". Their entries go to `dense`, all others to `resid`; both row
// views keep every row's ascending column order and values, and the band view of `dense` at the
// same height has exactly the dense tiles (a dense tile starts at its first entry's column, which
// stays the first uncovered column once the sparse tiles are gone). Units are not packed.
void split_dense_tiles(const RowViewHost& rv, const BandViewHost& bv, int M, int min_entries, int nthreads,
                       RowViewHost& dense, RowViewHost& resid);

struct BandPlanView {
    const int* tile_ptr;
    const int* tile_col;
    const int* tile_eptr;
    const uint32_t* ents;
    int n_bands, band_rows;
    int M, N;
    float scale;
    uint32_t* status;
};

cudaError_t spmm_band(const BandPlanView& P, const void* B, int b_is_f16, int64_t ldb, int O, float* C, int64_t ldc,
                      bool accumulate, cudaStream_t st);

}  // namespace dev
}  // namespace vcsrmc
