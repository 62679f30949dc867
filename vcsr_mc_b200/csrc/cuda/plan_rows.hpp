// Row-stationary SpMM plan over the row view of a VCSR-MC format (see plan_rows.cu).
#pragma once
#include <cuda_runtime.h>

#include <cstdint>
#include <vector>

#include "vcsrmc/vcsr_formats.hpp"

namespace vcsrmc {
namespace dev {

constexpr int kUnitNnzMax = 1024;  // entries per work unit: a power of two in [16, kUnitNnzMax]
constexpr int kUnitRows = 16;  // light rows per unit at most (one row end per lane of a 16-lane group)

// Host-side row view: row r's entries are cols/vals[rp[r], rp[r+1]) in ascending column order;
// units = {first row, end row | 0x80000000 for a heavy-row chunk, first entry, end entry}.
struct RowViewHost {
    std::vector<int> rp, cols;
    std::vector<float> vals;
    struct Unit { int x, y, z, w; };
    std::vector<Unit> units;
    std::vector<int> split_rows;
};

// unit_nnz: entries per work unit (rows with more are split into chunks of unit_nnz).
RowViewHost build_row_view(const VCSRMC& v, int unit_nnz);
// The work units of a row view from its row_ptr alone: every row with more than unit_nnz entries
// as unit_nnz-entry chunks (listed first, and in split_rows), then greedy runs of at most
// kUnitRows consecutive lighter rows with together at most unit_nnz entries.
void pack_units(const int* rp, int M, int unit_nnz, std::vector<RowViewHost::Unit>& units,
                std::vector<int>& split_rows);
// The unit size for a matrix of `nnz` entries on a GPU with `sms` SMs: the largest power of two
// in [16, 256] that still gives every resident lane group (48 per SM) about four units.
int choose_unit_nnz(int64_t nnz, int sms);

struct RowPlanView {
    const int4* units;
    int64_t n_units;
    const int* rp;
    const int* cols;
    const void* vals;  // __half if vals_f16 else float
    int vals_f16;
    const int* split_rows;
    int n_split_rows;
    int M;
    float scale;
};

cudaError_t spmm_rows(const RowPlanView& P, const void* B, int b_is_f16, int64_t ldb, int O, float* C, int64_t ldc,
                      bool accumulate, cudaStream_t st);

}  // namespace dev
}  // namespace vcsrmc
