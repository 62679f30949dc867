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
// kUnitRows consecutive lighter rows with together at most unit_nnz entries. With skip_empty, no
// run starts at an empty row (for a view run in accumulate mode only, where empty rows need no
// store; a run may still hold empty rows between non-empty ones).
void pack_units(const int* rp, int M, int unit_nnz, std::vector<RowViewHost::Unit>& units,
                std::vector<int>& split_rows, bool skip_empty = false);
// The unit size for a matrix of `nnz` entries on a GPU with `sms` SMs: the largest power of two
// in [16, 256] that still gives every resident lane group (48 per SM) about four units.
int choose_unit_nnz(int64_t nnz, int sms);

// Hot columns of the row view. The most used columns of A (rank 0 = most entries) are numbered
// 0 .. n_hot-1 and their entries hold ~rank (a negative value) in `cols` instead of the column;
// hot_cols[rank] is the column itself. Per SpMM call the B rows of the leading ranks, up to the
// copy budget, are copied into a compact buffer (one gather kernel), so that the most popular
// rows of B sit in one contiguous range (optionally under a persisting L2 window); the remaining
// hot ranks are looked up in hot_cols. Rows of unranked columns can be read evict-first.
struct RowHotView {
    const int* hot_cols = nullptr;  // n_hot original columns, by rank
    int n_hot = 0;
    void* buf = nullptr;            // compact rows of B: row pitch = B's pitch (ldb elements)
    int64_t buf_bytes = 0;          // capacity of buf
    int64_t budget_bytes = 0;       // most bytes of B rows to copy per call (0: no copy, lookups only)
    bool persist = false;           // give the copied rows a persisting L2 access-policy window
    bool cold_hint = false;         // read rows outside the hot set with evict-first loads
};

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
    int N = 0;  // columns of A (rows of B): bounds the B row offsets the kernel forms
    float scale;
    RowHotView hot;
};

// Number of hot ranks whose B rows one call copies for this B layout (rows of row_bytes bytes).
int rows_hot_copy_count(const RowHotView& H, int64_t row_bytes);

// Kernels this call launches (for the benchmark's launch count): zeroing of split rows, the hot
// row copy, the SpMM.
int rows_launch_count(const RowPlanView& P, int64_t ldb, int b_is_f16, int O, bool accumulate);

cudaError_t spmm_rows(const RowPlanView& P, const void* B, int b_is_f16, int64_t ldb, int O, float* C, int64_t ldc,
                      bool accumulate, cudaStream_t st);

// Hot-column set of a row view whose `cols` are in device memory: counts the entries of every
// column, ranks the columns by count (descending; ties by ascending column), keeps at most
// max_hot ranks of columns with at least two entries, and rewrites the hot entries of `cols` as
// ~rank. Returns the device array of hot columns (cudaMalloc'd; the caller frees it) and their
// number in *n_hot, or nullptr with *n_hot = 0 when max_hot is 0 or no column qualifies.
// Blocking; throws StatusError on failure.
int* build_hot_columns(int* cols, int64_t nnz, int N, int max_hot, int* n_hot, cudaStream_t st);

}  // namespace dev
}  // namespace vcsrmc
