// The VCSR-MC sparse format and its host construction.
//
// Same struct, fields and construction as the reference (include/vcsr_formats.hpp:14-26,
// src/vcsr_mc.cu:14-123):
//   * a segment is `segw` consecutive columns of A (= `segw` consecutive rows of B);
//   * within a segment, the rows of A that touch it are ordered by their entry count in that
//     segment, descending, and cut into groups of `bundle` = 16 rows;
//   * a group stores depth x 16 (lcol, val) slots, depth-major, padded with (-1, 0);
//   * a work item is a run of at most `chunk` consecutive groups of one segment; items are
//     ordered by slot count, heaviest first (stable).
// The arrays are bit-identical to the reference builder's output for the same CSR.
#pragma once
#include <cstdint>
#include <vector>
#include "csr.hpp"

#ifndef VCSRMC_CXX_API
#define VCSRMC_CXX_API __attribute__((visibility("default")))
#endif

namespace vcsrmc {

struct VCSRMC {
    int M{0}, N{0}, segw{16}, bundle{16}, num_segments{0};
    std::vector<int> group_ptr, group_depth, group_seg_base, group_rows, lcol;
    std::vector<float> val;
    std::vector<int> item_gbeg, item_gend;  // groups [gbeg, gend) of one segment per item
    float scale{1.0f};
    bool fp32{false};  // FP32 operands; FP16 path otherwise (values divided by `scale`)
};

// Factor that A is divided by before FP16 conversion (C is multiplied back by it).
VCSRMC_CXX_API float half_scale(const CSR& csr);

// segw must be 16, 32, 48 or 64. `nthreads` <= 0 picks the hardware concurrency; the result
// does not depend on it.
VCSRMC_CXX_API VCSRMC csr_to_vcsr_mc(const CSR& csr, bool fp32 = false, int segw = 16, int nthreads = 0);

}  // namespace vcsrmc
