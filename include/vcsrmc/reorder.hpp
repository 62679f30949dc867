// Reverse Cuthill-McKee column reordering.
//
// Same algorithm and results as the reference (include/reorder.hpp:17-108): the permutation
// clusters the columns that rows touch into narrow bands, so fewer VCSR segments (and staged
// B tiles) are needed per row. A and B are permuted consistently, so C = A*B is unchanged.
#pragma once
#include <vector>
#include "csr.hpp"

#ifndef VCSRMC_CXX_API
#define VCSRMC_CXX_API __attribute__((visibility("default")))
#endif

namespace vcsrmc {

// Returns new_position[old_column] (include/reorder.hpp:17-77).
VCSRMC_CXX_API std::vector<int> rcm_column_order(const CSR& csr);

// Relabels A's columns by `position`, re-sorts every row by column, and permutes the rows of
// the N x O row-major host matrix hB to match (include/reorder.hpp:82-108).
VCSRMC_CXX_API void apply_column_permutation(CSR& csr, std::vector<float>& hB, int O,
                              const std::vector<int>& position);

}  // namespace vcsrmc
