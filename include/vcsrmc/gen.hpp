// Seeded synthetic inputs (the benchmark configurations) and the multi-GPU row partition.
//
// All draws come from counter-based streams (vcsr_mc_b200/csrc/common/vrng.h): the output
// depends on the seed and the parameters only, never on the thread count.
#pragma once
#include <cstdint>
#include <vector>
#include "csr.hpp"

#ifndef VCSRMC_CXX_API
#define VCSRMC_CXX_API __attribute__((visibility("default")))
#endif

namespace vcsrmc {

// M x N, row length ~ Poisson(lambda) (inverse CDF), columns uniform without replacement
// (Floyd's algorithm), values U(-1,1).
VCSRMC_CXX_API CSR gen_uniform_poisson(int M, int N, double lambda, uint64_t seed, int nthreads = 0);

// M x N, row length k ~ Zipf(s) truncated to [1, kmax] (inverse CDF), then
// clamp(round(k * mean / E[k]), 1, kmax); columns uniform without replacement; values U(-1,1).
VCSRMC_CXX_API CSR gen_zipf_rows(int M, int N, double s, int kmax, double mean, uint64_t seed, int nthreads = 0);
VCSRMC_CXX_API double zipf_length_factor(double s, int kmax, double mean);

// 27-point stencil on an nx x ny x nz grid in natural (x fastest) order; diagonal 26,
// off-diagonal -1 + U(-0.01, 0.01).
VCSRMC_CXX_API CSR gen_stencil27(int nx, int ny, int nz, uint64_t seed, int nthreads = 0);

// The 27-point stencil of gen_stencil27 on n^3 plus `links` long-range links per row: link t of
// row i joins column (draw 2 (i links + t) of the links stream) mod n^3 with value U(-1,1) (the
// next draw); a link that falls on a stencil column or an earlier link of the row is dropped. A
// stand-in for a finite-element matrix with far couplings: dense diagonal bands plus scatter.
VCSRMC_CXX_API CSR gen_stencil27_links(int n, int links, uint64_t seed, int nthreads = 0);

// R-MAT graph with 2^scale vertices: `edges` samples with quadrant probabilities
// (a, b, c, 1-a-b-c), duplicates removed, values U(-1,1).
VCSRMC_CXX_API CSR gen_rmat(int scale, int64_t edges, double a, double b, double c, uint64_t seed, int nthreads = 0);

// rows x cols row-major U(-1,1), element i = row * cols + col of the dense stream.
VCSRMC_CXX_API void gen_dense(int64_t rows, int cols, uint64_t seed, float* out, int nthreads = 0);

VCSRMC_CXX_API int poisson_inverse(double u, double lambda, int cap);

// P+1 nnz-balanced row cuts: cuts[k] = first row whose nnz prefix reaches ceil(k*nnz/P).
VCSRMC_CXX_API std::vector<int> partition_rows(const int* row_ptr, int M, int parts);
// P+1 row cuts balancing the cost nnz + row_weight * rows of each block: cuts[k] = first row r
// whose prefix cost row_ptr[r] + row_weight * r reaches k/P of the total.
VCSRMC_CXX_API std::vector<int> partition_rows_weighted(const int* row_ptr, int M, int parts, double row_weight);

}  // namespace vcsrmc
