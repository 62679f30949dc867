// Host sparse-matrix containers and the Matrix Market loader.
//
// Same types, fields and behaviour as the reference's loaders:
//   COO, read_matrix_market_coo  <- include/mmio.hpp:12-75
//   CSR, coo_to_csr              <- include/csr.hpp:8-41
// Errors are reported by throwing std::runtime_error, as there; the C ABI (vcsrmc.h)
// turns them into status codes.
#pragma once
#include <cstdint>
#include <stdexcept>
#include <string>
#include <vector>

#ifndef VCSRMC_CXX_API
#define VCSRMC_CXX_API __attribute__((visibility("default")))
#endif

namespace vcsrmc {

// Thrown for a file that cannot be opened / for malformed or unsupported matrix data. Both
// derive from std::runtime_error, as the reference's errors do.
struct IoError : std::runtime_error {
    using std::runtime_error::runtime_error;
};
struct FormatError : std::runtime_error {
    using std::runtime_error::runtime_error;
};

struct COO {
    int M{0}, N{0};
    std::vector<int> rows, cols;
    std::vector<float> vals;
};

struct CSR {
    int M{0}, N{0}, nnz{0};
    std::vector<int> row_ptr;  // M + 1
    std::vector<int> col;      // nnz, ascending within each row
    std::vector<float> val;    // nnz
};

// Parses a Matrix Market "coordinate" file (real | integer | pattern; general | symmetric |
// skew-symmetric). Indices are one-based in the file; symmetric entries are expanded; values
// must be finite fp32; the expanded entry count must fit a signed 32-bit int.
VCSRMC_CXX_API COO read_matrix_market_coo(const std::string& path);

// Counting sort by row, then ascending columns within each row. Throws on an index out of
// range and on a duplicate (row, column) coordinate.
VCSRMC_CXX_API CSR coo_to_csr(const COO& coo);

// Rows [r0, r1) of `csr` as a CSR of their own (row ids rebased to 0; columns unchanged).
VCSRMC_CXX_API CSR csr_row_slice(const CSR& csr, int r0, int r1);

// Binary CSR cache (no reference counterpart): a 32-byte header ("VCSRMC1\0", int64 M, N, nnz)
// followed by row_ptr (int32, M + 1), col (int32, nnz) and val (fp32, nnz), little-endian.
// Loading checks the sizes, row_ptr (0 first, non-decreasing, nnz last) and the column range.
VCSRMC_CXX_API void save_csr_binary(const CSR& csr, const std::string& path);
VCSRMC_CXX_API CSR load_csr_binary(const std::string& path);

}  // namespace vcsrmc
