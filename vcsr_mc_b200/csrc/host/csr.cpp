// Matrix Market reader and COO -> CSR conversion (behaviour of include/mmio.hpp:19-75 and
// include/csr.hpp:16-41 of the reference; see vcsrmc/csr.hpp).
#include "vcsrmc/csr.hpp"

#include <algorithm>
#include <cerrno>
#include <cctype>
#include <climits>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <limits>
#include <stdexcept>
#include <string>
#include <utility>

namespace vcsrmc {
namespace {

// Whitespace-separated token scanner over one line. Integers and reals are parsed the way a
// C++ stream extraction accepts them for this file format: optional sign, decimal digits
// (and for reals a decimal fraction and exponent). Hexadecimal and inf/nan spellings are
// not numbers here.
struct LineScanner {
    const char* p;
    const char* end;
    explicit LineScanner(const std::string& s) : p(s.data()), end(s.data() + s.size()) {}
    void skip_ws() {
        while (p < end && std::isspace(static_cast<unsigned char>(*p))) ++p;
    }
    bool at_end() { skip_ws(); return p >= end; }
    std::string word() {
        skip_ws();
        const char* b = p;
        while (p < end && !std::isspace(static_cast<unsigned char>(*p))) ++p;
        return std::string(b, p);
    }
    bool integer(long long& out) {
        skip_ws();
        const char* b = p;
        const char* q = p;
        if (q < end && (*q == '+' || *q == '-')) ++q;
        if (q >= end || !std::isdigit(static_cast<unsigned char>(*q))) return false;
        while (q < end && std::isdigit(static_cast<unsigned char>(*q))) ++q;
        std::string tok(b, q);
        errno = 0;
        out = std::strtoll(tok.c_str(), nullptr, 10);
        if (errno == ERANGE) return false;
        p = q;
        return true;
    }
    bool real(double& out) {
        skip_ws();
        const char* b = p;
        const char* q = p;
        if (q < end && (*q == '+' || *q == '-')) ++q;
        bool digits = false;
        while (q < end && std::isdigit(static_cast<unsigned char>(*q))) { ++q; digits = true; }
        if (q < end && *q == '.') {
            ++q;
            while (q < end && std::isdigit(static_cast<unsigned char>(*q))) { ++q; digits = true; }
        }
        if (!digits) return false;
        if (q < end && (*q == 'e' || *q == 'E')) {
            const char* r = q + 1;
            if (r < end && (*r == '+' || *r == '-')) ++r;
            if (r < end && std::isdigit(static_cast<unsigned char>(*r))) {
                while (r < end && std::isdigit(static_cast<unsigned char>(*r))) ++r;
                q = r;
            }
        }
        std::string tok(b, q);
        out = std::strtod(tok.c_str(), nullptr);
        p = q;
        return true;
    }
};

bool next_data_line(std::ifstream& in, std::string& line) {
    while (std::getline(in, line)) {
        const auto first = line.find_first_not_of(" \t\r");
        if (first != std::string::npos && line[first] != '%') return true;
    }
    return false;
}

}  // namespace

COO read_matrix_market_coo(const std::string& path) {
    std::ifstream in(path);
    if (!in) throw IoError("Failed to open MTX: " + path);
    std::string line;
    if (!std::getline(in, line)) throw FormatError("Empty MTX file");
    LineScanner banner(line);
    const std::string magic = banner.word(), object = banner.word(), layout = banner.word();
    const std::string field = banner.word(), symmetry = banner.word();
    if (magic != "%%MatrixMarket" || object != "matrix" || layout != "coordinate")
        throw FormatError("Expected a Matrix Market coordinate matrix");
    if (field != "real" && field != "integer" && field != "pattern")
        throw FormatError("Unsupported MTX field: " + field);
    if (symmetry != "general" && symmetry != "symmetric" && symmetry != "skew-symmetric")
        throw FormatError("Unsupported MTX symmetry: " + symmetry);

    if (!next_data_line(in, line)) throw FormatError("Missing MTX dimensions");
    long long m = 0, n = 0, count = 0;
    {
        LineScanner dims(line);
        if (!dims.integer(m) || !dims.integer(n) || !dims.integer(count) || m <= 0 || n <= 0 ||
            m >= INT_MAX || n >= INT_MAX || count < 0 || count > INT_MAX)
            throw FormatError("Invalid or unsupported MTX dimensions/nnz");
    }
    if (symmetry != "general" && m != n) throw FormatError("Symmetric MTX must be square");

    const bool pattern = field == "pattern";
    const bool general = symmetry == "general";
    const bool skew = symmetry == "skew-symmetric";
    COO coo;
    coo.M = int(m);
    coo.N = int(n);
    const size_t expect = size_t(count) * (general ? 1 : 2);
    coo.rows.reserve(std::min<size_t>(expect, size_t(1) << 28));
    coo.cols.reserve(coo.rows.capacity());
    coo.vals.reserve(coo.rows.capacity());
    auto append = [&](int r, int c, float v) {
        if (coo.vals.size() >= size_t(INT_MAX))
            throw FormatError("Expanded MTX exceeds 32-bit nnz limit");
        coo.rows.push_back(r);
        coo.cols.push_back(c);
        coo.vals.push_back(v);
    };
    for (long long i = 0; i < count; ++i) {
        if (!next_data_line(in, line)) throw FormatError("Truncated MTX data");
        LineScanner e(line);
        long long r = 0, c = 0;
        double value = 1.0;
        if (!e.integer(r) || !e.integer(c) || (!pattern && !e.real(value)))
            throw FormatError("Bad MTX entry at index " + std::to_string(i));
        if (!e.at_end()) throw FormatError("Extra fields in MTX entry");
        if (r < 1 || r > m || c < 1 || c > n)
            throw FormatError("MTX row/column index out of range (expected one-based indices)");
        if (!std::isfinite(value) || std::abs(value) > std::numeric_limits<float>::max())
            throw FormatError("MTX value is not finite FP32");
        if (skew && r == c && value != 0)
            throw FormatError("Skew-symmetric MTX diagonal must be zero");
        append(int(r - 1), int(c - 1), float(value));
        if (!general && r != c) append(int(c - 1), int(r - 1), float(skew ? -value : value));
    }
    if (next_data_line(in, line)) throw FormatError("Extra entries after declared MTX nnz");
    return coo;
}

CSR coo_to_csr(const COO& coo) {
    CSR csr;
    csr.M = coo.M;
    csr.N = coo.N;
    csr.nnz = int(coo.vals.size());
    csr.row_ptr.assign(size_t(csr.M) + 1, 0);
    csr.col.resize(csr.nnz);
    csr.val.resize(csr.nnz);
    for (int r : coo.rows) {
        if (r < 0 || r >= csr.M) throw FormatError("row idx out of range");
        csr.row_ptr[size_t(r) + 1]++;
    }
    for (int i = 1; i <= csr.M; ++i) csr.row_ptr[i] += csr.row_ptr[i - 1];
    std::vector<int> cursor(csr.row_ptr.begin(), csr.row_ptr.end() - 1);
    for (size_t i = 0; i < coo.vals.size(); ++i) {
        const int dst = cursor[coo.rows[i]]++;
        if (coo.cols[i] < 0 || coo.cols[i] >= csr.N)
            throw FormatError("column idx out of range");
        csr.col[dst] = coo.cols[i];
        csr.val[dst] = coo.vals[i];
    }
    // Ascending columns within each row; a repeated column is an error, so the order of the
    // entries of a row is fully determined by their columns.
    std::vector<std::pair<int, float>> tmp;
    for (int r = 0; r < csr.M; ++r) {
        const int s = csr.row_ptr[r], e = csr.row_ptr[r + 1];
        bool sorted = true;
        for (int i = s + 1; i < e && sorted; ++i) sorted = csr.col[i - 1] < csr.col[i];
        if (!sorted) {
            tmp.resize(e - s);
            for (int i = s; i < e; ++i) tmp[i - s] = {csr.col[i], csr.val[i]};
            std::stable_sort(tmp.begin(), tmp.end(),
                             [](const auto& a, const auto& b) { return a.first < b.first; });
            for (int i = s; i < e; ++i) { csr.col[i] = tmp[i - s].first; csr.val[i] = tmp[i - s].second; }
        }
        for (int i = s + 1; i < e; ++i)
            if (csr.col[i] == csr.col[i - 1])
                throw FormatError(
                    "Duplicate MTX coordinates are unsupported; coalesce them before benchmarking");
    }
    return csr;
}

CSR csr_row_slice(const CSR& csr, int r0, int r1) {
    if (r0 < 0 || r1 < r0 || r1 > csr.M) throw std::runtime_error("row slice out of range");
    CSR out;
    out.M = r1 - r0;
    out.N = csr.N;
    const int base = csr.row_ptr[r0];
    out.row_ptr.resize(size_t(out.M) + 1);
    for (int r = r0; r <= r1; ++r) out.row_ptr[r - r0] = csr.row_ptr[r] - base;
    out.nnz = out.row_ptr.back();
    out.col.assign(csr.col.begin() + base, csr.col.begin() + csr.row_ptr[r1]);
    out.val.assign(csr.val.begin() + base, csr.val.begin() + csr.row_ptr[r1]);
    return out;
}

}  // namespace vcsrmc
