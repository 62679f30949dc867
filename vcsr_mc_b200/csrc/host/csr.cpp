// Matrix Market reader and COO -> CSR conversion (behaviour of include/mmio.hpp:19-75 and
// include/csr.hpp:16-41 of the reference; see vcsrmc/csr.hpp).
#include "vcsrmc/csr.hpp"

#include "parallel.hpp"

#include <algorithm>
#include <atomic>
#include <cerrno>
#include <cctype>
#include <climits>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <limits>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

namespace vcsrmc {
namespace {

// Whitespace-separated token scanner over one line [p, end). Integers and reals are parsed the
// way a C++ stream extraction accepts them for this file format: optional sign, decimal digits
// (and for reals a decimal fraction and exponent). Hexadecimal and inf/nan spellings are not
// numbers here.
struct LineScanner {
    const char* p;
    const char* end;
    LineScanner(const char* b, const char* e) : p(b), end(e) {}
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
    // strtoll / strtod over [b, q) (NUL-terminated copy: on the stack for the usual lengths)
    template <class F>
    static auto convert(const char* b, const char* q, F fn) {
        char small[64];
        const size_t n = size_t(q - b);
        if (n < sizeof small) {
            std::memcpy(small, b, n);
            small[n] = 0;
            return fn(small);
        }
        const std::string tok(b, q);
        return fn(tok.c_str());
    }
    bool integer(long long& out) {
        skip_ws();
        const char* b = p;
        const char* q = p;
        if (q < end && (*q == '+' || *q == '-')) ++q;
        if (q >= end || !std::isdigit(static_cast<unsigned char>(*q))) return false;
        while (q < end && std::isdigit(static_cast<unsigned char>(*q))) ++q;
        bool range = false;
        out = convert(b, q, [&](const char* t) {
            errno = 0;
            const long long v = std::strtoll(t, nullptr, 10);
            range = errno == ERANGE;
            return v;
        });
        if (range) return false;
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
        out = convert(b, q, [](const char* t) { return std::strtod(t, nullptr); });
        p = q;
        return true;
    }
};

// A line holds data unless it is blank or its first character other than ' ', '\t', '\r' is '%'.
bool is_data_line(const char* b, const char* e) {
    while (b < e && (*b == ' ' || *b == '\t' || *b == '\r')) ++b;
    return b < e && *b != '%';
}

// Lines of [b, e) as getline splits them (a final line without '\n' counts).
template <class Fn>
void for_each_line(const char* b, const char* e, Fn&& fn) {
    while (b < e) {
        const char* nl = static_cast<const char*>(std::memchr(b, '\n', size_t(e - b)));
        const char* le = nl ? nl : e;
        if (!fn(b, le)) return;
        b = nl ? nl + 1 : e;
    }
}

struct Header {
    bool pattern, general, skew;
    long long m, n, count;
    size_t data_begin;  // offset of the first byte after the dimensions line
};

// One chunk of data lines, parsed on its own.
struct Chunk {
    std::vector<int> rows, cols;
    std::vector<float> vals;
    long long lines = 0;         // data lines seen
    long long err_line = -1;     // first bad data line (chunk-local index)
    std::string err;
};

void parse_chunk(const Header& h, const char* b, const char* e, Chunk& out) {
    for_each_line(b, e, [&](const char* lb, const char* le) {
        if (!is_data_line(lb, le)) return true;
        const long long i = out.lines++;
        LineScanner sc(lb, le);
        long long r = 0, c = 0;
        double value = 1.0;
        auto fail = [&](std::string m) {
            out.err_line = i;
            out.err = std::move(m);
            return false;
        };
        if (!sc.integer(r) || !sc.integer(c) || (!h.pattern && !sc.real(value)))
            return fail("Bad MTX entry at index ");
        if (!sc.at_end()) return fail("Extra fields in MTX entry");
        if (r < 1 || r > h.m || c < 1 || c > h.n)
            return fail("MTX row/column index out of range (expected one-based indices)");
        if (!std::isfinite(value) || std::abs(value) > std::numeric_limits<float>::max())
            return fail("MTX value is not finite FP32");
        if (h.skew && r == c && value != 0) return fail("Skew-symmetric MTX diagonal must be zero");
        out.rows.push_back(int(r - 1));
        out.cols.push_back(int(c - 1));
        out.vals.push_back(float(value));
        if (!h.general && r != c) {
            out.rows.push_back(int(c - 1));
            out.cols.push_back(int(r - 1));
            out.vals.push_back(float(h.skew ? -value : value));
        }
        return true;
    });
    // data lines after a bad one are still counted: the caller needs the count only when the
    // first error lies beyond the declared entries
    if (out.err_line >= 0) {
        const char* q = b;
        long long n = 0;
        for_each_line(q, e, [&](const char* lb, const char* le) {
            if (is_data_line(lb, le)) ++n;
            return true;
        });
        out.lines = n;
    }
}

}  // namespace

COO read_matrix_market_coo(const std::string& path) {
    std::FILE* f = std::fopen(path.c_str(), "rb");
    if (!f) throw IoError("Failed to open MTX: " + path);
    std::string buf;
    {
        char tmp[1 << 16];
        size_t got;
        std::fseek(f, 0, SEEK_END);
        const long size = std::ftell(f);
        std::fseek(f, 0, SEEK_SET);
        if (size > 0) buf.reserve(size_t(size));
        while ((got = std::fread(tmp, 1, sizeof tmp, f)) > 0) buf.append(tmp, got);
        const bool bad = std::ferror(f) != 0;
        std::fclose(f);
        if (bad) throw IoError("Failed to read MTX: " + path);
    }
    const char* const B = buf.data();
    const char* const E = B + buf.size();

    // banner: the first line
    if (buf.empty()) throw FormatError("Empty MTX file");
    const char* nl = static_cast<const char*>(std::memchr(B, '\n', buf.size()));
    const char* cur = nl ? nl + 1 : E;
    LineScanner banner(B, nl ? nl : E);
    const std::string magic = banner.word(), object = banner.word(), layout = banner.word();
    const std::string field = banner.word(), symmetry = banner.word();
    if (magic != "%%MatrixMarket" || object != "matrix" || layout != "coordinate")
        throw FormatError("Expected a Matrix Market coordinate matrix");
    if (field != "real" && field != "integer" && field != "pattern")
        throw FormatError("Unsupported MTX field: " + field);
    if (symmetry != "general" && symmetry != "symmetric" && symmetry != "skew-symmetric")
        throw FormatError("Unsupported MTX symmetry: " + symmetry);

    // dimensions: the next data line
    const char* dims_b = nullptr;
    const char* dims_e = nullptr;
    for_each_line(cur, E, [&](const char* lb, const char* le) {
        if (!is_data_line(lb, le)) return true;
        dims_b = lb;
        dims_e = le;
        return false;
    });
    if (!dims_b) throw FormatError("Missing MTX dimensions");
    Header h{};
    {
        LineScanner dims(dims_b, dims_e);
        if (!dims.integer(h.m) || !dims.integer(h.n) || !dims.integer(h.count) || h.m <= 0 || h.n <= 0 ||
            h.m >= INT_MAX || h.n >= INT_MAX || h.count < 0 || h.count > INT_MAX)
            throw FormatError("Invalid or unsupported MTX dimensions/nnz");
    }
    if (symmetry != "general" && h.m != h.n) throw FormatError("Symmetric MTX must be square");
    h.pattern = field == "pattern";
    h.general = symmetry == "general";
    h.skew = symmetry == "skew-symmetric";
    h.data_begin = size_t(dims_e - B) + (dims_e < E ? 1 : 0);

    // data lines: chunks cut at line boundaries, parsed in parallel, joined in file order
    const char* db = B + h.data_begin;
    const size_t bytes = size_t(E - db);
    const int nth = bytes < (size_t(1) << 20) ? 1 : std::max(1, std::min(resolve_threads(0), int(bytes >> 20)));
    std::vector<const char*> cut(static_cast<size_t>(nth) + 1);
    cut[0] = db;
    cut[size_t(nth)] = E;
    for (int t = 1; t < nth; ++t) {
        const char* q = db + bytes * size_t(t) / size_t(nth);
        if (q < cut[size_t(t) - 1]) q = cut[size_t(t) - 1];
        const char* n2 = static_cast<const char*>(std::memchr(q, '\n', size_t(E - q)));
        cut[size_t(t)] = n2 ? n2 + 1 : E;
    }
    std::vector<Chunk> chunks(static_cast<size_t>(nth));
    parallel_for(0, nth, nth, [&](int64_t t0, int64_t t1) {
        for (int64_t t = t0; t < t1; ++t) parse_chunk(h, cut[size_t(t)], cut[size_t(t) + 1], chunks[size_t(t)]);
    });
    // The sequential reader stops at the first bad one of the declared entries, then reports a
    // short file, then data lines beyond the declared count.
    long long seen = 0;
    for (const Chunk& c : chunks) {
        if (c.err_line >= 0 && seen + c.err_line < h.count) {
            const long long idx = seen + c.err_line;
            if (c.err == "Bad MTX entry at index ") throw FormatError(c.err + std::to_string(idx));
            throw FormatError(c.err);
        }
        seen += c.lines;
    }
    if (seen < h.count) throw FormatError("Truncated MTX data");
    if (seen > h.count) throw FormatError("Extra entries after declared MTX nnz");
    size_t total = 0;
    for (const Chunk& c : chunks) total += c.vals.size();
    if (total > size_t(INT_MAX)) throw FormatError("Expanded MTX exceeds 32-bit nnz limit");

    COO coo;
    coo.M = int(h.m);
    coo.N = int(h.n);
    coo.rows.resize(total);
    coo.cols.resize(total);
    coo.vals.resize(total);
    std::vector<size_t> off(chunks.size() + 1, 0);
    for (size_t t = 0; t < chunks.size(); ++t) off[t + 1] = off[t] + chunks[t].vals.size();
    parallel_for(0, int64_t(chunks.size()), nth, [&](int64_t t0, int64_t t1) {
        for (int64_t t = t0; t < t1; ++t) {
            Chunk& c = chunks[size_t(t)];
            std::copy(c.rows.begin(), c.rows.end(), coo.rows.begin() + off[size_t(t)]);
            std::copy(c.cols.begin(), c.cols.end(), coo.cols.begin() + off[size_t(t)]);
            std::copy(c.vals.begin(), c.vals.end(), coo.vals.begin() + off[size_t(t)]);
            c = Chunk();
        }
    });
    return coo;
}

namespace {

// coo_to_csr for large inputs: the same CSR (rows end up sorted by their unique columns, so the
// order entries reach a row in does not matter), with the counting sort and the per-row sorts
// spread over the host threads.
CSR coo_to_csr_parallel(const COO& coo) {
    const int64_t nnz = int64_t(coo.vals.size());
    const int nth = resolve_threads(0);
    CSR csr;
    csr.M = coo.M;
    csr.N = coo.N;
    csr.nnz = int(nnz);
    std::atomic<bool> bad_row{false}, bad_col{false};
    parallel_for(0, nnz, nth, [&](int64_t a, int64_t b) {
        for (int64_t i = a; i < b; ++i) {
            if (coo.rows[size_t(i)] < 0 || coo.rows[size_t(i)] >= csr.M) bad_row = true;
            if (coo.cols[size_t(i)] < 0 || coo.cols[size_t(i)] >= csr.N) bad_col = true;
        }
    });
    if (bad_row) throw FormatError("row idx out of range");
    if (bad_col) throw FormatError("column idx out of range");
    std::vector<int> cnt(size_t(csr.M) + 1, 0);
    parallel_for(0, nnz, nth, [&](int64_t a, int64_t b) {
        for (int64_t i = a; i < b; ++i) __atomic_fetch_add(&cnt[size_t(coo.rows[size_t(i)]) + 1], 1, __ATOMIC_RELAXED);
    });
    csr.row_ptr.resize(size_t(csr.M) + 1);
    csr.row_ptr[0] = 0;
    for (int r = 0; r < csr.M; ++r) csr.row_ptr[size_t(r) + 1] = csr.row_ptr[size_t(r)] + cnt[size_t(r) + 1];
    std::vector<int> cursor(csr.row_ptr.begin(), csr.row_ptr.end() - 1);
    csr.col.resize(size_t(nnz));
    csr.val.resize(size_t(nnz));
    parallel_for(0, nnz, nth, [&](int64_t a, int64_t b) {
        for (int64_t i = a; i < b; ++i) {
            const int dst = __atomic_fetch_add(&cursor[size_t(coo.rows[size_t(i)])], 1, __ATOMIC_RELAXED);
            csr.col[size_t(dst)] = coo.cols[size_t(i)];
            csr.val[size_t(dst)] = coo.vals[size_t(i)];
        }
    });
    std::atomic<bool> dup{false};
    parallel_for_dynamic(0, csr.M, nth, 4096, [&](int64_t r0, int64_t r1) {
        std::vector<std::pair<int, float>> tmp;
        for (int64_t r = r0; r < r1; ++r) {
            const int s = csr.row_ptr[size_t(r)], e = csr.row_ptr[size_t(r) + 1];
            tmp.resize(size_t(e - s));
            for (int i = s; i < e; ++i) tmp[size_t(i - s)] = {csr.col[size_t(i)], csr.val[size_t(i)]};
            std::sort(tmp.begin(), tmp.end(), [](const auto& x, const auto& y) { return x.first < y.first; });
            for (int i = s; i < e; ++i) {
                csr.col[size_t(i)] = tmp[size_t(i - s)].first;
                csr.val[size_t(i)] = tmp[size_t(i - s)].second;
                if (i > s && csr.col[size_t(i)] == csr.col[size_t(i) - 1]) dup = true;
            }
        }
    });
    if (dup) throw FormatError("Duplicate MTX coordinates are unsupported; coalesce them before benchmarking");
    return csr;
}

}  // namespace

CSR coo_to_csr(const COO& coo) {
    if (coo.vals.size() >= (size_t(1) << 20)) return coo_to_csr_parallel(coo);
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

namespace {
constexpr char kCsrMagic[8] = {'V', 'C', 'S', 'R', 'M', 'C', '1', '\0'};

struct File {
    std::FILE* f;
    explicit File(std::FILE* x) : f(x) {}
    ~File() { if (f) std::fclose(f); }
};
}  // namespace

void save_csr_binary(const CSR& csr, const std::string& path) {
    if (int64_t(csr.row_ptr.size()) != int64_t(csr.M) + 1 || int64_t(csr.col.size()) != csr.nnz ||
        int64_t(csr.val.size()) != csr.nnz)
        throw std::runtime_error("inconsistent CSR");
    File out(std::fopen(path.c_str(), "wb"));
    if (!out.f) throw IoError("Failed to create " + path);
    const int64_t hdr[3] = {csr.M, csr.N, csr.nnz};
    bool ok = std::fwrite(kCsrMagic, 1, sizeof kCsrMagic, out.f) == sizeof kCsrMagic &&
              std::fwrite(hdr, sizeof hdr[0], 3, out.f) == 3 &&
              std::fwrite(csr.row_ptr.data(), sizeof(int), csr.row_ptr.size(), out.f) == csr.row_ptr.size() &&
              std::fwrite(csr.col.data(), sizeof(int), csr.col.size(), out.f) == csr.col.size() &&
              std::fwrite(csr.val.data(), sizeof(float), csr.val.size(), out.f) == csr.val.size();
    ok = (std::fclose(out.f) == 0) && ok;
    out.f = nullptr;
    if (!ok) throw IoError("Failed to write " + path);
}

CSR load_csr_binary(const std::string& path) {
    File in(std::fopen(path.c_str(), "rb"));
    if (!in.f) throw IoError("Failed to open " + path);
    char magic[8];
    int64_t hdr[3];
    if (std::fread(magic, 1, sizeof magic, in.f) != sizeof magic || std::memcmp(magic, kCsrMagic, sizeof magic) != 0 ||
        std::fread(hdr, sizeof hdr[0], 3, in.f) != 3)
        throw FormatError("Not a binary CSR file: " + path);
    const int64_t M = hdr[0], N = hdr[1], nnz = hdr[2];
    if (M < 0 || N < 0 || nnz < 0 || M >= INT_MAX || N >= INT_MAX || nnz > INT_MAX)
        throw FormatError("Binary CSR sizes out of range: " + path);
    std::fseek(in.f, 0, SEEK_END);
    const long long size = std::ftell(in.f);
    const long long want = 32 + (M + 1) * 4 + nnz * 8;
    if (size != want) throw FormatError("Binary CSR file has the wrong size: " + path);
    std::fseek(in.f, 32, SEEK_SET);
    CSR csr;
    csr.M = int(M);
    csr.N = int(N);
    csr.nnz = int(nnz);
    csr.row_ptr.resize(size_t(M) + 1);
    csr.col.resize(size_t(nnz));
    csr.val.resize(size_t(nnz));
    if (std::fread(csr.row_ptr.data(), sizeof(int), csr.row_ptr.size(), in.f) != csr.row_ptr.size() ||
        std::fread(csr.col.data(), sizeof(int), csr.col.size(), in.f) != csr.col.size() ||
        std::fread(csr.val.data(), sizeof(float), csr.val.size(), in.f) != csr.val.size())
        throw IoError("Failed to read " + path);
    if (csr.row_ptr[0] != 0 || csr.row_ptr[size_t(M)] != csr.nnz) throw FormatError("Binary CSR row_ptr is inconsistent");
    for (int64_t r = 0; r < M; ++r)
        if (csr.row_ptr[size_t(r) + 1] < csr.row_ptr[size_t(r)]) throw FormatError("Binary CSR row_ptr is inconsistent");
    std::atomic<bool> bad{false};
    parallel_for(0, nnz, resolve_threads(0), [&](int64_t a, int64_t b) {
        for (int64_t i = a; i < b; ++i)
            if (csr.col[size_t(i)] < 0 || csr.col[size_t(i)] >= csr.N) bad = true;
    });
    if (bad) throw FormatError("Binary CSR column index out of range");
    return csr;
}

}  // namespace vcsrmc
