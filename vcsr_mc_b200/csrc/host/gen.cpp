// Seeded synthetic inputs for the benchmark configurations (vcsrmc/gen.hpp). Every value
// is drawn from the counter-based streams of common/vrng.h, so the matrices do not depend on
// the thread count and the device-side dense generator reproduces B bit for bit.
#include "vcsrmc/gen.hpp"

#include <algorithm>
#include <atomic>
#include <climits>
#include <cmath>
#include <stdexcept>
#include <unordered_set>
#include <vector>

#include "../common/vrng.h"
#include "parallel.hpp"

namespace vcsrmc {
namespace {

// Floyd's algorithm (Bentley & Floyd, CACM 1987) for `len` distinct values of [0, n): the
// t-th draw of the row's sub-stream picks in [0, n - len + t]. Output ascending.
void floyd_sample(uint64_t key, uint64_t row, int len, int n, std::vector<int>& out) {
    out.clear();
    const uint64_t base = row << 32;
    if (len <= 64) {
        for (int t = 0; t < len; ++t) {
            const int j = n - len + t;
            const int x = int(vrng_at(key, base + uint64_t(t)) % uint64_t(j + 1));
            const bool taken = std::find(out.begin(), out.end(), x) != out.end();
            out.push_back(taken ? j : x);
        }
    } else {
        std::unordered_set<int> set;
        set.reserve(size_t(len) * 2);
        for (int t = 0; t < len; ++t) {
            const int j = n - len + t;
            const int x = int(vrng_at(key, base + uint64_t(t)) % uint64_t(j + 1));
            const int v = set.count(x) ? j : x;
            set.insert(v);
            out.push_back(v);
        }
    }
    std::sort(out.begin(), out.end());
}

// Row lengths -> CSR with Floyd-sampled columns and U(-1,1) values.
CSR rows_from_lengths(int M, int N, const std::vector<int>& len, uint64_t seed, int nthreads) {
    CSR csr;
    csr.M = M;
    csr.N = N;
    csr.row_ptr.assign(size_t(M) + 1, 0);
    int64_t total = 0;
    for (int r = 0; r < M; ++r) {
        total += len[r];
        if (total > INT_MAX) throw std::runtime_error("generated nnz exceeds 32-bit limit");
        csr.row_ptr[r + 1] = int(total);
    }
    csr.nnz = int(total);
    csr.col.resize(total);
    csr.val.resize(total);
    const uint64_t kcols = vrng_key(seed, VRNG_STREAM_COLS);
    const uint64_t kvals = vrng_key(seed, VRNG_STREAM_VALS);
    parallel_for_dynamic(0, M, nthreads, 256, [&](int64_t r0, int64_t r1) {
        std::vector<int> cols;
        for (int64_t r = r0; r < r1; ++r) {
            floyd_sample(kcols, uint64_t(r), len[r], N, cols);
            const int s = csr.row_ptr[r];
            for (size_t k = 0; k < cols.size(); ++k) {
                csr.col[s + k] = cols[k];
                csr.val[s + k] = vrng_sym(vrng_at(kvals, uint64_t(s + k)));
            }
        }
    });
    return csr;
}

}  // namespace

int poisson_inverse(double u, double lambda, int cap) {
    // Inverse CDF by summing the pmf upward from 0 (adequate for the small means used here).
    int k = 0;
    double p = std::exp(-lambda);
    double F = p;
    while (u >= F && k < cap) {
        ++k;
        p *= lambda / k;
        F += p;
    }
    return k;
}

CSR gen_uniform_poisson(int M, int N, double lambda, uint64_t seed, int nthreads) {
    if (M < 0 || N <= 0 || lambda < 0) throw std::runtime_error("bad uniform-Poisson parameters");
    nthreads = resolve_threads(nthreads);
    const uint64_t klen = vrng_key(seed, VRNG_STREAM_ROWLEN);
    std::vector<int> len(M);
    const int cap = int(std::min<double>(N, 10.0 * lambda + 100.0));
    for (int r = 0; r < M; ++r) len[r] = poisson_inverse(vrng_u01(vrng_at(klen, uint64_t(r))), lambda, cap);
    return rows_from_lengths(M, N, len, seed, nthreads);
}

double zipf_length_factor(double s, int kmax, double mean) {
    double z = 0, m = 0;
    for (int k = 1; k <= kmax; ++k) {
        const double w = std::pow(double(k), -s);
        z += w;
        m += k * w;
    }
    return mean / (m / z);
}

CSR gen_zipf_rows(int M, int N, double s, int kmax, double mean, uint64_t seed, int nthreads) {
    if (M < 0 || N <= 0 || kmax < 1 || s <= 0) throw std::runtime_error("bad Zipf parameters");
    nthreads = resolve_threads(nthreads);
    std::vector<double> cdf(kmax);
    double z = 0;
    for (int k = 1; k <= kmax; ++k) z += std::pow(double(k), -s);
    double acc = 0;
    for (int k = 1; k <= kmax; ++k) {
        acc += std::pow(double(k), -s);
        cdf[k - 1] = acc / z;
    }
    const double factor = zipf_length_factor(s, kmax, mean);
    const uint64_t klen = vrng_key(seed, VRNG_STREAM_ROWLEN);
    std::vector<int> len(M);
    const int cap = std::min(kmax, N);
    for (int r = 0; r < M; ++r) {
        const double u = vrng_u01(vrng_at(klen, uint64_t(r)));
        int k = int(std::upper_bound(cdf.begin(), cdf.end(), u) - cdf.begin()) + 1;
        k = std::min(k, kmax);
        const long long l = std::llround(double(k) * factor);
        len[r] = int(std::max<long long>(1, std::min<long long>(cap, l)));
    }
    return rows_from_lengths(M, N, len, seed, nthreads);
}

CSR gen_stencil27(int nx, int ny, int nz, uint64_t seed, int nthreads) {
    if (nx <= 0 || ny <= 0 || nz <= 0) throw std::runtime_error("bad stencil grid");
    nthreads = resolve_threads(nthreads);
    const int64_t n = int64_t(nx) * ny * nz;
    if (n > INT_MAX) throw std::runtime_error("stencil grid too large");
    CSR csr;
    csr.M = csr.N = int(n);
    csr.row_ptr.assign(size_t(n) + 1, 0);
    auto extent = [](int v, int lim) { return 1 + (v > 0) + (v + 1 < lim); };
    int64_t total = 0;
    for (int64_t i = 0; i < n; ++i) {
        const int x = int(i % nx), y = int((i / nx) % ny), zz = int(i / (int64_t(nx) * ny));
        total += int64_t(extent(x, nx)) * extent(y, ny) * extent(zz, nz);
        if (total > INT_MAX) throw std::runtime_error("stencil nnz exceeds 32-bit limit");
        csr.row_ptr[i + 1] = int(total);
    }
    csr.nnz = int(total);
    csr.col.resize(total);
    csr.val.resize(total);
    const uint64_t kvals = vrng_key(seed, VRNG_STREAM_VALS);
    parallel_for(0, n, nthreads, [&](int64_t i0, int64_t i1) {
        for (int64_t i = i0; i < i1; ++i) {
            const int x = int(i % nx), y = int((i / nx) % ny), zz = int(i / (int64_t(nx) * ny));
            int64_t p = csr.row_ptr[i];
            for (int dz = -1; dz <= 1; ++dz)
                for (int dy = -1; dy <= 1; ++dy)
                    for (int dx = -1; dx <= 1; ++dx) {
                        const int X = x + dx, Y = y + dy, Z = zz + dz;
                        if (X < 0 || X >= nx || Y < 0 || Y >= ny || Z < 0 || Z >= nz) continue;
                        csr.col[p] = int((int64_t(Z) * ny + Y) * nx + X);
                        if (dx == 0 && dy == 0 && dz == 0) {
                            csr.val[p] = 26.0f;
                        } else {
                            const uint64_t w = vrng_at(kvals, uint64_t(p));
                            const double noise = double(w >> 11) * (1.0 / 4503599627370496.0) - 1.0;
                            csr.val[p] = float(-1.0 + 0.01 * noise);
                        }
                        ++p;
                    }
        }
    });
    return csr;
}

CSR gen_stencil27_links(int n, int links, uint64_t seed, int nthreads) {
    if (links < 0 || links > 64) throw std::runtime_error("links per row out of range");
    const CSR st = gen_stencil27(n, n, n, seed, nthreads);
    nthreads = resolve_threads(nthreads);
    const int M = st.M;
    const uint64_t kl = vrng_key(seed, VRNG_STREAM_LINKS);
    // row i's extra columns, in draw order, without stencil columns or repeats
    auto extra = [&](int64_t i, std::vector<std::pair<int, float>>& out) {
        out.clear();
        const int* b = st.col.data() + st.row_ptr[i];
        const int* e = st.col.data() + st.row_ptr[i + 1];
        for (int t = 0; t < links; ++t) {
            const uint64_t d = 2 * (uint64_t(i) * uint64_t(links) + uint64_t(t));
            const int c = int(vrng_at(kl, d) % uint64_t(M));
            if (std::binary_search(b, e, c)) continue;
            bool seen = false;
            for (const auto& x : out) seen = seen || x.first == c;
            if (!seen) out.push_back({c, float(vrng_sym(vrng_at(kl, d + 1)))});
        }
    };
    CSR csr;
    csr.M = csr.N = M;
    csr.row_ptr.assign(size_t(M) + 1, 0);
    parallel_for(0, M, nthreads, [&](int64_t lo, int64_t hi) {
        std::vector<std::pair<int, float>> x;
        for (int64_t i = lo; i < hi; ++i) {
            extra(i, x);
            csr.row_ptr[size_t(i) + 1] = (st.row_ptr[i + 1] - st.row_ptr[i]) + int(x.size());
        }
    });
    int64_t total = 0;
    for (int r = 0; r < M; ++r) {
        total += csr.row_ptr[size_t(r) + 1];
        if (total > INT_MAX) throw std::runtime_error("generated nnz exceeds 32-bit limit");
        csr.row_ptr[size_t(r) + 1] = int(total);
    }
    csr.nnz = int(total);
    csr.col.resize(size_t(total));
    csr.val.resize(size_t(total));
    parallel_for(0, M, nthreads, [&](int64_t lo, int64_t hi) {
        std::vector<std::pair<int, float>> x;
        for (int64_t i = lo; i < hi; ++i) {
            extra(i, x);
            for (int p = st.row_ptr[i]; p < st.row_ptr[i + 1]; ++p) x.push_back({st.col[size_t(p)], st.val[size_t(p)]});
            std::sort(x.begin(), x.end(), [](const auto& u, const auto& v) { return u.first < v.first; });
            int q = csr.row_ptr[size_t(i)];
            for (const auto& e : x) {
                csr.col[size_t(q)] = e.first;
                csr.val[size_t(q++)] = e.second;
            }
        }
    });
    return csr;
}

CSR gen_rmat(int scale, int64_t edges, double a, double b, double c, uint64_t seed, int nthreads) {
    if (scale < 1 || scale > 30 || edges < 0 || a < 0 || b < 0 || c < 0 || a + b + c > 1)
        throw std::runtime_error("bad R-MAT parameters");
    nthreads = resolve_threads(nthreads);
    const int64_t n = int64_t(1) << scale;
    const uint64_t ta = uint64_t(std::floor(a * 4294967296.0));
    const uint64_t tab = uint64_t(std::floor((a + b) * 4294967296.0));
    const uint64_t tabc = uint64_t(std::floor((a + b + c) * 4294967296.0));
    const uint64_t krmat = vrng_key(seed, VRNG_STREAM_RMAT);
    const int words = (scale + 1) / 2;  // two 32-bit quadrant draws per 64-bit word
    // Bucket by the top `hb` row bits so each bucket can be sorted on its own.
    const int hb = std::min(scale, 12);
    const int nb = 1 << hb;
    const int shift_b = 2 * scale - hb;  // key = row << scale | col
    auto edge_key = [&](int64_t e) -> uint64_t {
        uint64_t row = 0, col = 0;
        uint64_t w = 0;
        for (int l = 0; l < scale; ++l) {
            if ((l & 1) == 0) w = vrng_at(krmat, uint64_t(e) * uint64_t(words) + uint64_t(l / 2));
            const uint64_t u = (l & 1) ? (w >> 32) : (w & 0xffffffffULL);
            const uint64_t rb = u >= tab, cb = (u >= ta && u < tab) || u >= tabc;
            row = (row << 1) | rb;
            col = (col << 1) | cb;
        }
        return (row << scale) | col;
    };
    const int T = int(std::max<int64_t>(1, std::min<int64_t>(nthreads, edges / 4096 + 1)));
    std::vector<std::vector<int64_t>> tcount(T, std::vector<int64_t>(nb, 0));
    std::vector<uint64_t> keys(edges);
    detail::run_threads(T, [&](int t) {
        const int64_t e0 = edges * t / T, e1 = edges * (t + 1) / T;
        std::vector<int64_t>& cnt = tcount[t];
        for (int64_t e = e0; e < e1; ++e) {
            const uint64_t k = edge_key(e);
            keys[e] = k;
            ++cnt[k >> shift_b];
        }
    });
    std::vector<int64_t> boff(size_t(nb) + 1, 0);
    std::vector<std::vector<int64_t>> tcur(T, std::vector<int64_t>(nb));
    for (int bk = 0; bk < nb; ++bk) {
        int64_t s = boff[bk];
        for (int t = 0; t < T; ++t) { tcur[t][bk] = s; s += tcount[t][bk]; }
        boff[bk + 1] = s;
    }
    std::vector<uint64_t> sorted(edges);
    detail::run_threads(T, [&](int t) {
        const int64_t e0 = edges * t / T, e1 = edges * (t + 1) / T;
        std::vector<int64_t>& cur = tcur[t];
        for (int64_t e = e0; e < e1; ++e) sorted[cur[keys[e] >> shift_b]++] = keys[e];
    });
    keys.clear();
    keys.shrink_to_fit();
    std::vector<int64_t> bkeep(size_t(nb) + 1, 0);
    parallel_for_dynamic(0, nb, nthreads, 1, [&](int64_t b0, int64_t b1) {
        for (int64_t bk = b0; bk < b1; ++bk) {
            auto first = sorted.begin() + boff[bk], last = sorted.begin() + boff[bk + 1];
            std::sort(first, last);
            bkeep[bk + 1] = std::unique(first, last) - first;
        }
    });
    for (int bk = 0; bk < nb; ++bk) bkeep[bk + 1] += bkeep[bk];
    const int64_t nnz = bkeep[nb];
    if (nnz > INT_MAX) throw std::runtime_error("R-MAT nnz exceeds 32-bit limit");
    CSR csr;
    csr.M = csr.N = int(n);
    csr.nnz = int(nnz);
    csr.col.resize(nnz);
    csr.val.resize(nnz);
    std::vector<int> rowcount(n, 0);
    const uint64_t cmask = (uint64_t(1) << scale) - 1;
    const uint64_t kvals = vrng_key(seed, VRNG_STREAM_VALS);
    // Buckets hold disjoint row ranges, so each row's count is written by one thread.
    parallel_for_dynamic(0, nb, nthreads, 1, [&](int64_t b0, int64_t b1) {
        for (int64_t bk = b0; bk < b1; ++bk) {
            const int64_t kept = bkeep[bk + 1] - bkeep[bk];
            for (int64_t i = 0; i < kept; ++i) {
                const uint64_t k = sorted[boff[bk] + i];
                const int64_t p = bkeep[bk] + i;
                csr.col[p] = int(k & cmask);
                csr.val[p] = vrng_sym(vrng_at(kvals, uint64_t(p)));
                ++rowcount[k >> scale];
            }
        }
    });
    csr.row_ptr.assign(size_t(n) + 1, 0);
    for (int64_t r = 0; r < n; ++r) csr.row_ptr[r + 1] = csr.row_ptr[r] + rowcount[r];
    return csr;
}

void gen_dense(int64_t rows, int cols, uint64_t seed, float* out, int nthreads) {
    nthreads = resolve_threads(nthreads);
    const uint64_t k = vrng_key(seed, VRNG_STREAM_DENSE);
    const int64_t total = rows * int64_t(cols);
    parallel_for(0, total, nthreads, [&](int64_t i0, int64_t i1) {
        for (int64_t i = i0; i < i1; ++i) out[i] = vrng_sym(vrng_at(k, uint64_t(i)));
    });
}

std::vector<int> partition_rows(const int* row_ptr, int M, int parts) {
    if (parts < 1 || M < 0) throw std::runtime_error("bad partition request");
    std::vector<int> cuts(size_t(parts) + 1, 0);
    const int64_t base = row_ptr[0], nnz = int64_t(row_ptr[M]) - base;
    cuts[parts] = M;
    for (int k = 1; k < parts; ++k) {
        // first row boundary whose prefix reaches ceil(k * nnz / parts)
        const int64_t target = base + (int64_t(k) * nnz + parts - 1) / parts;
        int r = int(std::lower_bound(row_ptr, row_ptr + M + 1, target,
                                     [](int v, int64_t t) { return int64_t(v) < t; }) - row_ptr);
        cuts[k] = std::max(cuts[k - 1], std::min(r, M));
    }
    return cuts;
}

std::vector<int> partition_rows_weighted(const int* row_ptr, int M, int parts, double row_weight) {
    if (parts < 1 || M < 0 || !(row_weight >= 0)) throw std::runtime_error("bad partition request");
    std::vector<int> cuts(size_t(parts) + 1, 0);
    const double base = row_ptr[0];
    const double total = (double(row_ptr[M]) - base) + row_weight * M;
    cuts[parts] = M;
    int r = 0;
    for (int k = 1; k < parts; ++k) {
        const double target = total * k / parts;
        // the prefix cost is non-decreasing in r: advance to the first row that reaches the target
        while (r < M && (double(row_ptr[r]) - base) + row_weight * r < target) ++r;
        cuts[k] = std::max(cuts[k - 1], r);
    }
    return cuts;
}

}  // namespace vcsrmc
