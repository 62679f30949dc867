// Host-side layout builders of the ROWS and BAND plans, checked on the CPU (no GPU involved):
// build_row_view (a host-built format transposed back into rows) and pack_units (its work units),
// build_band_view / choose_band (the BAND view).
// Each rule is stated here as properties of the output, not re-run: heavy rows become
// unit_nnz-entry chunks listed first; light rows form maximal greedy runs of at most kUnitRows rows
// and unit_nnz entries; the BAND view holds exactly each band's entries, in (column, row) order,
// in tiles whose starts are the greedy starts over the band's sorted columns.
// A row view is the CSR itself (a row with ascending columns lists its entries in the format's
// order) with the format's work units.
// Linked against the library's own objects (vcsr_mc_b200/_build/cuda/plan_rows.o, plan_band.o) and
// libvcsrmc.so (csr_to_vcsr_mc) by tests/test_layouts_cpu.py. Prints "OK ..." and exits 0, or names the first failed check.
#include <cuda_fp16.h>

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <random>
#include <set>
#include <tuple>
#include <vector>

#include "cuda/plan_band.hpp"
#include "cuda/plan_rows.hpp"
#include "vcsrmc/csr.hpp"
#include "vcsrmc/gen.hpp"
#include "vcsrmc/vcsr_formats.hpp"

using namespace vcsrmc::dev;

namespace {

using ll = long long;
int failures = 0;
ll densest_tile = 0;
void expect(bool ok, const char* what, long long a = 0, long long b = 0) {
    if (!ok && failures++ < 5) std::printf("FAIL %s (%lld, %lld)\n", what, a, b);
}

struct Csr {
    int M = 0, N = 0;
    std::vector<int> rp, col;
    std::vector<float> val;
};

// Row lengths from `draw`, columns sorted and distinct in [0, N), values U(-2, 2).
template <class Draw>
Csr make_csr(int M, int N, std::mt19937_64& g, Draw draw) {
    Csr a;
    a.M = M;
    a.N = N;
    a.rp.assign(size_t(M) + 1, 0);
    std::uniform_real_distribution<float> uv(-2.f, 2.f);
    for (int r = 0; r < M; ++r) {
        std::set<int> cs;
        const int len = std::min(N, draw(r));
        std::uniform_int_distribution<int> uc(0, N - 1);
        while (int(cs.size()) < len) cs.insert(uc(g));
        for (int c : cs) {
            a.col.push_back(c);
            a.val.push_back(uv(g));
        }
        a.rp[size_t(r) + 1] = int(a.col.size());
    }
    return a;
}

// A banded matrix like a 3-D stencil: row r holds columns r + d for d in three windows of three
// (offsets 0, +-w, +-w*w with w = 10), clipped to [0, M), plus an occasional random column.
Csr make_banded(int M, std::mt19937_64& g) {
    Csr a;
    a.M = a.N = M;
    a.rp.assign(size_t(M) + 1, 0);
    std::uniform_real_distribution<float> uv(-2.f, 2.f);
    std::uniform_int_distribution<int> uc(0, M - 1);
    for (int r = 0; r < M; ++r) {
        std::set<int> cs;
        for (int plane : {-100, 0, 100})
            for (int line : {-10, 0, 10})
                for (int d : {-1, 0, 1}) {
                    const int c = r + plane + line + d;
                    if (c >= 0 && c < M) cs.insert(c);
                }
        if (g() % 8 == 0) cs.insert(uc(g));
        for (int c : cs) {
            a.col.push_back(c);
            a.val.push_back(uv(g));
        }
        a.rp[size_t(r) + 1] = int(a.col.size());
    }
    return a;
}

void check_units(const std::vector<int>& rp, int M, int u) {
    std::vector<RowViewHost::Unit> units;
    std::vector<int> split;
    pack_units(rp.data(), M, u, units, split);
    auto len = [&](int r) { return rp[size_t(r) + 1] - rp[size_t(r)]; };
    size_t k = 0;
    std::vector<int> heavy;
    for (int r = 0; r < M; ++r)
        if (len(r) > u) heavy.push_back(r);
    expect(split == heavy, "split_rows are exactly the rows longer than unit_nnz", ll(split.size()), ll(heavy.size()));
    for (int r : heavy)  // chunks of the heavy rows first, in row order
        for (int p = rp[size_t(r)]; p < rp[size_t(r) + 1]; p += u, ++k) {
            const bool ok = k < units.size() && units[k].x == r && units[k].y == int(unsigned(r + 1) | 0x80000000u) &&
                            units[k].z == p && units[k].w == std::min(rp[size_t(r) + 1], p + u);
            expect(ok, "heavy-row chunk", r, p);
        }
    int next = 0;  // first row not yet covered by a light run
    for (; k < units.size(); ++k) {
        const auto& t = units[k];
        while (next < M && len(next) > u) ++next;
        expect(t.x == next, "light run starts at the first uncovered light row", t.x, next);
        expect(t.y > t.x && t.y - t.x <= kUnitRows && t.y <= M, "light run of 1 .. kUnitRows rows", t.x, t.y);
        expect(t.z == rp[size_t(t.x)] && t.w == rp[size_t(t.y)], "light run entry range", t.z, t.w);
        int n = 0;
        for (int r = t.x; r < t.y; ++r) {
            expect(len(r) <= u, "light run holds only light rows", r, len(r));
            n += len(r);
        }
        expect(n <= u, "light run within unit_nnz entries", n, u);
        if (t.y < M && t.y - t.x < kUnitRows && len(t.y) <= u)
            expect(n + len(t.y) > u, "light run is maximal", t.y, n);
        next = t.y;
    }
    while (next < M && len(next) > u) ++next;
    expect(next == M, "light runs cover every light row", next, M);
}

// skip_empty: the same heavy-row chunks; light runs never start at an empty row, and every
// non-empty light row is in exactly one run (empty rows may sit inside a run).
void check_units_skip_empty(const std::vector<int>& rp, int M, int u) {
    std::vector<RowViewHost::Unit> units;
    std::vector<int> split;
    pack_units(rp.data(), M, u, units, split, true);
    auto len = [&](int r) { return rp[size_t(r) + 1] - rp[size_t(r)]; };
    std::vector<int> covered(size_t(std::max(M, 1)), 0);
    for (const auto& t : units) {
        if (t.y & 0x80000000) continue;  // heavy-row chunk (checked by check_units)
        expect(len(t.x) > 0, "no run starts at an empty row", t.x, 0);
        expect(t.y > t.x && t.y - t.x <= kUnitRows && t.y <= M, "run of 1 .. kUnitRows rows", t.x, t.y);
        expect(t.z == rp[size_t(t.x)] && t.w == rp[size_t(t.y)], "run entry range", t.z, t.w);
        int n = 0;
        for (int r = t.x; r < t.y; ++r) {
            expect(len(r) <= u, "run holds only light rows", r, len(r));
            n += len(r);
            ++covered[size_t(r)];
        }
        expect(n <= u, "run within unit_nnz entries", n, u);
    }
    for (int r = 0; r < M; ++r)
        if (len(r) > 0 && len(r) <= u) expect(covered[size_t(r)] == 1, "non-empty light row in exactly one run", r, covered[size_t(r)]);
}

void check_row_view(const Csr& a, bool fp32, int segw, int u) {
    vcsrmc::CSR c;
    c.M = a.M;
    c.N = a.N;
    c.nnz = int(a.col.size());
    c.row_ptr = a.rp;
    c.col = a.col;
    c.val = a.val;
    const vcsrmc::VCSRMC v = vcsrmc::csr_to_vcsr_mc(c, fp32, segw, 2);
    expect(v.scale == 1.0f, "values in (-2, 2) keep half_scale at 1", 0, 0);
    const RowViewHost rv = build_row_view(v, u);
    expect(rv.rp == a.rp, "row view row_ptr is the CSR's", a.M, segw);
    expect(rv.cols == a.col, "row view columns are the CSR's, in order", a.M, segw);
    expect(rv.vals == a.val, "row view values are the CSR's", a.M, segw);
    std::vector<RowViewHost::Unit> units;
    std::vector<int> split;
    pack_units(a.rp.data(), a.M, u, units, split);
    bool same = units.size() == rv.units.size() && split == rv.split_rows;
    for (size_t i = 0; same && i < units.size(); ++i)
        same = units[i].x == rv.units[i].x && units[i].y == rv.units[i].y && units[i].z == rv.units[i].z &&
               units[i].w == rv.units[i].w;
    expect(same, "row view units are pack_units of its row_ptr", a.M, u);
}

unsigned short half_bits(float v) { return __half_as_ushort(__float2half_rn(v)); }

void check_band(const Csr& a, int H) {
    RowViewHost rv;
    rv.rp = a.rp;
    rv.cols = a.col;
    rv.vals = a.val;
    const BandViewHost b = build_band_view(rv, a.M, H, 2);
    const int nb = (a.M + H - 1) / H;
    expect(int(b.tile_ptr.size()) == nb + 1 && b.tile_ptr[0] == 0, "tile_ptr size", ll(b.tile_ptr.size()), nb + 1);
    const int T = b.tile_ptr[size_t(nb)];
    expect(int(b.tile_col.size()) == T && int(b.tile_eptr.size()) == T + 1, "tile arrays", T, ll(b.tile_col.size()));
    expect(b.ents.size() == a.col.size() && b.tile_eptr[size_t(T)] == int(a.col.size()), "entries", ll(b.ents.size()),
           ll(a.col.size()));
    for (int band = 0; band < nb; ++band) {
        const int r0 = band * H, r1 = std::min(a.M, r0 + H);
        const int t0 = b.tile_ptr[size_t(band)], t1 = b.tile_ptr[size_t(band) + 1];
        expect(t1 >= t0, "tile_ptr non-decreasing", band, t1 - t0);
        // the band's entries as (column, row, fp16 bits), and its greedy tile starts
        std::vector<std::tuple<int, int, int>> want;
        for (int r = r0; r < r1; ++r)
            for (int p = a.rp[size_t(r)]; p < a.rp[size_t(r) + 1]; ++p)
                want.emplace_back(a.col[size_t(p)], r, half_bits(a.val[size_t(p)]));
        std::sort(want.begin(), want.end());
        std::vector<int> starts;
        long long end = -1;
        for (const auto& w : want)
            if (std::get<0>(w) >= end) {
                starts.push_back(std::get<0>(w));
                end = std::get<0>(w) + (long long)kBandK;
            }
        expect(int(starts.size()) == t1 - t0, "tile count = greedy count", band, ll(starts.size()));
        if (want.empty()) continue;
        expect(b.tile_eptr[size_t(t0)] == a.rp[size_t(r0)] && b.tile_eptr[size_t(t1)] == a.rp[size_t(r1)],
               "band's tiles cover exactly its entries", band, 0);
        std::vector<std::tuple<int, int, int>> got;
        for (int t = t0; t < t1; ++t) {
            if (t - t0 < int(starts.size())) expect(b.tile_col[size_t(t)] == starts[size_t(t - t0)], "tile start", t, b.tile_col[size_t(t)]);
            expect(b.tile_eptr[size_t(t) + 1] > b.tile_eptr[size_t(t)], "tile not empty", t, 0);
            densest_tile = std::max<ll>(densest_tile, b.tile_eptr[size_t(t) + 1] - b.tile_eptr[size_t(t)]);
            for (int e = b.tile_eptr[size_t(t)]; e < b.tile_eptr[size_t(t) + 1]; ++e) {
                const uint32_t w = b.ents[size_t(e)];
                const int lc = int(w & uint32_t(kBandK - 1)), row = int((w >> kBandColBits) & 127u);
                expect(((w >> (kBandColBits + 7)) & ((1u << (16 - kBandColBits - 7)) - 1u)) == 0u, "unused entry bits", e, w);
                expect(row < r1 - r0, "row within band", e, row);
                got.emplace_back(b.tile_col[size_t(t)] + lc, r0 + row, int(w >> 16));
            }
        }
        expect(got == want, "band entries in (column, row) order with their fp16 values", band, ll(got.size()));
    }
}

// Hybrid split: the dense and residual row views partition every row's entries (each in ascending
// column order, together the row), the dense ones are exactly the entries of tiles holding at
// least min_entries entries, and the band view of the dense part has exactly those tiles.
void check_hybrid_split(const Csr& a, int H, int min_entries) {
    RowViewHost rv;
    rv.rp = a.rp;
    rv.cols = a.col;
    rv.vals = a.val;
    const BandViewHost bv = build_band_view(rv, a.M, H, 2);
    RowViewHost dense, resid;
    split_dense_tiles(rv, bv, a.M, min_entries, 2, dense, resid);
    std::vector<int> want_cols;  // tile columns of the dense tiles, in order
    std::vector<int> want_n;
    long long dense_nnz = 0;
    for (size_t t = 0; t + 1 < bv.tile_eptr.size(); ++t) {
        const int n = bv.tile_eptr[t + 1] - bv.tile_eptr[t];
        if (n >= min_entries) {
            want_cols.push_back(bv.tile_col[t]);
            want_n.push_back(n);
            dense_nnz += n;
        }
    }
    expect(ll(dense.cols.size()) == dense_nnz, "dense part holds the dense tiles' entries", ll(dense.cols.size()), dense_nnz);
    expect(dense.cols.size() + resid.cols.size() == a.col.size(), "the split keeps every entry", ll(dense.cols.size()),
           ll(resid.cols.size()));
    for (int r = 0; r < a.M; ++r) {
        std::vector<std::pair<int, float>> merged;
        for (int p = dense.rp[size_t(r)]; p < dense.rp[size_t(r) + 1]; ++p) {
            expect(p == dense.rp[size_t(r)] || dense.cols[size_t(p)] > dense.cols[size_t(p) - 1], "dense row ascending", r, p);
            merged.push_back({dense.cols[size_t(p)], dense.vals[size_t(p)]});
        }
        for (int p = resid.rp[size_t(r)]; p < resid.rp[size_t(r) + 1]; ++p) {
            expect(p == resid.rp[size_t(r)] || resid.cols[size_t(p)] > resid.cols[size_t(p) - 1], "residual row ascending", r, p);
            merged.push_back({resid.cols[size_t(p)], resid.vals[size_t(p)]});
        }
        std::sort(merged.begin(), merged.end(), [](auto x, auto y) { return x.first < y.first; });
        bool same = merged.size() == size_t(a.rp[size_t(r) + 1] - a.rp[size_t(r)]);
        for (size_t i = 0; same && i < merged.size(); ++i)
            same = merged[i].first == a.col[size_t(a.rp[size_t(r)]) + i] && merged[i].second == a.val[size_t(a.rp[size_t(r)]) + i];
        expect(same, "dense and residual rows together are the row", r, H);
    }
    const BandViewHost dv = build_band_view(dense, a.M, H, 2);
    std::vector<int> got_n;
    for (size_t t = 0; t + 1 < dv.tile_eptr.size(); ++t) got_n.push_back(dv.tile_eptr[t + 1] - dv.tile_eptr[t]);
    expect(dv.tile_col == want_cols && got_n == want_n, "the dense part's band view has exactly the dense tiles",
           ll(dv.tile_col.size()), ll(want_cols.size()));
}

}  // namespace

int main() {
    std::mt19937_64 g(20260923);
    long long n_units_checked = 0, n_bands_checked = 0, n_row_views = 0;
    // work units: short, empty, exactly-unit_nnz and heavy rows
    for (int trial = 0; trial < 40; ++trial) {
        const int M = trial == 0 ? 0 : (trial == 1 ? 1 : 1 + int(g() % 3000));
        std::vector<int> rp(size_t(M) + 1, 0);
        for (int r = 0; r < M; ++r) {
            const int kind = int(g() % 20);
            const int len = kind < 6 ? 0 : kind < 16 ? int(g() % 20) : kind < 18 ? 16 << (g() % 7) : int(g() % 5000);
            rp[size_t(r) + 1] = rp[size_t(r)] + len;
        }
        for (int u : {16, 64, 256, 1024}) {
            check_units(rp, M, u);
            check_units_skip_empty(rp, M, u);
            ++n_units_checked;
        }
    }
    // BAND view: random and banded matrices, several heights, narrow N, empty rows
    for (int trial = 0; trial < 24; ++trial) {
        Csr a;
        if (trial % 3 == 0) {
            a = make_banded(1 + int(g() % 1500), g);
        } else {
            const int M = 1 + int(g() % 500), N = trial % 3 == 1 ? 1 + int(g() % 70) : 1 + int(g() % 5000);
            a = make_csr(M, N, g, [&](int) { return int(g() % 5) == 0 ? 0 : int(g() % 40); });
        }
        for (int H : {1, 37, 64, 112, 128}) {
            check_band(a, H);
            for (int min_entries : {1, 8, 64}) check_hybrid_split(a, H, min_entries);
            ++n_bands_checked;
        }
        check_row_view(a, trial % 2 == 0, trial % 4 < 2 ? 16 : 32, trial % 3 == 0 ? 64 : 16);
        ++n_row_views;
        RowViewHost rv;
        rv.rp = a.rp;
        rv.cols = a.col;
        rv.vals = a.val;
        const BandChoice c = choose_band(rv, a.M);
        const std::set<int> cand = {128, 127, 126, 124, 120, 112, 96, 64, 62, 60, 56, 48, 32};
        expect(cand.count(c.band_rows) == 1, "chosen band height is a candidate", c.band_rows, 0);
        expect(a.col.empty() || c.entries_per_tile >= 1.0, "entries per tile", trial, 0);
    }
    Csr empty;  // M = 0
    empty.rp = {0};
    check_band(empty, 128);
    // The 27-point stencil on 100^3: at 62-row bands each of a band's 9 column windows is exactly 64
    // columns wide (one tile each) and runs at MMA N = 64, which the chooser must prefer.
    int stencil_rows = 0;
    {
        const vcsrmc::CSR st = vcsrmc::gen_stencil27(100, 100, 100, 0);
        RowViewHost rv;
        rv.rp = st.row_ptr;
        rv.cols = st.col;
        rv.vals = st.val;
        const BandChoice c = choose_band(rv, st.M);
        stencil_rows = c.band_rows;
        expect(c.band_rows == 62, "stencil band height", c.band_rows, 62);
        expect(c.entries_per_tile > 150.0, "stencil entries per tile", int(c.entries_per_tile), 150);
    }
    if (failures) {
        std::printf("%d checks failed\n", failures);
        return 1;
    }
    std::printf("OK unit_sets=%lld band_views=%lld row_views=%lld tile_width=%d densest_tile=%lld stencil_band=%d\n",
                n_units_checked, n_bands_checked, n_row_views, kBandK, densest_tile, stencil_rows);
    return 0;
}
