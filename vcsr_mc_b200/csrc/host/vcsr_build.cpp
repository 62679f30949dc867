// Host VCSR-MC construction (vcsrmc/vcsr_formats.hpp), bit-identical to the reference builder
// (src/vcsr_mc.cu:25-123) and parallel over segments.
//
// What fixes the output bits, and how this file reproduces each part:
//   * entry order inside a (segment, row) pair: ascending local column. For rows whose columns
//     are strictly ascending (every CSR made by coo_to_csr) this is the CSR order. Other rows
//     are rewritten first: a stable partition by segment, then the library's std::sort by
//     local column on each (segment, row) run, which is the sequence and predicate the
//     reference sorts.
//   * row order inside a segment: the reference visits a per-segment std::unordered_map keyed
//     by row, filled in ascending row order, and then std::sort's those rows by descending
//     entry count (not stable). The tie order of equal-count rows therefore comes from the
//     standard library's hash-table iteration order and its introsort. This builder calls the
//     same two library components, with the same key type, the same insertion sequence and the
//     same predicate, so equal-count rows land in the same order. It re-implements neither.
//   * groups, depth, slots and padding; items (runs of <= chunk groups of one segment, then a
//     stable sort by slot count, heaviest first): plain arithmetic, restated below.
#include "vcsrmc/vcsr_formats.hpp"

#include <algorithm>
#include <atomic>
#include <climits>
#include <cmath>
#include <cstdint>
#include <stdexcept>
#include <thread>
#include <unordered_map>
#include <vector>

#include "parallel.hpp"

namespace vcsrmc {

float half_scale_from_absmax(float amax) {
    constexpr float kHalfHeadroom = 60000.0f;           // largest |a| kept after scaling
    constexpr float kHalfMinNormal = 6.103515625e-05f;  // smallest normal fp16
    if (amax > kHalfHeadroom) return amax / kHalfHeadroom;
    if (amax > 0.0f && amax < kHalfMinNormal) return amax / kHalfHeadroom;
    return 1.0f;
}

float half_scale(const CSR& csr) {
    float amax = 0.0f;
    for (float v : csr.val) amax = std::max(amax, std::fabs(v));
    return half_scale_from_absmax(amax);
}

namespace {

// Returns true when every row has strictly ascending columns.
bool rows_strictly_sorted(const CSR& csr, int nthreads) {
    std::atomic<bool> ok{true};
    parallel_for(0, csr.M, nthreads, [&](int64_t r0, int64_t r1) {
        for (int64_t r = r0; r < r1 && ok.load(std::memory_order_relaxed); ++r)
            for (int p = csr.row_ptr[r] + 1; p < csr.row_ptr[r + 1]; ++p)
                if (csr.col[p - 1] >= csr.col[p]) { ok = false; break; }
    });
    return ok.load();
}

// Copy of `csr` whose rows list their entries segment by segment (ascending segment, and
// within a segment in the order the reference's per-pair std::sort by local column leaves).
CSR segment_ordered_copy(const CSR& csr, int segw) {
    CSR out = csr;
    struct Entry { int lcol; float v; int sid; };
    std::vector<Entry> row;
    for (int r = 0; r < csr.M; ++r) {
        const int s = csr.row_ptr[r], e = csr.row_ptr[r + 1];
        row.clear();
        for (int p = s; p < e; ++p) row.push_back({csr.col[p] % segw, csr.val[p], csr.col[p] / segw});
        std::stable_sort(row.begin(), row.end(),
                         [](const Entry& a, const Entry& b) { return a.sid < b.sid; });
        for (size_t i = 0; i < row.size();) {
            size_t j = i;
            while (j < row.size() && row[j].sid == row[i].sid) ++j;
            std::vector<std::pair<int, float>> run;  // (lcol, v), the reference's Entry
            for (size_t k = i; k < j; ++k) run.push_back({row[k].lcol, row[k].v});
            std::sort(run.begin(), run.end(), [](const std::pair<int, float>& a,
                                                 const std::pair<int, float>& b) {
                return a.first < b.first;
            });
            for (size_t k = i; k < j; ++k) {
                out.col[s + k] = row[i].sid * segw + run[k - i].first;
                out.val[s + k] = run[k - i].second;
            }
            i = j;
        }
    }
    return out;
}

struct Pair {       // one (segment, row) pair: the row's entries in that segment
    int row;
    int count;      // entries
    int64_t first;  // CSR position of the first entry
};

}  // namespace

VCSRMC csr_to_vcsr_mc(const CSR& in, bool fp32, int segw, int nthreads) {
    if (segw != 16 && segw != 32 && segw != 48 && segw != 64)
        throw std::runtime_error("vcsr_mc supports segw in {16, 32, 48, 64}");
    if (in.M < 0 || in.N < 0 || int64_t(in.row_ptr.size()) != int64_t(in.M) + 1 ||
        int64_t(in.col.size()) != in.nnz || int64_t(in.val.size()) != in.nnz)
        throw std::runtime_error("inconsistent CSR");
    nthreads = resolve_threads(nthreads);
    constexpr int bundle = 16;

    VCSRMC V;
    V.M = in.M;
    V.N = in.N;
    V.segw = segw;
    V.bundle = bundle;
    V.fp32 = fp32;
    V.scale = fp32 ? 1.0f : half_scale(in);
    const float inv_scale = 1.0f / V.scale;
    const int S = (in.N + segw - 1) / segw;
    V.num_segments = S;

    CSR sorted_copy;
    const bool sorted = rows_strictly_sorted(in, nthreads);
    if (!sorted) sorted_copy = segment_ordered_copy(in, segw);
    const CSR& csr = sorted ? in : sorted_copy;

    // ---- (segment, row) pairs, bucketed by segment in ascending row order -------------------
    const int M = csr.M;
    const int nblk = std::max(1, std::min(nthreads * 4, M));
    std::vector<int64_t> blk_row(nblk + 1);
    for (int b = 0; b <= nblk; ++b) blk_row[b] = int64_t(M) * b / nblk;
    // per block, per segment pair counts -> stable counting sort
    std::vector<std::vector<int>> blk_seg_count(nblk);
    parallel_for(0, nblk, nthreads, [&](int64_t b0, int64_t b1) {
        for (int64_t b = b0; b < b1; ++b) {
            std::vector<int>& cnt = blk_seg_count[b];
            cnt.assign(S, 0);
            for (int64_t r = blk_row[b]; r < blk_row[b + 1]; ++r) {
                int prev = -1;
                for (int p = csr.row_ptr[r]; p < csr.row_ptr[r + 1]; ++p) {
                    const int sid = csr.col[p] / segw;
                    if (sid != prev) { ++cnt[sid]; prev = sid; }
                }
            }
        }
    });
    std::vector<int64_t> seg_off(size_t(S) + 1, 0);
    for (int s = 0; s < S; ++s) {
        int64_t t = 0;
        for (int b = 0; b < nblk; ++b) t += blk_seg_count[b][s];
        seg_off[s + 1] = seg_off[s] + t;
    }
    const int64_t npairs = seg_off[S];
    std::vector<Pair> pairs(npairs);
    {
        // cursor of block b in segment s = seg_off[s] + sum of counts of blocks < b
        std::vector<std::vector<int64_t>> cursor(nblk);
        for (int b = 0; b < nblk; ++b) cursor[b].resize(S);
        parallel_for(0, S, nthreads, [&](int64_t s0, int64_t s1) {
            for (int64_t s = s0; s < s1; ++s) {
                int64_t c = seg_off[s];
                for (int b = 0; b < nblk; ++b) { cursor[b][s] = c; c += blk_seg_count[b][s]; }
            }
        });
        blk_seg_count.clear();
        blk_seg_count.shrink_to_fit();
        parallel_for(0, nblk, nthreads, [&](int64_t b0, int64_t b1) {
            for (int64_t b = b0; b < b1; ++b) {
                std::vector<int64_t>& cur = cursor[b];
                for (int64_t r = blk_row[b]; r < blk_row[b + 1]; ++r) {
                    const int e = csr.row_ptr[r + 1];
                    for (int p = csr.row_ptr[r]; p < e;) {
                        const int sid = csr.col[p] / segw;
                        int q = p + 1;
                        while (q < e && csr.col[q] / segw == sid) ++q;
                        pairs[cur[sid]++] = Pair{int(r), q - p, p};
                        p = q;
                    }
                }
            }
        });
    }

    // ---- per segment: row order, groups, slots ----------------------------------------------
    std::vector<int64_t> seg_groups(size_t(S) + 1, 0), seg_slots(size_t(S) + 1, 0);
    parallel_for_dynamic(0, S, nthreads, 64, [&](int64_t s0, int64_t s1) {
        std::vector<Pair> ordered;
        for (int64_t s = s0; s < s1; ++s) {
            Pair* P = pairs.data() + seg_off[s];
            const int64_t n = seg_off[s + 1] - seg_off[s];
            if (n == 0) continue;
            // iteration order of the standard hash map filled in ascending row order
            std::unordered_map<int, int> by_row;
            for (int64_t i = 0; i < n; ++i) by_row.emplace(P[i].row, int(i));
            ordered.clear();
            for (const auto& kv : by_row) ordered.push_back(P[kv.second]);
            std::sort(ordered.begin(), ordered.end(),
                      [](const Pair& a, const Pair& b) { return a.count > b.count; });
            std::copy(ordered.begin(), ordered.end(), P);
            int64_t g = 0, slots = 0;
            for (int64_t i = 0; i < n; i += bundle) {
                int depth = 0;
                for (int64_t j = i; j < std::min(n, i + bundle); ++j) depth = std::max(depth, P[j].count);
                ++g;
                slots += int64_t(depth) * bundle;
            }
            seg_groups[s + 1] = g;
            seg_slots[s + 1] = slots;
        }
    });
    for (int s = 0; s < S; ++s) {
        seg_groups[s + 1] += seg_groups[s];
        seg_slots[s + 1] += seg_slots[s];
    }
    const int64_t G = seg_groups[S];
    const int64_t total_slots = seg_slots[S];
    if (total_slots > INT_MAX || G * bundle > INT_MAX)
        throw std::runtime_error("VCSR slot count exceeds the format's 32-bit offsets");

    V.group_ptr.resize(size_t(G) + 1);
    V.group_depth.resize(G);
    V.group_seg_base.resize(G);
    V.group_rows.resize(size_t(G) * bundle);
    V.lcol.resize(total_slots);
    V.val.resize(total_slots);
    parallel_for_dynamic(0, S, nthreads, 64, [&](int64_t s0, int64_t s1) {
        for (int64_t s = s0; s < s1; ++s) {
            const Pair* P = pairs.data() + seg_off[s];
            const int64_t n = seg_off[s + 1] - seg_off[s];
            int64_t g = seg_groups[s];
            int64_t slot = seg_slots[s];
            for (int64_t i = 0; i < n; i += bundle, ++g) {
                const int64_t end = std::min(n, i + bundle);
                int depth = 0;
                for (int64_t j = i; j < end; ++j) depth = std::max(depth, P[j].count);
                V.group_ptr[g] = int(slot);
                V.group_depth[g] = depth;
                V.group_seg_base[g] = int(s) * segw;
                for (int lane = 0; lane < bundle; ++lane)
                    V.group_rows[size_t(g) * bundle + lane] = i + lane < n ? P[i + lane].row : -1;
                for (int d = 0; d < depth; ++d)
                    for (int lane = 0; lane < bundle; ++lane, ++slot) {
                        const int64_t j = i + lane;
                        if (j < n && d < P[j].count) {
                            const int64_t p = P[j].first + d;
                            V.lcol[slot] = csr.col[p] % segw;
                            V.val[slot] = csr.val[p] * inv_scale;
                        } else {
                            V.lcol[slot] = -1;
                            V.val[slot] = 0.f;
                        }
                    }
            }
        }
    });
    V.group_ptr[G] = int(total_slots);

    // ---- work items: runs of <= chunk groups of one segment, heaviest first (stable) -------
    const int Gi = int(G);
    const int chunk = std::max(1, std::min(32, Gi / 4096));
    struct Item { int b, e; long long work; };
    std::vector<Item> items;
    items.reserve(size_t(Gi / chunk) + size_t(S) + 1);
    for (int g = 0; g < Gi;) {
        int e = g;
        while (e < Gi && e - g < chunk && V.group_seg_base[e] == V.group_seg_base[g]) ++e;
        items.push_back({g, e, (long long)V.group_ptr[e] - V.group_ptr[g]});
        g = e;
    }
    std::stable_sort(items.begin(), items.end(),
                     [](const Item& a, const Item& b) { return a.work > b.work; });
    V.item_gbeg.resize(items.size());
    V.item_gend.resize(items.size());
    for (size_t i = 0; i < items.size(); ++i) {
        V.item_gbeg[i] = items[i].b;
        V.item_gend[i] = items[i].e;
    }
    return V;
}

}  // namespace vcsrmc
