// Reverse Cuthill-McKee column order (vcsrmc/reorder.hpp).
//
// The reference's permutation (include/reorder.hpp:17-77) is defined by the exact steps of its
// BFS: roots in ascending degree order (stable), and each vertex's newly seen neighbours put in
// ascending degree order with std::sort before they are queued. std::sort is not stable, so
// the neighbour step calls the same library sort with the same ordering predicate on the same
// input sequence (neighbours in ascending column order); any other sort could order
// equal-degree neighbours differently and change the permutation.
#include "vcsrmc/reorder.hpp"

#include <algorithm>
#include <stdexcept>
#include <vector>

namespace vcsrmc {

std::vector<int> rcm_column_order(const CSR& csr) {
    const int n = csr.N;
    // Symmetrised pattern on the column set: row r < n is identified with column r; an entry
    // (r, c) links r and c, and for r >= n it contributes a self-link on c.
    std::vector<int> offs(size_t(n) + 1, 0);
    for (int r = 0; r < csr.M; ++r)
        for (int p = csr.row_ptr[r]; p < csr.row_ptr[r + 1]; ++p) {
            if (r < n) ++offs[size_t(r) + 1];
            ++offs[size_t(csr.col[p]) + 1];
        }
    for (int i = 0; i < n; ++i) offs[i + 1] += offs[i];
    std::vector<int> nbr(offs[n]);
    {
        std::vector<int> fill(offs.begin(), offs.end() - 1);
        for (int r = 0; r < csr.M; ++r)
            for (int p = csr.row_ptr[r]; p < csr.row_ptr[r + 1]; ++p) {
                const int c = csr.col[p];
                if (r < n) nbr[fill[r]++] = c;
                nbr[fill[c]++] = r < n ? r : c;
            }
    }
    // Sorted, de-duplicated neighbour lists; degree = distinct neighbours (self included).
    std::vector<int> degree(n);
    for (int i = 0; i < n; ++i) {
        auto b = nbr.begin() + offs[i], e = nbr.begin() + offs[i + 1];
        std::sort(b, e);
        degree[i] = int(std::unique(b, e) - b);
    }

    std::vector<int> roots(n);
    for (int i = 0; i < n; ++i) roots[i] = i;
    std::stable_sort(roots.begin(), roots.end(),
                     [&](int a, int b) { return degree[a] < degree[b]; });

    std::vector<char> seen(n, 0);
    std::vector<int> order;  // BFS order; also serves as the FIFO queue (head index)
    order.reserve(n);
    std::vector<int> fresh;
    for (int root : roots) {
        if (seen[root]) continue;
        seen[root] = 1;
        size_t head = order.size();
        order.push_back(root);
        while (head < order.size()) {
            const int v = order[head++];
            fresh.clear();
            for (int k = offs[v]; k < offs[v] + degree[v]; ++k) {
                const int u = nbr[k];
                if (!seen[u]) { seen[u] = 1; fresh.push_back(u); }
            }
            std::sort(fresh.begin(), fresh.end(),
                      [&](int a, int b) { return degree[a] < degree[b]; });
            order.insert(order.end(), fresh.begin(), fresh.end());
        }
    }
    std::vector<int> position(n);
    for (int i = 0; i < n; ++i) position[order[n - 1 - i]] = i;
    return position;
}

void apply_column_permutation(CSR& csr, std::vector<float>& hB, int O,
                              const std::vector<int>& position) {
    if (int(position.size()) != csr.N) throw std::runtime_error("permutation size != N");
    for (int& c : csr.col) c = position[c];
    std::vector<std::pair<int, float>> tmp;
    for (int r = 0; r < csr.M; ++r) {
        const int s = csr.row_ptr[r], e = csr.row_ptr[r + 1];
        if (e - s < 2) continue;
        tmp.resize(e - s);
        for (int i = s; i < e; ++i) tmp[i - s] = {csr.col[i], csr.val[i]};
        // columns are distinct within a row, so the sorted order is unique
        std::sort(tmp.begin(), tmp.end(),
                  [](const auto& a, const auto& b) { return a.first < b.first; });
        for (int i = s; i < e; ++i) { csr.col[i] = tmp[i - s].first; csr.val[i] = tmp[i - s].second; }
    }
    if (hB.empty()) return;
    std::vector<float> moved(hB.size());
    for (int old_row = 0; old_row < csr.N; ++old_row)
        std::copy(hB.begin() + size_t(old_row) * O, hB.begin() + size_t(old_row + 1) * O,
                  moved.begin() + size_t(position[old_row]) * O);
    hB.swap(moved);
}

}  // namespace vcsrmc
