// Host half of the C ABI (vcsrmc.h): CSR, reordering, host format, generators, partition.
#include <algorithm>
#include <climits>
#include <cstring>
#include <string>
#include <vector>

#include "capi_internal.hpp"
#include "vcsrmc/gen.hpp"
#include "vcsrmc/reorder.hpp"

namespace vcsrmc {
namespace {
thread_local int t_last_status = VCSRMC_OK;
thread_local std::string t_last_msg;

void check_csr_arrays(int32_t M, int32_t N, int64_t nnz, const int32_t* row_ptr) {
    if (M < 0 || N < 0 || nnz < 0 || nnz > INT_MAX) throw StatusError(VCSRMC_INVALID_ARG, "bad CSR sizes");
    if (!row_ptr) throw StatusError(VCSRMC_INVALID_ARG, "row_ptr is NULL");
    if (row_ptr[0] != 0 || row_ptr[M] != nnz)
        throw StatusError(VCSRMC_INVALID_ARG, "row_ptr must start at 0 and end at nnz");
    for (int32_t r = 0; r < M; ++r)
        if (row_ptr[r + 1] < row_ptr[r]) throw StatusError(VCSRMC_INVALID_ARG, "row_ptr not monotone");
}
}  // namespace

void set_last_error(int status, const std::string& msg) {
    t_last_status = status;
    t_last_msg = msg;
}

int fail(int status, const std::string& msg) {
    set_last_error(status, msg);
    return status;
}

}  // namespace vcsrmc

using namespace vcsrmc;

VCSRMC_EXPORT int vcsrmc_version(void) { return 1; }

VCSRMC_EXPORT int vcsrmc_last_error(char* buf, size_t len) {
    if (buf && len) {
        const size_t n = std::min(len - 1, t_last_msg.size());
        std::memcpy(buf, t_last_msg.data(), n);
        buf[n] = '\0';
    }
    return t_last_status;
}

VCSRMC_EXPORT int vcsrmc_csr_read_mtx(const char* path, vcsrmc_csr** out) {
    return guarded([&] {
        if (!path || !out) throw StatusError(VCSRMC_INVALID_ARG, "NULL argument");
        auto* h = new vcsrmc_csr;
        try { h->csr = coo_to_csr(read_matrix_market_coo(path)); } catch (...) { delete h; throw; }
        *out = h;
    });
}

VCSRMC_EXPORT int vcsrmc_csr_save(const vcsrmc_csr* h, const char* path) {
    return guarded([&] {
        if (!h || !path) throw StatusError(VCSRMC_INVALID_ARG, "NULL argument");
        save_csr_binary(h->csr, path);
    });
}

VCSRMC_EXPORT int vcsrmc_csr_load(const char* path, vcsrmc_csr** out) {
    return guarded([&] {
        if (!path || !out) throw StatusError(VCSRMC_INVALID_ARG, "NULL argument");
        auto* h = new vcsrmc_csr;
        try { h->csr = load_csr_binary(path); } catch (...) { delete h; throw; }
        *out = h;
    });
}

VCSRMC_EXPORT int vcsrmc_csr_from_coo(int32_t M, int32_t N, int64_t nnz, const int32_t* rows,
                                      const int32_t* cols, const float* vals, vcsrmc_csr** out) {
    return guarded([&] {
        if (!out || M < 0 || N < 0 || nnz < 0 || nnz > INT_MAX || (nnz && (!rows || !cols || !vals)))
            throw StatusError(VCSRMC_INVALID_ARG, "bad COO arguments");
        COO coo;
        coo.M = M;
        coo.N = N;
        coo.rows.assign(rows, rows + nnz);
        coo.cols.assign(cols, cols + nnz);
        coo.vals.assign(vals, vals + nnz);
        auto* h = new vcsrmc_csr;
        try { h->csr = coo_to_csr(coo); } catch (...) { delete h; throw; }
        *out = h;
    });
}

VCSRMC_EXPORT int vcsrmc_csr_from_arrays(int32_t M, int32_t N, int64_t nnz, const int32_t* row_ptr,
                                         const int32_t* col, const float* val, vcsrmc_csr** out) {
    return guarded([&] {
        if (!out) throw StatusError(VCSRMC_INVALID_ARG, "NULL out");
        check_csr_arrays(M, N, nnz, row_ptr);
        if (nnz && (!col || !val)) throw StatusError(VCSRMC_INVALID_ARG, "NULL col/val");
        for (int64_t p = 0; p < nnz; ++p)
            if (col[p] < 0 || col[p] >= N) throw StatusError(VCSRMC_INVALID_ARG, "column index out of range");
        auto* h = new vcsrmc_csr;
        h->csr.M = M;
        h->csr.N = N;
        h->csr.nnz = int(nnz);
        h->csr.row_ptr.assign(row_ptr, row_ptr + M + 1);
        h->csr.col.assign(col, col + nnz);
        h->csr.val.assign(val, val + nnz);
        *out = h;
    });
}

VCSRMC_EXPORT int vcsrmc_csr_view_get(const vcsrmc_csr* h, vcsrmc_csr_view* out) {
    return guarded([&] {
        if (!h || !out) throw StatusError(VCSRMC_INVALID_ARG, "NULL argument");
        out->M = h->csr.M;
        out->N = h->csr.N;
        out->nnz = h->csr.nnz;
        out->row_ptr = h->csr.row_ptr.data();
        out->col = h->csr.col.data();
        out->val = h->csr.val.data();
    });
}

VCSRMC_EXPORT int vcsrmc_csr_row_slice(const vcsrmc_csr* h, int32_t r0, int32_t r1, vcsrmc_csr** out) {
    return guarded([&] {
        if (!h || !out) throw StatusError(VCSRMC_INVALID_ARG, "NULL argument");
        auto* s = new vcsrmc_csr;
        try { s->csr = csr_row_slice(h->csr, r0, r1); } catch (...) { delete s; throw; }
        *out = s;
    });
}

VCSRMC_EXPORT void vcsrmc_csr_free(vcsrmc_csr* h) { delete h; }

VCSRMC_EXPORT int vcsrmc_rcm_column_order(const vcsrmc_csr* h, int32_t* position) {
    return guarded([&] {
        if (!h || !position) throw StatusError(VCSRMC_INVALID_ARG, "NULL argument");
        const std::vector<int> pos = rcm_column_order(h->csr);
        std::copy(pos.begin(), pos.end(), position);
    });
}

VCSRMC_EXPORT int vcsrmc_apply_column_permutation(vcsrmc_csr* h, float* B, int32_t O,
                                                  const int32_t* position) {
    return guarded([&] {
        if (!h || !position || (B && O <= 0)) throw StatusError(VCSRMC_INVALID_ARG, "bad argument");
        const int N = h->csr.N;
        std::vector<int> pos(position, position + N);
        std::vector<char> hit(N, 0);
        for (int v : pos) {
            if (v < 0 || v >= N || hit[v]) throw StatusError(VCSRMC_INVALID_ARG, "position is not a permutation");
            hit[v] = 1;
        }
        std::vector<float> hB;
        if (B) hB.assign(B, B + size_t(N) * size_t(O));
        apply_column_permutation(h->csr, hB, O, pos);
        if (B) std::copy(hB.begin(), hB.end(), B);
    });
}

VCSRMC_EXPORT int vcsrmc_half_scale(const vcsrmc_csr* h, float* scale) {
    return guarded([&] {
        if (!h || !scale) throw StatusError(VCSRMC_INVALID_ARG, "NULL argument");
        *scale = half_scale(h->csr);
    });
}

VCSRMC_EXPORT int vcsrmc_build_host(const vcsrmc_csr* h, int fp32, int segw, int nthreads,
                                    vcsrmc_format** out) {
    return guarded([&] {
        if (!h || !out) throw StatusError(VCSRMC_INVALID_ARG, "NULL argument");
        auto* f = new vcsrmc_format;
        try { f->v = csr_to_vcsr_mc(h->csr, fp32 != 0, segw, nthreads); } catch (...) { delete f; throw; }
        *out = f;
    });
}

VCSRMC_EXPORT int vcsrmc_format_view_get(const vcsrmc_format* f, vcsrmc_format_view* out) {
    return guarded([&] {
        if (!f || !out) throw StatusError(VCSRMC_INVALID_ARG, "NULL argument");
        const VCSRMC& v = f->v;
        out->M = v.M;
        out->N = v.N;
        out->segw = v.segw;
        out->bundle = v.bundle;
        out->num_segments = v.num_segments;
        out->fp32 = v.fp32 ? 1 : 0;
        out->scale = v.scale;
        out->n_groups = int64_t(v.group_depth.size());
        out->n_slots = int64_t(v.lcol.size());
        out->n_items = int64_t(v.item_gbeg.size());
        out->group_ptr = v.group_ptr.data();
        out->group_depth = v.group_depth.data();
        out->group_seg_base = v.group_seg_base.data();
        out->group_rows = v.group_rows.data();
        out->lcol = v.lcol.data();
        out->val = v.val.data();
        out->item_gbeg = v.item_gbeg.data();
        out->item_gend = v.item_gend.data();
    });
}

VCSRMC_EXPORT int vcsrmc_format_from_view(const vcsrmc_format_view* in, vcsrmc_format** out) {
    return guarded([&] {
        if (!in || !out || in->n_groups < 0 || in->n_slots < 0 || in->n_items < 0 || in->M < 0 || in->N < 0)
            throw StatusError(VCSRMC_INVALID_ARG, "bad format view");
        auto need = [](const void* p, int64_t n) {
            if (n > 0 && !p) throw StatusError(VCSRMC_INVALID_ARG, "NULL array in format view");
        };
        need(in->group_ptr, in->n_groups + 1);
        need(in->group_depth, in->n_groups);
        need(in->group_seg_base, in->n_groups);
        need(in->group_rows, 16 * in->n_groups);
        need(in->lcol, in->n_slots);
        need(in->val, in->n_slots);
        need(in->item_gbeg, in->n_items);
        need(in->item_gend, in->n_items);
        auto* f = new vcsrmc_format;
        VCSRMC& v = f->v;
        v.M = in->M;
        v.N = in->N;
        v.segw = in->segw;
        v.bundle = in->bundle;
        v.num_segments = in->num_segments;
        v.fp32 = in->fp32 != 0;
        v.scale = in->scale;
        v.group_ptr.assign(in->group_ptr, in->group_ptr + in->n_groups + 1);
        v.group_depth.assign(in->group_depth, in->group_depth + in->n_groups);
        v.group_seg_base.assign(in->group_seg_base, in->group_seg_base + in->n_groups);
        v.group_rows.assign(in->group_rows, in->group_rows + 16 * in->n_groups);
        v.lcol.assign(in->lcol, in->lcol + in->n_slots);
        v.val.assign(in->val, in->val + in->n_slots);
        v.item_gbeg.assign(in->item_gbeg, in->item_gbeg + in->n_items);
        v.item_gend.assign(in->item_gend, in->item_gend + in->n_items);
        *out = f;
    });
}

VCSRMC_EXPORT void vcsrmc_format_free(vcsrmc_format* f) { delete f; }

VCSRMC_EXPORT int vcsrmc_gen_csr(int kind, int32_t param, uint64_t seed, int nthreads, vcsrmc_csr** out) {
    return guarded([&] {
        if (!out || param <= 0) throw StatusError(VCSRMC_INVALID_ARG, "bad generator arguments");
        auto* h = new vcsrmc_csr;
        try {
            switch (kind) {
                case VCSRMC_GEN_UNIFORM_POISSON:
                    h->csr = gen_uniform_poisson(param, param, 16.0, seed, nthreads);
                    break;
                case VCSRMC_GEN_ZIPF:
                    h->csr = gen_zipf_rows(param, param, 1.8, 8192, 10.0, seed, nthreads);
                    break;
                case VCSRMC_GEN_STENCIL27:
                    h->csr = gen_stencil27(param, param, param, seed, nthreads);
                    break;
                case VCSRMC_GEN_STENCIL27_LINKS:
                    h->csr = gen_stencil27_links(param, 3, seed, nthreads);
                    break;
                case VCSRMC_GEN_RMAT:
                    if (param > 27) throw StatusError(VCSRMC_INVALID_ARG, "R-MAT scale > 27");
                    h->csr = gen_rmat(param, int64_t(1) << (param + 4), 0.57, 0.19, 0.19, seed, nthreads);
                    break;
                default:
                    throw StatusError(VCSRMC_INVALID_ARG, "unknown generator kind");
            }
        } catch (...) {
            delete h;
            throw;
        }
        *out = h;
    });
}

VCSRMC_EXPORT int vcsrmc_gen_dense_host(int64_t rows, int32_t cols, uint64_t seed, float* out, int nthreads) {
    return guarded([&] {
        if (rows < 0 || cols <= 0 || (rows && !out)) throw StatusError(VCSRMC_INVALID_ARG, "bad dense arguments");
        gen_dense(rows, cols, seed, out, nthreads);
    });
}

VCSRMC_EXPORT int vcsrmc_partition_rows(const int32_t* row_ptr, int32_t M, int32_t parts, int32_t* cuts) {
    return guarded([&] {
        if (!row_ptr || !cuts || M < 0 || parts < 1) throw StatusError(VCSRMC_INVALID_ARG, "bad partition arguments");
        const std::vector<int> c = partition_rows(row_ptr, M, parts);
        std::copy(c.begin(), c.end(), cuts);
    });
}

VCSRMC_EXPORT int vcsrmc_partition_rows_weighted(const int32_t* row_ptr, int32_t M, int32_t parts, double row_weight,
                                                 int32_t* cuts) {
    return guarded([&] {
        if (!row_ptr || !cuts || M < 0 || parts < 1) throw StatusError(VCSRMC_INVALID_ARG, "bad partition arguments");
        const std::vector<int> c = partition_rows_weighted(row_ptr, M, parts, row_weight);
        std::copy(c.begin(), c.end(), cuts);
    });
}
