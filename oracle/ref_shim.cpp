// TEST INFRASTRUCTURE — ORACLE ONLY. Never linked into, loaded by or called from the
// product library (vcsr_mc_b200). Only tests/, __graft_entry__.smoke() and the
// cpu_baseline / --impl reference legs of bench.py may load the library built from it.
//
// Exposes the reference implementation itself (MuuSeoTia/VCSR_MC), compiled from its own
// sources where they lie, behind a plain C ABI so the tests can pin the oracle and the
// product against it:
//   * include/mmio.hpp:19-75   read_matrix_market_coo
//   * include/csr.hpp:16-41    coo_to_csr
//   * include/reorder.hpp:17-108 rcm_column_order / apply_column_permutation
//   * src/vcsr_mc.cu:13-123    half_scale / csr_to_vcsr_mc (extracted to _ref/ by the
//                               Makefile; the device half of that file is not compiled)
//   * src/main.cpp:202-207     the fp64 CPU CSR SpMM loop (extracted likewise)
// Nothing from the reference is copied into this repository: the Makefile reads the
// files under the reference checkout at build time and writes only into oracle/_ref/.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <numeric>
#include <stdexcept>
#include <string>
#include <thread>
#include <unordered_map>
#include <vector>

#include "mmio.hpp"
#include "csr.hpp"
#include "reorder.hpp"
#include "vcsr_formats.hpp"

#include "vcsr_mc_host.inc"

#define REF_API extern "C" __attribute__((visibility("default")))

namespace {

void set_err(char* err, size_t len, const char* msg) {
    if (err && len) { std::snprintf(err, len, "%s", msg); }
}

CSR make_csr(int M, int N, int64_t nnz, const int* row_ptr, const int* col, const float* val) {
    CSR c;
    c.M = M; c.N = N; c.nnz = int(nnz);
    c.row_ptr.assign(row_ptr, row_ptr + M + 1);
    c.col.assign(col, col + nnz);
    c.val.assign(val, val + nnz);
    return c;
}

}  // namespace

extern "C" {

typedef struct {
    int32_t M, N, segw, bundle, num_segments, fp32;
    float scale;
    int64_t n_groups, n_slots, n_items;
    const int32_t *group_ptr, *group_depth, *group_seg_base, *group_rows, *lcol;
    const float* val;
    const int32_t *item_gbeg, *item_gend;
    void* impl;
} ref_vcsr_view;

typedef struct {
    int32_t M, N;
    int64_t nnz;
    const int32_t *row_ptr, *col;
    const float* val;
    void* impl;
} ref_csr_view;

}  // extern "C"

static void fill_csr_view(CSR* c, ref_csr_view* out) {
    out->M = c->M; out->N = c->N; out->nnz = c->nnz;
    out->row_ptr = c->row_ptr.data(); out->col = c->col.data(); out->val = c->val.data();
    out->impl = c;
}

REF_API int ref_build_vcsr(int M, int N, int64_t nnz, const int* row_ptr, const int* col,
                           const float* val, int fp32, int segw, ref_vcsr_view* out,
                           char* err, size_t errlen) {
    try {
        CSR c = make_csr(M, N, nnz, row_ptr, col, val);
        VCSRMC* V = new VCSRMC(csr_to_vcsr_mc(c, fp32 != 0, segw));
        out->M = V->M; out->N = V->N; out->segw = V->segw; out->bundle = V->bundle;
        out->num_segments = V->num_segments; out->fp32 = V->fp32 ? 1 : 0; out->scale = V->scale;
        out->n_groups = (int64_t)V->group_depth.size();
        out->n_slots = (int64_t)V->lcol.size();
        out->n_items = (int64_t)V->item_gbeg.size();
        out->group_ptr = V->group_ptr.data(); out->group_depth = V->group_depth.data();
        out->group_seg_base = V->group_seg_base.data(); out->group_rows = V->group_rows.data();
        out->lcol = V->lcol.data(); out->val = V->val.data();
        out->item_gbeg = V->item_gbeg.data(); out->item_gend = V->item_gend.data();
        out->impl = V;
        return 0;
    } catch (const std::exception& e) {
        set_err(err, errlen, e.what());
        return 1;
    }
}

REF_API void ref_vcsr_free(ref_vcsr_view* v) {
    if (v && v->impl) { delete static_cast<VCSRMC*>(v->impl); v->impl = nullptr; }
}

REF_API float ref_half_scale(int64_t nnz, const float* val) {
    CSR c;
    c.val.assign(val, val + nnz);
    return half_scale(c);
}

REF_API int ref_read_mtx(const char* path, ref_csr_view* out, char* err, size_t errlen) {
    try {
        CSR* c = new CSR(coo_to_csr(read_matrix_market_coo(path)));
        fill_csr_view(c, out);
        return 0;
    } catch (const std::exception& e) {
        set_err(err, errlen, e.what());
        return 1;
    }
}

REF_API int ref_coo_to_csr(int M, int N, int64_t nnz, const int* rows, const int* cols,
                           const float* vals, ref_csr_view* out, char* err, size_t errlen) {
    try {
        COO coo;
        coo.M = M; coo.N = N;
        coo.rows.assign(rows, rows + nnz);
        coo.cols.assign(cols, cols + nnz);
        coo.vals.assign(vals, vals + nnz);
        CSR* c = new CSR(coo_to_csr(coo));
        fill_csr_view(c, out);
        return 0;
    } catch (const std::exception& e) {
        set_err(err, errlen, e.what());
        return 1;
    }
}

REF_API void ref_csr_free(ref_csr_view* v) {
    if (v && v->impl) { delete static_cast<CSR*>(v->impl); v->impl = nullptr; }
}

REF_API int ref_rcm_column_order(int M, int N, int64_t nnz, const int* row_ptr, const int* col,
                                 int* position_out) {
    CSR c;
    c.M = M; c.N = N; c.nnz = int(nnz);
    c.row_ptr.assign(row_ptr, row_ptr + M + 1);
    c.col.assign(col, col + nnz);
    c.val.assign(nnz, 0.f);
    std::vector<int> pos = rcm_column_order(c);
    std::copy(pos.begin(), pos.end(), position_out);
    return 0;
}

// In place on col/val (and on B when non-null, an N x O fp32 row-major buffer).
REF_API int ref_apply_column_permutation(int M, int N, int64_t nnz, const int* row_ptr, int* col,
                                         float* val, float* B, int O, const int* position) {
    CSR c = make_csr(M, N, nnz, row_ptr, col, val);
    std::vector<float> hB;
    if (B) hB.assign(B, B + size_t(N) * O);
    std::vector<int> pos(position, position + N);
    apply_column_permutation(c, hB, O, pos);
    std::copy(c.col.begin(), c.col.end(), col);
    std::copy(c.val.begin(), c.val.end(), val);
    if (B) std::copy(hB.begin(), hB.end(), B);
    return 0;
}

// ---- The reference's fp64 CPU SpMM (src/main.cpp:202-207) --------------------------------
//
// One slice = a contiguous block of rows held as its own CSR, with the slice's own output
// vector. The loop body is the reference's, verbatim, compiled from its source; the local
// names below (csr, hB, O, reference) are the ones that loop uses.
namespace {
struct SpmmSlice {
    CSR csr;
    std::vector<double> out;
    int64_t row0 = 0;
};
struct SpmmCtx {
    std::vector<float> B;
    int O = 0;
    std::vector<SpmmSlice> slices;
};

void run_reference_loop(const CSR& csr, const std::vector<float>& hB, int O,
                        std::vector<double>& reference) {
    std::fill(reference.begin(), reference.end(), 0.0);
#include "cpu_spmm.inc"
}
}  // namespace

REF_API void* ref_spmm_ctx_create(int M, int N, int64_t nnz, const int* row_ptr, const int* col,
                                  const float* val, const float* B, int O, int nslices) {
    (void)nnz;
    SpmmCtx* ctx = new SpmmCtx;
    ctx->B.assign(B, B + size_t(N) * O);
    ctx->O = O;
    if (nslices < 1) nslices = 1;
    if (nslices > M && M > 0) nslices = M;
    const int64_t total = row_ptr[M] - row_ptr[0];
    int r = 0;
    for (int s = 0; s < nslices; ++s) {
        // cut at the first row whose prefix reaches the s+1-th share of the nonzeros
        int r1 = M;
        if (s + 1 < nslices) {
            const int64_t target = row_ptr[0] + (total * (s + 1)) / nslices;
            r1 = int(std::lower_bound(row_ptr + r, row_ptr + M + 1, (int)target) - row_ptr);
            r1 = std::max(r1, r);
            r1 = std::min(r1, M);
        }
        SpmmSlice sl;
        sl.row0 = r;
        sl.csr.M = r1 - r; sl.csr.N = N;
        sl.csr.row_ptr.resize(r1 - r + 1);
        for (int i = r; i <= r1; ++i) sl.csr.row_ptr[i - r] = row_ptr[i] - row_ptr[r];
        sl.csr.nnz = sl.csr.row_ptr.back();
        sl.csr.col.assign(col + row_ptr[r], col + row_ptr[r1]);
        sl.csr.val.assign(val + row_ptr[r], val + row_ptr[r1]);
        sl.out.assign(size_t(r1 - r) * O, 0.0);
        ctx->slices.push_back(std::move(sl));
        r = r1;
    }
    return ctx;
}

// Runs every slice (each on its own thread when there is more than one) and, when out is
// non-null, gathers the M x O fp64 result into it.
REF_API void ref_spmm_ctx_run(void* vctx, double* out) {
    SpmmCtx* ctx = static_cast<SpmmCtx*>(vctx);
    if (ctx->slices.size() == 1) {
        SpmmSlice& s = ctx->slices[0];
        run_reference_loop(s.csr, ctx->B, ctx->O, s.out);
    } else {
        std::vector<std::thread> th;
        for (SpmmSlice& s : ctx->slices)
            th.emplace_back([&s, ctx] { run_reference_loop(s.csr, ctx->B, ctx->O, s.out); });
        for (auto& t : th) t.join();
    }
    if (out) {
        for (const SpmmSlice& s : ctx->slices)
            std::copy(s.out.begin(), s.out.end(), out + size_t(s.row0) * ctx->O);
    }
}

REF_API void ref_spmm_ctx_free(void* vctx) { delete static_cast<SpmmCtx*>(vctx); }
