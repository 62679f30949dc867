/* Plain-C use of the library's host entry points (no GPU): read a Matrix Market file, build the
 * VCSR-MC format, walk its arrays, and round-trip the CSR through the binary cache. Prints one
 * line of results; exits non-zero on any failure. Built and run by tests/test_c_abi.py. */
#include <stdio.h>
#include <stdlib.h>

#include "vcsrmc.h"

static int fail(const char* what) {
    char msg[256];
    vcsrmc_last_error(msg, sizeof msg);
    fprintf(stderr, "%s: %s\n", what, msg);
    return 1;
}

int main(int argc, char** argv) {
    if (argc != 3) return 2;
    vcsrmc_csr *A = NULL, *B = NULL;
    vcsrmc_format* F = NULL;
    if (vcsrmc_csr_read_mtx(argv[1], &A) != VCSRMC_OK) return fail("read");
    vcsrmc_csr_view a;
    if (vcsrmc_csr_view_get(A, &a) != VCSRMC_OK) return fail("view");
    if (vcsrmc_build_host(A, /*fp32=*/0, /*segw=*/32, /*nthreads=*/0, &F) != VCSRMC_OK) return fail("build");
    vcsrmc_format_view v;
    if (vcsrmc_format_view_get(F, &v) != VCSRMC_OK) return fail("format view");
    long long filled = 0;
    for (long long s = 0; s < v.n_slots; ++s) filled += v.lcol[s] >= 0;
    if (vcsrmc_csr_save(A, argv[2]) != VCSRMC_OK || vcsrmc_csr_load(argv[2], &B) != VCSRMC_OK) return fail("cache");
    vcsrmc_csr_view b;
    vcsrmc_csr_view_get(B, &b);
    int same = a.M == b.M && a.N == b.N && a.nnz == b.nnz;
    for (long long i = 0; same && i < a.nnz; ++i) same = a.col[i] == b.col[i] && a.val[i] == b.val[i];
    printf("M=%d N=%d nnz=%lld groups=%lld slots=%lld filled=%lld items=%lld scale=%g cache=%s\n", a.M, a.N,
           (long long)a.nnz, (long long)v.n_groups, (long long)v.n_slots, filled, (long long)v.n_items, v.scale,
           same ? "same" : "DIFFERENT");
    vcsrmc_format_free(F);
    vcsrmc_csr_free(A);
    vcsrmc_csr_free(B);
    return same && filled == a.nnz ? 0 : 1;
}
