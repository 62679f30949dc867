/* TEST INFRASTRUCTURE — ORACLE ONLY. A plain-C CPU restatement of the reference's hot path
 * (MuuSeoTia/VCSR_MC). Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg
 * may load liboracle.so, and only as the checker; the product never links or calls it.
 *
 * Parity is pinned: tests/test_oracle.py checks every function here against the reference's
 * own code compiled from its sources (oracle/_ref, see ref_shim.cpp) and against the committed
 * golden vectors in tests/golden/ that were produced by that reference build.
 */
#ifndef VCSRMC_ORACLE_H
#define VCSRMC_ORACLE_H
#include <stdint.h>

typedef struct {
    int32_t M, N, segw, bundle, num_segments, fp32;
    float scale;
    int64_t n_groups, n_slots, n_items;
    int32_t *group_ptr, *group_depth, *group_seg_base, *group_rows, *lcol;
    float* val;
    int32_t *item_gbeg, *item_gend;
} oracle_vcsr;

/* fp64 CSR SpMM, src/main.cpp:202-207: out[r*O+k] = sum_p double(val[p]) * B[col[p]*O+k].
 * abs_out (may be NULL) gets sum_p |val[p] * B[col[p]*O+k]| for error bounds. */
void oracle_spmm_fp64(int32_t M, const int32_t* row_ptr, const int32_t* col, const float* val, const float* B,
                      int32_t O, double* out, double* abs_out, int nthreads);
/* Same, for the listed rows only; out/abs_out are nrows x O. */
void oracle_spmm_fp64_rows(const int32_t* row_ptr, const int32_t* col, const float* val, const float* B, int32_t O,
                           const int32_t* rows, int32_t nrows, double* out, double* abs_out);

/* src/vcsr_mc.cu:14-22 */
float oracle_half_scale(int64_t nnz, const float* val);

/* src/vcsr_mc.cu:25-123 with one deliberate difference: rows with equal entry counts in a
 * segment are ordered by ascending row id (the reference's order among them comes from its
 * standard library's hash table and unstable sort). Returns 0, or 1 for an unsupported segw. */
int oracle_build_vcsr(int32_t M, int32_t N, const int32_t* row_ptr, const int32_t* col, const float* val,
                      int fp32, int segw, oracle_vcsr* out);
void oracle_vcsr_free(oracle_vcsr* v);

/* Rewrites group_rows/lcol/val of a VCSR (any tie order) into the canonical tie order above,
 * in place. group_ptr, group_depth and group_seg_base are unchanged by construction. */
void oracle_canonicalize_vcsr(int64_t n_groups, int32_t segw, const int32_t* group_ptr, const int32_t* group_depth,
                              const int32_t* group_seg_base, int32_t* group_rows, int32_t* lcol, float* val);

/* include/reorder.hpp:17-77, with stable sorts wherever the reference sorts. Equal to the
 * reference whenever no vertex has more than 16 newly seen neighbours of equal degree
 * (below that size the reference's library sort is an insertion sort, hence stable). */
void oracle_rcm_column_order(int32_t M, int32_t N, const int32_t* row_ptr, const int32_t* col, int32_t* position);

/* include/reorder.hpp:82-108, in place; B (N x O, may be NULL) is permuted by rows. */
void oracle_apply_column_permutation(int32_t M, int32_t N, const int32_t* row_ptr, int32_t* col, float* val,
                                     float* B, int32_t O, const int32_t* position);

#endif
