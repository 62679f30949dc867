/* vcsrmc.h - C ABI of the B200 VCSR-MC SpMM library (libvcsrmc.so).
 *
 * C (M x O, fp32, row-major) += A (M x N, sparse CSR) * B (N x O, dense, row-major).
 *
 * This is the boundary a host program binds (ctypes, cgo, JNI, a C++ driver). It replaces the
 * reference's in-process C++ interface of MuuSeoTia/VCSR_MC:
 *   include/vcsr_formats.hpp:11,22-26  half_scale, csr_to_vcsr_mc, upload_vcsr_mc_device,
 *                                      run_vcsr_mc_spmm_gpu, destroy_vcsr_mc_device
 *   include/mmio.hpp:19, include/csr.hpp:16, include/reorder.hpp:17,82  host loaders/reorder
 * Differences, all deliberate:
 *   - no exceptions and no exit(): every call returns a status (VCSRMC_OK = 0) and
 *     vcsrmc_last_error() gives the message of the calling thread's last failure;
 *   - the device copy of a format is a handle (one per format and device), not a set of
 *     module-global pointers, so several formats and devices can be live at once;
 *   - vcsrmc_spmm is asynchronous on the caller's stream; vcsrmc_spmm_timed is the blocking,
 *     event-timed form of run_vcsr_mc_spmm_gpu;
 *   - B and C offsets are 64-bit (ldb, ldc), so N*O and M*O may exceed INT_MAX.
 * All pointers are plain host or device addresses; `stream` is a cudaStream_t (NULL = the
 * legacy default stream). Handles may be used from several threads, one stream at a time.
 */
#ifndef VCSRMC_H
#define VCSRMC_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes -------------------------------------------------------------------- */
#define VCSRMC_OK 0
#define VCSRMC_INVALID_ARG 1  /* bad size/flag, e.g. segw not in {16,32,48,64}            */
#define VCSRMC_CUDA_ERR 2     /* a CUDA runtime/driver call failed                        */
#define VCSRMC_OOM 3          /* host or device allocation failed                         */
#define VCSRMC_TIMEOUT 4      /* a bounded device-side wait expired (see device_status)   */
#define VCSRMC_IO_ERR 5       /* file could not be opened/read                            */
#define VCSRMC_FORMAT_ERR 6   /* malformed Matrix Market data, duplicate coordinates, ... */
#define VCSRMC_INTERNAL 7

/* ---- element types ------------------------------------------------------------------- */
#define VCSRMC_F32 0
#define VCSRMC_F16 1

/* ---- execution plans (vcsrmc_upload_ex / vcsrmc_spmm_ex) ------------------------------
 * SEGMENT: the reference's dataflow (src/vcsr_mc.cu:143-329): per work item, stage the B
 *          segment once, multiply every 16-row group, add it into C with reductions.
 * ROWS:    row-stationary over the format's row view (built at upload): each C row is
 *          accumulated in registers from gathered B rows and stored once.
 * BAND:    FP16 format only: bands of <= 128 rows, tiles of 64 columns multiplied on the tensor
 *          cores into one accumulator per band, C stored once. For matrices whose rows touch
 *          few column windows (stencils, banded or reordered matrices).
 * HYBRID:  FP16 format only: the band tiles that hold at least 64 entries run as BAND (C written
 *          once), every other entry then runs on ROWS, added into C. For matrices with dense
 *          blocks and scattered entries.
 * AUTO:    the first resident layout of BAND (fp16 B only), HYBRID (fp16 B only), ROWS,
 *          SEGMENT, BAND, HYBRID.                                                           */
#define VCSRMC_PLAN_AUTO 0
#define VCSRMC_PLAN_SEGMENT 1
#define VCSRMC_PLAN_ROWS 2
#define VCSRMC_PLAN_BAND 3
#define VCSRMC_PLAN_HYBRID 4

/* ---- synthetic configurations (vcsrmc_gen_csr) ---------------------------------------- */
#define VCSRMC_GEN_UNIFORM_POISSON 1 /* param: M = N; mean row length 16                   */
#define VCSRMC_GEN_ZIPF 2            /* param: M = N; Zipf(1.8) lengths, mean 10, cap 8192  */
#define VCSRMC_GEN_STENCIL27 3       /* param: grid edge n (n^3 rows)                       */
#define VCSRMC_GEN_RMAT 4            /* param: scale (2^scale rows); 2^(scale+4) samples     */
#define VCSRMC_GEN_STENCIL27_LINKS 5 /* param: grid edge n; the 27-point stencil plus 3 random
                                        long-range links per row (no reference counterpart)  */

typedef struct vcsrmc_csr vcsrmc_csr;                     /* host CSR                    */
typedef struct vcsrmc_format vcsrmc_format;               /* host VCSR-MC format         */
typedef struct vcsrmc_device_format vcsrmc_device_format; /* VCSR-MC format on one GPU   */

typedef struct {
    int32_t M, N;
    int64_t nnz;
    const int32_t* row_ptr; /* M + 1 */
    const int32_t* col;     /* nnz   */
    const float* val;       /* nnz   */
} vcsrmc_csr_view;

/* Read-only view of a host format; fields and array contents are those of the reference's
 * struct VCSRMC (include/vcsr_formats.hpp:14-21). */
typedef struct {
    int32_t M, N, segw, bundle, num_segments, fp32;
    float scale;
    int64_t n_groups, n_slots, n_items;
    const int32_t* group_ptr;      /* n_groups + 1 slot offsets          */
    const int32_t* group_depth;    /* n_groups                           */
    const int32_t* group_seg_base; /* n_groups, first column of segment  */
    const int32_t* group_rows;     /* 16 * n_groups, -1 = padding lane   */
    const int32_t* lcol;           /* n_slots, -1 = padding slot         */
    const float* val;              /* n_slots (divided by scale if FP16) */
    const int32_t* item_gbeg;      /* n_items                            */
    const int32_t* item_gend;      /* n_items                            */
} vcsrmc_format_view;

/* ---- library -------------------------------------------------------------------------- */
int vcsrmc_version(void);
/* Copies the calling thread's last error message (NUL-terminated) and returns its status. */
int vcsrmc_last_error(char* buf, size_t len);

/* ---- host CSR: include/mmio.hpp:19-75 read_matrix_market_coo + include/csr.hpp:16-41
 *      coo_to_csr (the two are one call here, as in src/main.cpp:150) ------------------- */
int vcsrmc_csr_read_mtx(const char* path, vcsrmc_csr** out);
/* coo_to_csr on caller arrays: counting sort by row, ascending columns, duplicates rejected. */
int vcsrmc_csr_from_coo(int32_t M, int32_t N, int64_t nnz, const int32_t* rows,
                        const int32_t* cols, const float* vals, vcsrmc_csr** out);
/* Copies a CSR given as arrays (no reordering; rows may be unsorted). */
int vcsrmc_csr_from_arrays(int32_t M, int32_t N, int64_t nnz, const int32_t* row_ptr,
                           const int32_t* col, const float* val, vcsrmc_csr** out);
int vcsrmc_csr_view_get(const vcsrmc_csr* csr, vcsrmc_csr_view* out);
/* Rows [r0, r1) as a CSR of their own (row ids rebased to 0). */
int vcsrmc_csr_row_slice(const vcsrmc_csr* csr, int32_t r0, int32_t r1, vcsrmc_csr** out);
void vcsrmc_csr_free(vcsrmc_csr* csr);
/* Binary CSR cache: a 32-byte header ("VCSRMC1\0", int64 M, N, nnz), then row_ptr (int32,
 * M + 1), col (int32, nnz), val (fp32, nnz), little-endian. Loading validates sizes, row_ptr
 * and the column range (IO_ERR for an unreadable file, FORMAT_ERR for a malformed one). */
int vcsrmc_csr_save(const vcsrmc_csr* csr, const char* path);
int vcsrmc_csr_load(const char* path, vcsrmc_csr** out);

/* ---- reordering: include/reorder.hpp:17-77 rcm_column_order, :82-108
 *      apply_column_permutation ---------------------------------------------------------- */
int vcsrmc_rcm_column_order(const vcsrmc_csr* csr, int32_t* position /* N */);
/* B: N x O fp32 row-major host buffer permuted in place (may be NULL). */
int vcsrmc_apply_column_permutation(vcsrmc_csr* csr, float* B, int32_t O,
                                    const int32_t* position);

/* ---- format: src/vcsr_mc.cu:14-22 half_scale, :25-123 csr_to_vcsr_mc ----------------- */
int vcsrmc_half_scale(const vcsrmc_csr* csr, float* scale);
/* fp32 = 0 builds the FP16 format (values divided by half_scale), 1 the FP32 format.
 * nthreads <= 0: all host threads. Output is bit-identical to the reference builder's. */
int vcsrmc_build_host(const vcsrmc_csr* csr, int fp32, int segw, int nthreads,
                      vcsrmc_format** out);
int vcsrmc_format_view_get(const vcsrmc_format* f, vcsrmc_format_view* out);
/* Copies a format given as arrays (e.g. one built by another implementation of
 * csr_to_vcsr_mc) into a library handle; vcsrmc_upload validates its indices. */
int vcsrmc_format_from_view(const vcsrmc_format_view* v, vcsrmc_format** out);
void vcsrmc_format_free(vcsrmc_format* f);

/* ---- device format: src/vcsr_mc.cu:332-349 upload_vcsr_mc_device, :397-404
 *      destroy_vcsr_mc_device ------------------------------------------------------------ */
/* Validates the format's index arrays on the host, then copies them to `device` (< 0: the
 * calling thread's current device) in the kernels' layout (FP16 formats keep fp16 values on
 * the device). Blocking. */
int vcsrmc_upload(const vcsrmc_format* f, int device, void* stream, vcsrmc_device_format** out);
/* Same, choosing which plan layouts to make resident: a bit mask of (1 << VCSRMC_PLAN_SEGMENT),
 * (1 << VCSRMC_PLAN_ROWS), (1 << VCSRMC_PLAN_BAND) and (1 << VCSRMC_PLAN_HYBRID). 0 (what
 * vcsrmc_upload does) = SEGMENT and ROWS, plus, for an FP16 format, BAND where its band x 64-column
 * tiles hold enough entries on average to beat ROWS, else HYBRID where at least half the entries
 * sit in tiles that dense (both estimated from a sample of bands). */
int vcsrmc_upload_ex(const vcsrmc_format* f, int device, int plans, void* stream,
                     vcsrmc_device_format** out);
/* Upload tuning; zero-initialise and set what you need (0 = the library's choice). */
typedef struct {
    int32_t plans;         /* plan layouts to make resident, as in vcsrmc_upload_ex           */
    int32_t rows_unit_nnz; /* ROWS plan: entries per work unit, a power of two in [16, 1024];
                              rows with more entries are split into chunks of this size.
                              0 = chosen from the matrix so that every SM gets enough units.  */
    int32_t band_rows;     /* BAND plan: rows per band, 1 .. 128; 0 = chosen from the matrix    */
    /* ROWS plan, hot columns (off by default). The most used columns of A get a rank (most
     * entries first); a call can then copy their rows of B into one compact buffer that the
     * next gathers read, optionally under a persisting L2 window, and read the other rows with
     * evict-first loads. C is the same either way. On the 2^24-row R-MAT none of these made
     * the SpMM faster on a B200 (the kernel is bound by gathers in flight, not DRAM bytes); they
     * are kept for matrices and GPUs where L2 policy decides.                                  */
    int32_t hot_rows;       /* 0 = no hot columns; > 0 = rank at most this many columns       */
    int32_t hot_budget_mib; /* MiB of hot B rows copied per call, 0 = no copy (0 .. 4096)      */
    int32_t hot_persist;    /* 1 = the copied rows get a persisting L2 access-policy window;
                               raises this process's persisting-L2 limit on the device up to
                               the device's maximum (a context setting, gone at exit)         */
    int32_t hot_evict_first;/* 1 = rows of unranked columns are read with evict-first loads  */
    int32_t reserved[1];    /* must be 0                                                       */
} vcsrmc_upload_options;
int vcsrmc_upload_opts(const vcsrmc_format* f, int device, const vcsrmc_upload_options* opts,
                       void* stream, vcsrmc_device_format** out);
/* Device-side construction: builds the format of a CSR already in device memory (row_ptr[M+1],
 * col[nnz], val[nnz] on `device`; row_ptr from 0 to nnz, rows with strictly ascending columns)
 * and makes its plan layouts resident there, without a host copy of the matrix. opts may be NULL;
 * plans 0 = SEGMENT and ROWS, plus BAND on the same rule as vcsrmc_upload_ex; the BAND view is
 * the one an upload of the same matrix makes (same band height, tiles and entry order).
 * Rows with equal per-segment entry counts are ordered by ascending row, so group_rows, lcol and
 * val can differ from vcsrmc_build_host's by a permutation inside such runs (the reference takes
 * that order from its hash map); every other array is identical. Blocking. */
int vcsrmc_build_device(int32_t M, int32_t N, int64_t nnz, const int32_t* row_ptr, const int32_t* col,
                        const float* val, int fp32, int segw, int device,
                        const vcsrmc_upload_options* opts, void* stream, vcsrmc_device_format** out);
/* The fp16 range scale of nnz fp32 values that are already in device memory (current device):
 * the largest |value| is reduced on the GPU and turned into the scale that vcsrmc_half_scale
 * gives for the same values (1 when the largest magnitude is already in fp16's comfortable range).
 * Blocking. Has no counterpart in the reference: it exists for callers that cannot allocate
 * device memory (a caller running under a fixed memory budget or its own pool allocator, or a
 * process whose allocator is not to be touched), so it makes no cudaMalloc, cudaFree or
 * library allocation. Its scratch is one 32-bit word in a file-scope device array that every
 * device loading this library holds until the process exits; the word is cleared on the stream
 * before each reduction, and calls in one process are serialised by a lock, because two
 * reductions overlapping on the GPU would race on that word. */
int vcsrmc_half_scale_device(const float* val, int64_t nnz, void* stream, float* scale);
/* Copies the SEGMENT arrays of a device format back into a host format (values as the device
 * holds them: FP16 formats keep them rounded to fp16). */
int vcsrmc_device_download(const vcsrmc_device_format* d, vcsrmc_format** out);
int vcsrmc_device_free(vcsrmc_device_format* d);
/* Shape and resident layouts of a device format. */
typedef struct {
    int32_t device, M, N, segw, fp32;
    float scale;
    int32_t plans;                        /* resident layouts: bits (1 << VCSRMC_PLAN_*)     */
    int64_t n_groups, n_slots, n_items;   /* SEGMENT layout                                 */
    int64_t n_units;                      /* ROWS layout: work units                        */
    int32_t rows_unit_nnz, n_split_rows;  /* ROWS: entries per unit, rows split into chunks */
    int32_t band_rows, n_bands;           /* BAND layout                                    */
    int64_t n_tiles;
    int32_t band_cols;                    /* BAND: columns per tile (this build's tile width) */
    int32_t n_hot;                        /* ROWS: ranked hot columns (0: none)              */
    int32_t hybrid_band_rows, reserved2;  /* HYBRID: rows per band of its band part          */
    int64_t hybrid_tiles;                 /* HYBRID: dense tiles                             */
    int64_t hybrid_band_nnz;              /* HYBRID: entries run on the tensor cores         */
    int64_t hybrid_rows_nnz;              /* HYBRID: entries run on the rows plan            */
} vcsrmc_device_info;
int vcsrmc_device_info_get(const vcsrmc_device_format* d, vcsrmc_device_info* out);
/* Error flags raised by kernels of this format since the last clear (bit 0: a bounded wait
 * timed out). Blocking read. */
int vcsrmc_device_status(const vcsrmc_device_format* d, uint32_t* flags, int clear);

/* Diagnostic of the bounded device waits (no counterpart in the reference): one CTA on d's device
 * holds tensor memory and waits up to budget_cycles SM clock cycles (1 .. 2e9) on an mbarrier
 * phase that cannot complete, as an SpMM kernel would on a lost copy. The wait must expire: it
 * sets the timeout flag in d's status word (vcsrmc_device_status), frees the tensor memory, and
 * *completed = 0 (1 would mean the phase completed). Blocking; nothing else is in flight. */
int vcsrmc_device_wait_check(const vcsrmc_device_format* d, int64_t budget_cycles, void* stream,
                             int* completed);

/* ---- SpMM: src/vcsr_mc.cu:352-394 run_vcsr_mc_spmm_gpu ----------------------------------
 * C[M x O] (+)= A * B[N x O]. B is fp32 (both formats) or fp16 (FP16 format only), with row
 * stride ldb elements; C is fp32 with row stride ldc. accumulate = 1 adds into C, as the
 * reference does (its caller zeroes C first, src/main.cpp:242); 0 overwrites C.
 * tileK: columns of B/C per CTA, one of 16, 32, 64, 128, 256 (the FP16 tensor-core kernel
 * runs 16 and 32 as 64-column slabs; results do not depend on tileK).
 * Asynchronous on `stream`. */
int vcsrmc_spmm(const vcsrmc_device_format* d, const void* B, int b_dtype, int64_t ldb, int32_t O,
                int32_t tileK, float* C, int64_t ldc, int accumulate, void* stream);
/* Same, with an explicit plan (VCSRMC_PLAN_*); the plan's layout must be resident. */
int vcsrmc_spmm_ex(const vcsrmc_device_format* d, const void* B, int b_dtype, int64_t ldb,
                   int32_t O, int32_t tileK, float* C, int64_t ldc, int accumulate, int plan,
                   void* stream);
/* Blocking form with the reference's semantics: records events around the launch, waits,
 * returns the elapsed milliseconds in *ms (src/vcsr_mc.cu:380-393). */
int vcsrmc_spmm_timed(const vcsrmc_device_format* d, const void* B, int b_dtype, int64_t ldb,
                      int32_t O, int32_t tileK, float* C, int64_t ldc, int accumulate,
                      void* stream, float* ms);

/* ---- synthetic inputs (no reference counterpart; the benchmark configurations) --------- */
int vcsrmc_gen_csr(int kind, int32_t param, uint64_t seed, int nthreads, vcsrmc_csr** out);
/* rows x cols U(-1,1) row-major; element (i, j) is draw i*cols + j of the dense stream. */
int vcsrmc_gen_dense_host(int64_t rows, int32_t cols, uint64_t seed, float* out, int nthreads);
/* Same values on the device (dtype F32, or F16 = the fp32 value rounded to nearest even),
 * written with row stride ld. Asynchronous on `stream`. */
int vcsrmc_gen_dense_device(int64_t rows, int32_t cols, uint64_t seed, int dtype, void* out,
                            int64_t ld, void* stream);

/* ---- multi-GPU row partition (no reference counterpart) --------------------------------
 * cuts[0..parts]: cuts[k] = first row whose nnz prefix reaches ceil(k * nnz / parts). */
int vcsrmc_partition_rows(const int32_t* row_ptr, int32_t M, int32_t parts, int32_t* cuts);
/* Same, balancing nnz + row_weight * rows per block (each output row also costs a C row store;
 * row_weight = 0 is the nnz balance above). */
int vcsrmc_partition_rows_weighted(const int32_t* row_ptr, int32_t M, int32_t parts, double row_weight,
                                   int32_t* cuts);

#ifdef __cplusplus
}
#endif
#endif /* VCSRMC_H */
