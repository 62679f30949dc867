// Device half of the C ABI (vcsrmc.h): format upload/free/status, SpMM dispatch, dense
// generator. Replaces the reference's module-global device copies and launcher
// (src/vcsr_mc.cu:126-131, 332-404) with one handle per (format, device).
//
// Device layout of a format (all arrays 256-byte aligned by cudaMalloc):
//   items  int2[n_items]    {gbeg, gend}
//   gmeta  int4[n_groups]   {slot_begin, depth, seg_base, 0}   (one 16-byte load per group)
//   grows  int [16*n_groups]
//   lcol   int8[n_slots]    local column, -1 = padding (segw <= 64 fits a byte)
//   val    fp16[n_slots] for the FP16 format (rounded to nearest even, as the reference's
//          (_Float16) conversion), fp32[n_slots] for the FP32 format
//   status uint32           kernel error flags (bounded waits)
// plus, for the ROWS plan (plan_rows.cu), the row view: rp int32[M+1], cols int32[nnz],
//   vals fp16|fp32[nnz], units int4[n_units], split_rows int32[n_split_rows];
// and for the BAND plan (plan_band.cu, FP16 format), the band view: tile_ptr int32[bands+1],
//   tile_col int32[tiles], tile_eptr int32[tiles+1], ents uint32[nnz] (column, row, fp16 value).
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>
#include <string>
#include <vector>

#include "../capi_internal.hpp"
#include "../common/vrng.h"
#include "../host/parallel.hpp"
#include "common.cuh"
#include "build_device.hpp"
#include "plan_band.hpp"
#include "plan_rows.hpp"
#include "spmm_launch.hpp"
#include "wait_check.hpp"

struct vcsrmc_device_format {
    int device = 0;
    int M = 0, N = 0, segw = 0, fp32 = 0, num_segments = 0;
    float scale = 1.f;
    int64_t n_groups = 0, n_slots = 0, n_items = 0;
    int2* items = nullptr;
    int4* gmeta = nullptr;
    int* grows = nullptr;
    int8_t* lcol = nullptr;
    void* val = nullptr;
    uint32_t* status = nullptr;
    bool has_segment = false;
    // ROWS plan
    bool has_rows = false;
    int4* units = nullptr;
    int64_t n_units = 0;
    int* rp = nullptr;
    int* cols = nullptr;
    void* rvals = nullptr;
    int* split_rows = nullptr;
    int n_split_rows = 0;
    int unit_nnz = 0;
    // BAND plan
    bool has_band = false;
    int n_bands = 0, band_rows = 0;
    int64_t n_tiles = 0;
    int* tile_ptr = nullptr;
    int* tile_col = nullptr;
    int* tile_eptr = nullptr;
    uint32_t* ents = nullptr;
    // HYBRID plan: the dense band tiles (a band view of their entries) and the other entries as a
    // row view, run on the rows plan in accumulate mode after the band kernel
    bool has_hybrid = false;
    int hb_bands = 0, hb_rows = 0;
    int64_t hb_tiles = 0, hb_nnz = 0;
    int* hb_tile_ptr = nullptr;
    int* hb_tile_col = nullptr;
    int* hb_tile_eptr = nullptr;
    uint32_t* hb_ents = nullptr;
    int* hr_rp = nullptr;
    int* hr_cols = nullptr;
    void* hr_vals = nullptr;
    int4* hr_units = nullptr;
    int64_t hr_n_units = 0, hr_nnz = 0;
    int* hr_split = nullptr;
    int hr_n_split = 0;
    // ROWS plan, hot columns (RowHotView): ranked columns, and the compact copy of their B rows
    // that each call refreshes (grown on demand; launches of one handle are ordered).
    int* hot_cols = nullptr;
    int n_hot = 0;
    int64_t hot_budget = 0;
    bool hot_persist = false;
    bool hot_evict_first = false;
    void* hot_buf = nullptr;
    int64_t hot_buf_bytes = 0;
    std::mutex hot_mu;
};

namespace vcsrmc {
namespace {

void cuda_check(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return;
    // A failed call also leaves its error as the thread's last runtime error, which the next
    // launch check (cudaGetLastError) would report again; clear it (a sticky error stays).
    cudaGetLastError();
    const int s = e == cudaErrorMemoryAllocation ? VCSRMC_OOM : VCSRMC_CUDA_ERR;
    throw StatusError(s, std::string(what) + ": " + cudaGetErrorString(e));
}

// Restores the calling thread's current device on scope exit.
struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        cuda_check(cudaGetDevice(&prev), "cudaGetDevice");
        if (prev != dev) cuda_check(cudaSetDevice(dev), "cudaSetDevice");
    }
    ~DeviceGuard() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

template <class T>
T* upload_array(const T* src, size_t n, cudaStream_t st) {
    T* p = nullptr;
    cuda_check(cudaMalloc(&p, sizeof(T) * std::max<size_t>(n, 1)), "cudaMalloc");
    if (n) {
        const cudaError_t e = cudaMemcpyAsync(p, src, sizeof(T) * n, cudaMemcpyHostToDevice, st);
        if (e != cudaSuccess) {
            cudaFree(p);
            cuda_check(e, "cudaMemcpyAsync");
        }
    }
    return p;
}

void free_device(vcsrmc_device_format* d) {
    if (!d) return;
    int prev = -1;
    cudaGetDevice(&prev);
    cudaSetDevice(d->device);
    cudaFree(d->items);
    cudaFree(d->gmeta);
    cudaFree(d->grows);
    cudaFree(d->lcol);
    cudaFree(d->val);
    cudaFree(d->status);
    cudaFree(d->units);
    cudaFree(d->rp);
    cudaFree(d->cols);
    cudaFree(d->rvals);
    cudaFree(d->split_rows);
    cudaFree(d->tile_ptr);
    cudaFree(d->tile_col);
    cudaFree(d->tile_eptr);
    cudaFree(d->ents);
    cudaFree(d->hb_tile_ptr);
    cudaFree(d->hb_tile_col);
    cudaFree(d->hb_tile_eptr);
    cudaFree(d->hb_ents);
    cudaFree(d->hr_rp);
    cudaFree(d->hr_cols);
    cudaFree(d->hr_vals);
    cudaFree(d->hr_units);
    cudaFree(d->hr_split);
    cudaFree(d->hot_cols);
    cudaFree(d->hot_buf);
    // Lines marked persisting stay in L2's set-aside until reset and slow later kernels: return
    // them to normal once the handle that marked them is gone.
    if (d->hot_persist && d->n_hot > 0 && d->hot_budget > 0) {
        cudaCtxResetPersistingL2Cache();
        cudaGetLastError();
    }
    if (prev >= 0) cudaSetDevice(prev);
    delete d;
}

// Every index the kernels dereference is checked here, once, so that a malformed format is an
// error status instead of an out-of-bounds access on the GPU.
void validate_format(const VCSRMC& v) {
    const int64_t G = int64_t(v.group_depth.size());
    const int64_t S = int64_t(v.lcol.size());
    auto bad = [](const char* what) { throw StatusError(VCSRMC_INVALID_ARG, std::string("invalid format: ") + what); };
    if (v.segw != 16 && v.segw != 32 && v.segw != 48 && v.segw != 64) bad("segw");
    if (v.bundle != 16) bad("bundle");
    if (int64_t(v.group_ptr.size()) != G + 1 || int64_t(v.group_seg_base.size()) != G ||
        int64_t(v.group_rows.size()) != 16 * G || int64_t(v.val.size()) != S ||
        v.item_gbeg.size() != v.item_gend.size())
        bad("array sizes");
    if (G * 16 > INT32_MAX || S > INT32_MAX) bad("sizes exceed 32-bit offsets");
    if (v.group_ptr[0] != 0 || v.group_ptr[G] != S) bad("group_ptr ends");
    for (int64_t g = 0; g < G; ++g) {
        if (v.group_depth[g] < 0 || int64_t(v.group_ptr[g + 1]) - v.group_ptr[g] != 16 * int64_t(v.group_depth[g]))
            bad("group_ptr/group_depth");
        if (v.group_seg_base[g] < 0 || v.group_seg_base[g] >= std::max(v.N, 1) || v.group_seg_base[g] % v.segw)
            bad("group_seg_base");
    }
    for (int64_t i = 0; i < 16 * G; ++i)
        if (v.group_rows[i] < -1 || v.group_rows[i] >= v.M) bad("group_rows");
    for (int64_t s = 0; s < S; ++s)
        if (v.lcol[s] < -1 || v.lcol[s] >= v.segw) bad("lcol");
    for (int64_t g = 0; g < G; ++g)
        for (int64_t s = v.group_ptr[g]; s < v.group_ptr[g + 1]; ++s)
            if (v.lcol[s] >= 0 && int64_t(v.group_seg_base[g]) + v.lcol[s] >= v.N) bad("column beyond N");
    for (size_t i = 0; i < v.item_gbeg.size(); ++i) {
        const int b = v.item_gbeg[i], e = v.item_gend[i];
        if (b < 0 || e <= b || e > G) bad("item range");
        for (int g = b + 1; g < e; ++g)
            if (v.group_seg_base[g] != v.group_seg_base[b]) bad("item spans segments");
    }
}

// ROWS plan hot columns (RowHotView): the most MiB of B rows one call may copy.
constexpr int kHotBudgetMiBMax = 4096;

void check_hot_options(const vcsrmc_upload_options& o) {
    if (o.hot_rows < 0) throw StatusError(VCSRMC_INVALID_ARG, "hot_rows must be 0 or positive");
    if (o.hot_budget_mib < 0 || o.hot_budget_mib > kHotBudgetMiBMax)
        throw StatusError(VCSRMC_INVALID_ARG, "hot_budget_mib must be in [0, 4096]");
    if (o.hot_persist < 0 || o.hot_persist > 1) throw StatusError(VCSRMC_INVALID_ARG, "hot_persist must be 0 or 1");
    if (o.hot_evict_first < 0 || o.hot_evict_first > 1)
        throw StatusError(VCSRMC_INVALID_ARG, "hot_evict_first must be 0 or 1");
}

// Ranks the hot columns of a resident ROWS layout (rewriting its device cols) as the options ask,
// and, for a persisting window, raises this process's persisting-L2 limit on the device to the
// copy budget (at most the device's maximum).
void make_hot_columns(vcsrmc_device_format* d, int64_t nnz, const vcsrmc_upload_options& o, cudaStream_t st) {
    d->hot_budget = int64_t(o.hot_budget_mib) << 20;
    d->hot_persist = o.hot_persist == 1;
    d->hot_evict_first = o.hot_evict_first == 1;
    if (o.hot_rows <= 0 || !d->has_rows) return;
    d->hot_cols = dev::build_hot_columns(d->cols, nnz, d->N, o.hot_rows, &d->n_hot, st);
    if (d->n_hot > 0 && d->hot_persist && d->hot_budget > 0) {
        int max_persist = 0;
        size_t cur = 0;
        cuda_check(cudaDeviceGetAttribute(&max_persist, cudaDevAttrMaxPersistingL2CacheSize, d->device),
                   "cudaDeviceGetAttribute");
        cuda_check(cudaDeviceGetLimit(&cur, cudaLimitPersistingL2CacheSize), "cudaDeviceGetLimit");
        const size_t want = size_t(std::min<int64_t>(d->hot_budget, max_persist));
        if (cur < want) cuda_check(cudaDeviceSetLimit(cudaLimitPersistingL2CacheSize, want), "cudaDeviceSetLimit");
    }
}

// The hot-row buffer for a call whose B rows are row_bytes apart: grown (after the stream's
// earlier work, which may still read the old one) when the copy needs more than it holds.
void ensure_hot_buffer(const vcsrmc_device_format* cd, int64_t row_bytes, cudaStream_t st) {
    auto* d = const_cast<vcsrmc_device_format*>(cd);
    if (d->n_hot <= 0 || row_bytes <= 0) return;
    const int64_t need = std::min<int64_t>(d->hot_budget, int64_t(d->n_hot) * row_bytes);
    if (need < row_bytes) return;
    std::lock_guard<std::mutex> lock(d->hot_mu);
    if (d->hot_buf_bytes >= need) return;
    if (d->hot_buf) {
        cuda_check(cudaStreamSynchronize(st), "cudaStreamSynchronize");
        cudaFree(d->hot_buf);
        d->hot_buf = nullptr;
        d->hot_buf_bytes = 0;
    }
    cuda_check(cudaMalloc(&d->hot_buf, size_t(need)), "cudaMalloc");
    d->hot_buf_bytes = need;
}

dev::DeviceFormatView view_of(const vcsrmc_device_format* d) {
    dev::DeviceFormatView F;
    F.items = d->items;
    F.gmeta = d->gmeta;
    F.grows = d->grows;
    F.lcol = d->lcol;
    F.val = d->val;
    F.status = d->status;
    F.num_items = int(d->n_items);
    F.M = d->M;
    F.N = d->N;
    F.segw = d->segw;
    F.scale = d->scale;
    return F;
}

void check_spmm_args(const vcsrmc_device_format* d, const void* B, int b_dtype, int64_t ldb, int32_t O,
                     int32_t tileK, const float* C, int64_t ldc) {
    if (!d) throw StatusError(VCSRMC_INVALID_ARG, "NULL format");
    if (O < 1) throw StatusError(VCSRMC_INVALID_ARG, "O must be >= 1");
    if (tileK != 16 && tileK != 32 && tileK != 64 && tileK != 128 && tileK != 256)
        throw StatusError(VCSRMC_INVALID_ARG, "tileK must be one of 16, 32, 64, 128, 256");
    if (b_dtype != VCSRMC_F32 && b_dtype != VCSRMC_F16) throw StatusError(VCSRMC_INVALID_ARG, "unknown B dtype");
    if (b_dtype == VCSRMC_F16 && d->fp32)
        throw StatusError(VCSRMC_INVALID_ARG, "the FP32 format takes fp32 B only");
    if (ldb < O || ldc < O) throw StatusError(VCSRMC_INVALID_ARG, "ldb and ldc must be >= O");
    if ((d->N > 0 && !B) || (d->M > 0 && !C)) throw StatusError(VCSRMC_INVALID_ARG, "NULL B or C");
}

// AUTO: BAND for fp16 B (its tiles are TMA copies of fp16 B; fp32 B would be converted tile by
// tile), then ROWS, then SEGMENT, then BAND for fp32 B; the first whose layout is resident.
int resolve_plan(const vcsrmc_device_format* d, int plan, int b_dtype) {
    if (plan == VCSRMC_PLAN_AUTO) {
        if (d->has_band && b_dtype == VCSRMC_F16) plan = VCSRMC_PLAN_BAND;
        else if (d->has_hybrid && b_dtype == VCSRMC_F16) plan = VCSRMC_PLAN_HYBRID;
        else if (d->has_rows) plan = VCSRMC_PLAN_ROWS;
        else if (d->has_segment) plan = VCSRMC_PLAN_SEGMENT;
        else if (d->has_band) plan = VCSRMC_PLAN_BAND;
        else plan = VCSRMC_PLAN_HYBRID;
    }
    if (plan == VCSRMC_PLAN_HYBRID && !d->has_hybrid)
        throw StatusError(VCSRMC_INVALID_ARG, "the HYBRID plan layout was not uploaded");
    if (plan == VCSRMC_PLAN_ROWS && !d->has_rows)
        throw StatusError(VCSRMC_INVALID_ARG, "the ROWS plan layout was not uploaded");
    if (plan == VCSRMC_PLAN_SEGMENT && !d->has_segment)
        throw StatusError(VCSRMC_INVALID_ARG, "the SEGMENT plan layout was not uploaded");
    if (plan == VCSRMC_PLAN_BAND && !d->has_band)
        throw StatusError(VCSRMC_INVALID_ARG, "the BAND plan layout was not uploaded");
    if (plan != VCSRMC_PLAN_ROWS && plan != VCSRMC_PLAN_SEGMENT && plan != VCSRMC_PLAN_BAND &&
        plan != VCSRMC_PLAN_HYBRID)
        throw StatusError(VCSRMC_INVALID_ARG, "unknown plan");
    return plan;
}

void launch_spmm(const vcsrmc_device_format* d, const void* B, int b_dtype, int64_t ldb, int32_t O, int32_t tileK,
                 float* C, int64_t ldc, int accumulate, int plan, cudaStream_t st) {
    plan = resolve_plan(d, plan, b_dtype);
    cudaError_t e;
    if (plan == VCSRMC_PLAN_ROWS) {
        dev::RowPlanView P;
        P.units = d->units;
        P.n_units = d->n_units;
        P.rp = d->rp;
        P.cols = d->cols;
        P.vals = d->rvals;
        P.vals_f16 = d->fp32 ? 0 : 1;
        P.split_rows = d->split_rows;
        P.n_split_rows = d->n_split_rows;
        P.M = d->M;
        P.N = d->N;
        P.scale = d->scale;
        const int64_t row_bytes = ldb * (b_dtype == VCSRMC_F16 ? 2 : 4);
        ensure_hot_buffer(d, row_bytes, st);
        P.hot.hot_cols = d->hot_cols;
        P.hot.n_hot = d->n_hot;
        P.hot.buf = d->hot_buf;
        P.hot.buf_bytes = d->hot_buf_bytes;
        P.hot.budget_bytes = d->hot_budget;
        P.hot.persist = d->hot_persist;
        P.hot.cold_hint = d->hot_evict_first;
        e = dev::spmm_rows(P, B, b_dtype == VCSRMC_F16 ? 1 : 0, ldb, O, C, ldc, accumulate != 0, st);
        cuda_check(e, "SpMM launch (rows plan)");
        return;
    }
    if (plan == VCSRMC_PLAN_HYBRID) {
        // dense tiles on the tensor cores (every row of C written, or added to), then the other
        // entries added by the rows plan
        dev::BandPlanView P;
        P.tile_ptr = d->hb_tile_ptr;
        P.tile_col = d->hb_tile_col;
        P.tile_eptr = d->hb_tile_eptr;
        P.ents = d->hb_ents;
        P.n_bands = d->hb_bands;
        P.band_rows = d->hb_rows;
        P.M = d->M;
        P.N = d->N;
        P.scale = d->scale;
        P.status = d->status;
        e = dev::spmm_band(P, B, b_dtype == VCSRMC_F16 ? 1 : 0, ldb, O, C, ldc, accumulate != 0, st);
        cuda_check(e, "SpMM launch (hybrid plan, band part)");
        if (d->hr_nnz > 0) {
            dev::RowPlanView R;
            R.units = d->hr_units;
            R.n_units = d->hr_n_units;
            R.rp = d->hr_rp;
            R.cols = d->hr_cols;
            R.vals = d->hr_vals;
            R.vals_f16 = 1;
            R.split_rows = d->hr_split;
            R.n_split_rows = d->hr_n_split;
            R.M = d->M;
            R.N = d->N;
            R.scale = d->scale;
            e = dev::spmm_rows(R, B, b_dtype == VCSRMC_F16 ? 1 : 0, ldb, O, C, ldc, true, st);
            cuda_check(e, "SpMM launch (hybrid plan, rows part)");
        }
        return;
    }
    if (plan == VCSRMC_PLAN_BAND) {
        dev::BandPlanView P;
        P.tile_ptr = d->tile_ptr;
        P.tile_col = d->tile_col;
        P.tile_eptr = d->tile_eptr;
        P.ents = d->ents;
        P.n_bands = d->n_bands;
        P.band_rows = d->band_rows;
        P.M = d->M;
        P.N = d->N;
        P.scale = d->scale;
        P.status = d->status;
        e = dev::spmm_band(P, B, b_dtype == VCSRMC_F16 ? 1 : 0, ldb, O, C, ldc, accumulate != 0, st);
        cuda_check(e, "SpMM launch (band plan)");
        return;
    }
    if (!accumulate && d->M > 0) {
        if (ldc == O)
            cuda_check(cudaMemsetAsync(C, 0, sizeof(float) * size_t(d->M) * size_t(O), st), "cudaMemsetAsync");
        else
            cuda_check(cudaMemset2DAsync(C, size_t(ldc) * sizeof(float), 0, size_t(O) * sizeof(float), size_t(d->M), st),
                       "cudaMemset2DAsync");
    }
    const dev::DeviceFormatView F = view_of(d);
    if (d->fp32)
        e = dev::spmm_fp32_atomic(F, static_cast<const float*>(B), ldb, O, tileK, C, ldc, st);
    else
        e = dev::spmm_fp16_tc_atomic(F, B, b_dtype == VCSRMC_F16 ? 1 : 0, ldb, O, tileK, C, ldc, st);
    cuda_check(e, "SpMM launch (segment plan)");
}

__global__ void gen_dense_kernel(int64_t rows, int cols, uint64_t key, int f16, void* out, int64_t ld) {
    const int64_t total = rows * int64_t(cols);
    for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
        const int64_t r = i / cols, c = i % cols;
        const float v = vrng_sym(vrng_at(key, uint64_t(i)));
        if (f16)
            static_cast<__half*>(out)[r * ld + c] = __float2half_rn(v);
        else
            static_cast<float*>(out)[r * ld + c] = v;
    }
}

}  // namespace

namespace dev {
cudaError_t gen_dense_device(int64_t rows, int cols, uint64_t seed, int f16, void* out, int64_t ld, cudaStream_t st) {
    const int64_t total = rows * int64_t(cols);
    if (total == 0) return cudaSuccess;
    int sms = 0, dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
    const int64_t blocks = std::min<int64_t>((total + 255) / 256, int64_t(sms) * 16);
    gen_dense_kernel<<<unsigned(blocks), 256, 0, st>>>(rows, cols, vrng_key(seed, VRNG_STREAM_DENSE), f16, out, ld);
    return cudaGetLastError();
}
}  // namespace dev

}  // namespace vcsrmc

using namespace vcsrmc;

VCSRMC_EXPORT int vcsrmc_upload_opts(const vcsrmc_format* f, int device, const vcsrmc_upload_options* opts,
                                     void* stream, vcsrmc_device_format** out) {
    return guarded([&] {
        if (!f || !out || !opts) throw StatusError(VCSRMC_INVALID_ARG, "NULL argument");
        for (int r : opts->reserved)
            if (r != 0) throw StatusError(VCSRMC_INVALID_ARG, "reserved upload options must be 0");
        int plans = opts->plans;
        const bool default_plans = plans == 0;
        if (default_plans) plans = (1 << VCSRMC_PLAN_SEGMENT) | (1 << VCSRMC_PLAN_ROWS);
        if (plans & ~((1 << VCSRMC_PLAN_SEGMENT) | (1 << VCSRMC_PLAN_ROWS) | (1 << VCSRMC_PLAN_BAND) |
                      (1 << VCSRMC_PLAN_HYBRID)))
            throw StatusError(VCSRMC_INVALID_ARG, "unknown plan bits");
        if ((plans & ((1 << VCSRMC_PLAN_BAND) | (1 << VCSRMC_PLAN_HYBRID))) && f->v.fp32)
            throw StatusError(VCSRMC_INVALID_ARG,
                              "the BAND and HYBRID plans run on the tensor cores and need the FP16 format");
        int unit_nnz = opts->rows_unit_nnz;
        if (unit_nnz != 0 && (unit_nnz < 16 || unit_nnz > dev::kUnitNnzMax || (unit_nnz & (unit_nnz - 1))))
            throw StatusError(VCSRMC_INVALID_ARG, "rows_unit_nnz must be 0 or a power of two in [16, 1024]");
        if (opts->band_rows < 0 || opts->band_rows > dev::kBandRows)
            throw StatusError(VCSRMC_INVALID_ARG, "band_rows must be 0 or in [1, 128]");
        check_hot_options(*opts);
        const VCSRMC& v = f->v;
        validate_format(v);
        if (device < 0) cuda_check(cudaGetDevice(&device), "cudaGetDevice");
        DeviceGuard guard(device);
        cudaStream_t st = static_cast<cudaStream_t>(stream);
        auto* d = new vcsrmc_device_format;
        d->device = device;
        d->M = v.M;
        d->N = v.N;
        d->segw = v.segw;
        d->num_segments = v.num_segments;
        d->fp32 = v.fp32 ? 1 : 0;
        d->scale = v.scale;
        d->n_groups = int64_t(v.group_depth.size());
        d->n_slots = int64_t(v.lcol.size());
        d->n_items = int64_t(v.item_gbeg.size());
        try {
            const int64_t G = d->n_groups, S = d->n_slots, I = d->n_items;
            const int nth = resolve_threads(0);
            if (plans & (1 << VCSRMC_PLAN_SEGMENT)) {
                std::vector<int2> items(I);
                for (int64_t i = 0; i < I; ++i) items[i] = make_int2(v.item_gbeg[i], v.item_gend[i]);
                std::vector<int4> gmeta(G);
                for (int64_t g = 0; g < G; ++g)
                    gmeta[g] = make_int4(v.group_ptr[g], v.group_depth[g], v.group_seg_base[g], 0);
                std::vector<int8_t> lcol(S);
                parallel_for(0, S, nth, [&](int64_t a, int64_t b) {
                    for (int64_t s = a; s < b; ++s) lcol[s] = int8_t(v.lcol[s]);
                });
                d->items = upload_array(items.data(), items.size(), st);
                d->gmeta = upload_array(gmeta.data(), gmeta.size(), st);
                d->grows = upload_array(v.group_rows.data(), v.group_rows.size(), st);
                d->lcol = upload_array(lcol.data(), lcol.size(), st);
                if (d->fp32) {
                    d->val = upload_array(v.val.data(), v.val.size(), st);
                } else {
                    std::vector<__half> h(S);
                    parallel_for(0, S, nth, [&](int64_t a, int64_t b) {
                        for (int64_t s = a; s < b; ++s) h[s] = __float2half_rn(v.val[s]);
                    });
                    d->val = upload_array(h.data(), h.size(), st);
                    cuda_check(cudaStreamSynchronize(st), "cudaStreamSynchronize");
                }
                d->has_segment = true;
            }
            dev::RowViewHost rv;
            if (plans & ((1 << VCSRMC_PLAN_ROWS) | (1 << VCSRMC_PLAN_BAND) | (1 << VCSRMC_PLAN_HYBRID))) {
                if (unit_nnz == 0) {
                    int sms = 0;
                    cuda_check(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device), "cudaDeviceGetAttribute");
                    const int64_t nnz = std::count_if(v.lcol.begin(), v.lcol.end(), [](int c) { return c >= 0; });
                    unit_nnz = dev::choose_unit_nnz(nnz, sms);
                }
                rv = dev::build_row_view(v, unit_nnz);
                // The default layouts add the BAND plan (FP16 format) where it beats ROWS:
                // enough entries per tensor-core tile.
                dev::BandChoice bc{dev::kBandRows, 0.0};
                if ((plans & ((1 << VCSRMC_PLAN_BAND) | (1 << VCSRMC_PLAN_HYBRID))) || (default_plans && !v.fp32))
                    bc = dev::choose_band(rv, v.M);
                if (opts->band_rows > 0) bc.band_rows = opts->band_rows;
                if (default_plans && !v.fp32 && bc.entries_per_tile >= dev::kBandMinEntriesPerTile)
                    plans |= 1 << VCSRMC_PLAN_BAND;
                else if (default_plans && !v.fp32 && bc.dense_fraction >= dev::kHybridMinDenseFraction)
                    plans |= 1 << VCSRMC_PLAN_HYBRID;
                if (plans & (1 << VCSRMC_PLAN_BAND)) {
                    dev::BandViewHost bv = dev::build_band_view(rv, v.M, bc.band_rows, nth);
                    d->band_rows = bv.band_rows;
                    d->n_bands = int(bv.tile_ptr.size()) - 1;
                    d->n_tiles = int64_t(bv.tile_col.size());
                    d->tile_ptr = upload_array(bv.tile_ptr.data(), bv.tile_ptr.size(), st);
                    d->tile_col = upload_array(bv.tile_col.data(), bv.tile_col.size(), st);
                    d->tile_eptr = upload_array(bv.tile_eptr.data(), bv.tile_eptr.size(), st);
                    d->ents = upload_array(bv.ents.data(), bv.ents.size(), st);
                    cuda_check(cudaStreamSynchronize(st), "cudaStreamSynchronize");
                    d->has_band = true;
                }
                if (plans & (1 << VCSRMC_PLAN_HYBRID)) {
                    const dev::BandViewHost full = dev::build_band_view(rv, v.M, bc.band_rows, nth);
                    dev::RowViewHost dense, resid;
                    dev::split_dense_tiles(rv, full, v.M, int(dev::kBandMinEntriesPerTile), nth, dense, resid);
                    const dev::BandViewHost bv = dev::build_band_view(dense, v.M, bc.band_rows, nth);
                    // the rows part runs in accumulate mode only: units over non-empty rows
                    dev::pack_units(resid.rp.data(), v.M, unit_nnz, resid.units, resid.split_rows, true);
                    d->hb_rows = bv.band_rows;
                    d->hb_bands = int(bv.tile_ptr.size()) - 1;
                    d->hb_tiles = int64_t(bv.tile_col.size());
                    d->hb_nnz = int64_t(bv.ents.size());
                    d->hb_tile_ptr = upload_array(bv.tile_ptr.data(), bv.tile_ptr.size(), st);
                    d->hb_tile_col = upload_array(bv.tile_col.data(), bv.tile_col.size(), st);
                    d->hb_tile_eptr = upload_array(bv.tile_eptr.data(), bv.tile_eptr.size(), st);
                    d->hb_ents = upload_array(bv.ents.data(), bv.ents.size(), st);
                    d->hr_nnz = int64_t(resid.cols.size());
                    d->hr_rp = upload_array(resid.rp.data(), resid.rp.size(), st);
                    d->hr_cols = upload_array(resid.cols.data(), resid.cols.size(), st);
                    std::vector<__half> h(resid.vals.size());
                    for (size_t i = 0; i < h.size(); ++i) h[i] = __float2half_rn(resid.vals[i]);
                    d->hr_vals = upload_array(h.data(), h.size(), st);
                    d->hr_units = reinterpret_cast<int4*>(upload_array(resid.units.data(), resid.units.size(), st));
                    d->hr_n_units = int64_t(resid.units.size());
                    d->hr_split = upload_array(resid.split_rows.data(), resid.split_rows.size(), st);
                    d->hr_n_split = int(resid.split_rows.size());
                    cuda_check(cudaStreamSynchronize(st), "cudaStreamSynchronize");
                    d->has_hybrid = true;
                }
            }
            if (plans & (1 << VCSRMC_PLAN_ROWS)) {
                d->rp = upload_array(rv.rp.data(), rv.rp.size(), st);
                d->cols = upload_array(rv.cols.data(), rv.cols.size(), st);
                static_assert(sizeof(dev::RowViewHost::Unit) == sizeof(int4), "unit layout");
                d->units = reinterpret_cast<int4*>(upload_array(rv.units.data(), rv.units.size(), st));
                d->n_units = int64_t(rv.units.size());
                d->split_rows = upload_array(rv.split_rows.data(), rv.split_rows.size(), st);
                d->n_split_rows = int(rv.split_rows.size());
                d->unit_nnz = unit_nnz;
                if (d->fp32) {
                    d->rvals = upload_array(rv.vals.data(), rv.vals.size(), st);
                } else {
                    std::vector<__half> h(rv.vals.size());
                    parallel_for(0, int64_t(h.size()), nth, [&](int64_t a, int64_t b) {
                        for (int64_t s = a; s < b; ++s) h[s] = __float2half_rn(rv.vals[s]);
                    });
                    d->rvals = upload_array(h.data(), h.size(), st);
                }
                cuda_check(cudaStreamSynchronize(st), "cudaStreamSynchronize");
                d->has_rows = true;
                make_hot_columns(d, int64_t(rv.cols.size()), *opts, st);
            }
            cuda_check(cudaMalloc(&d->status, sizeof(uint32_t)), "cudaMalloc");
            cuda_check(cudaMemsetAsync(d->status, 0, sizeof(uint32_t), st), "cudaMemsetAsync");
            cuda_check(cudaStreamSynchronize(st), "cudaStreamSynchronize");
        } catch (...) {
            free_device(d);
            throw;
        }
        *out = d;
    });
}

VCSRMC_EXPORT int vcsrmc_upload_ex(const vcsrmc_format* f, int device, int plans, void* stream,
                                   vcsrmc_device_format** out) {
    vcsrmc_upload_options o{};
    o.plans = plans;
    return vcsrmc_upload_opts(f, device, &o, stream, out);
}

VCSRMC_EXPORT int vcsrmc_upload(const vcsrmc_format* f, int device, void* stream, vcsrmc_device_format** out) {
    return vcsrmc_upload_ex(f, device, 0, stream, out);
}

VCSRMC_EXPORT int vcsrmc_device_free(vcsrmc_device_format* d) {
    return guarded([&] { free_device(d); });
}

VCSRMC_EXPORT int vcsrmc_device_info_get(const vcsrmc_device_format* d, vcsrmc_device_info* out) {
    return guarded([&] {
        if (!d || !out) throw StatusError(VCSRMC_INVALID_ARG, "NULL argument");
        vcsrmc_device_info i{};
        i.device = d->device;
        i.M = d->M;
        i.N = d->N;
        i.segw = d->segw;
        i.fp32 = d->fp32;
        i.scale = d->scale;
        i.plans = (d->has_segment ? 1 << VCSRMC_PLAN_SEGMENT : 0) | (d->has_rows ? 1 << VCSRMC_PLAN_ROWS : 0) |
                  (d->has_band ? 1 << VCSRMC_PLAN_BAND : 0) | (d->has_hybrid ? 1 << VCSRMC_PLAN_HYBRID : 0);
        i.hybrid_band_rows = d->hb_rows;
        i.hybrid_tiles = d->hb_tiles;
        i.hybrid_band_nnz = d->hb_nnz;
        i.hybrid_rows_nnz = d->hr_nnz;
        i.n_groups = d->n_groups;
        i.n_slots = d->n_slots;
        i.n_items = d->n_items;
        i.n_units = d->n_units;
        i.rows_unit_nnz = d->unit_nnz;
        i.n_split_rows = d->n_split_rows;
        i.band_rows = d->band_rows;
        i.n_bands = d->n_bands;
        i.n_tiles = d->n_tiles;
        i.band_cols = dev::kBandK;
        i.n_hot = d->n_hot;
        *out = i;
    });
}

VCSRMC_EXPORT int vcsrmc_device_status(const vcsrmc_device_format* d, uint32_t* flags, int clear) {
    return guarded([&] {
        if (!d || !flags) throw StatusError(VCSRMC_INVALID_ARG, "NULL argument");
        DeviceGuard guard(d->device);
        cuda_check(cudaMemcpy(flags, d->status, sizeof(uint32_t), cudaMemcpyDeviceToHost), "cudaMemcpy");
        if (clear) cuda_check(cudaMemset(d->status, 0, sizeof(uint32_t)), "cudaMemset");
    });
}

VCSRMC_EXPORT int vcsrmc_device_wait_check(const vcsrmc_device_format* d, int64_t budget_cycles, void* stream,
                                           int* completed) {
    return guarded([&] {
        if (!d || !completed) throw StatusError(VCSRMC_INVALID_ARG, "NULL argument");
        if (budget_cycles < 1 || budget_cycles > dev::kWaitBudgetCycles)
            throw StatusError(VCSRMC_INVALID_ARG, "budget_cycles must be in [1, 2e9]");
        DeviceGuard guard(d->device);
        cudaStream_t st = static_cast<cudaStream_t>(stream);
        uint32_t* flag = nullptr;
        cuda_check(cudaMalloc(&flag, sizeof(uint32_t)), "cudaMalloc");
        uint32_t h = 0;
        cudaError_t e = cudaMemsetAsync(flag, 0, sizeof(uint32_t), st);
        if (e == cudaSuccess) e = dev::bounded_wait_check(d->status, budget_cycles, flag, st);
        if (e == cudaSuccess) e = cudaMemcpyAsync(&h, flag, sizeof(uint32_t), cudaMemcpyDeviceToHost, st);
        if (e == cudaSuccess) e = cudaStreamSynchronize(st);
        cudaFree(flag);
        cuda_check(e, "bounded wait check");
        *completed = int(h);
    });
}

VCSRMC_EXPORT int vcsrmc_spmm_ex(const vcsrmc_device_format* d, const void* B, int b_dtype, int64_t ldb,
                                 int32_t O, int32_t tileK, float* C, int64_t ldc, int accumulate, int plan,
                                 void* stream) {
    return guarded([&] {
        check_spmm_args(d, B, b_dtype, ldb, O, tileK, C, ldc);
        DeviceGuard guard(d->device);
        launch_spmm(d, B, b_dtype, ldb, O, tileK, C, ldc, accumulate, plan, static_cast<cudaStream_t>(stream));
    });
}

VCSRMC_EXPORT int vcsrmc_spmm(const vcsrmc_device_format* d, const void* B, int b_dtype, int64_t ldb, int32_t O,
                              int32_t tileK, float* C, int64_t ldc, int accumulate, void* stream) {
    return vcsrmc_spmm_ex(d, B, b_dtype, ldb, O, tileK, C, ldc, accumulate, VCSRMC_PLAN_AUTO, stream);
}

VCSRMC_EXPORT int vcsrmc_spmm_timed(const vcsrmc_device_format* d, const void* B, int b_dtype, int64_t ldb,
                                    int32_t O, int32_t tileK, float* C, int64_t ldc, int accumulate, void* stream,
                                    float* ms) {
    return guarded([&] {
        if (!ms) throw StatusError(VCSRMC_INVALID_ARG, "NULL ms");
        check_spmm_args(d, B, b_dtype, ldb, O, tileK, C, ldc);
        DeviceGuard guard(d->device);
        cudaStream_t st = static_cast<cudaStream_t>(stream);
        cudaEvent_t t0 = nullptr, t1 = nullptr;
        cuda_check(cudaEventCreate(&t0), "cudaEventCreate");
        cudaError_t e = cudaEventCreate(&t1);
        if (e != cudaSuccess) { cudaEventDestroy(t0); cuda_check(e, "cudaEventCreate"); }
        try {
            cuda_check(cudaEventRecord(t0, st), "cudaEventRecord");
            launch_spmm(d, B, b_dtype, ldb, O, tileK, C, ldc, accumulate, VCSRMC_PLAN_AUTO, st);
            cuda_check(cudaEventRecord(t1, st), "cudaEventRecord");
            cuda_check(cudaEventSynchronize(t1), "cudaEventSynchronize");
            cuda_check(cudaEventElapsedTime(ms, t0, t1), "cudaEventElapsedTime");
        } catch (...) {
            cudaEventDestroy(t0);
            cudaEventDestroy(t1);
            throw;
        }
        cudaEventDestroy(t0);
        cudaEventDestroy(t1);
        uint32_t flags = 0;
        cuda_check(cudaMemcpy(&flags, d->status, sizeof(uint32_t), cudaMemcpyDeviceToHost), "cudaMemcpy");
        if (flags & dev::kStatusTimeout) throw StatusError(VCSRMC_TIMEOUT, "a bounded device wait expired");
    });
}

VCSRMC_EXPORT int vcsrmc_gen_dense_device(int64_t rows, int32_t cols, uint64_t seed, int dtype, void* out,
                                          int64_t ld, void* stream) {
    return guarded([&] {
        if (rows < 0 || cols <= 0 || ld < cols || (rows && !out) || (dtype != VCSRMC_F32 && dtype != VCSRMC_F16))
            throw StatusError(VCSRMC_INVALID_ARG, "bad dense arguments");
        cuda_check(dev::gen_dense_device(rows, cols, seed, dtype == VCSRMC_F16 ? 1 : 0, out, ld,
                                         static_cast<cudaStream_t>(stream)),
                   "gen_dense_device");
    });
}

VCSRMC_EXPORT int vcsrmc_build_device(int32_t M, int32_t N, int64_t nnz, const int32_t* row_ptr, const int32_t* col,
                                      const float* val, int fp32, int segw, int device,
                                      const vcsrmc_upload_options* opts, void* stream, vcsrmc_device_format** out) {
    return guarded([&] {
        if (!out) throw StatusError(VCSRMC_INVALID_ARG, "NULL output");
        if (segw != 16 && segw != 32 && segw != 48 && segw != 64)
            throw StatusError(VCSRMC_INVALID_ARG, "vcsr_mc supports segw in {16, 32, 48, 64}");
        if (M < 0 || N < 0 || nnz < 0 || nnz > INT32_MAX) throw StatusError(VCSRMC_INVALID_ARG, "bad CSR sizes");
        if (!row_ptr || (nnz > 0 && (!col || !val))) throw StatusError(VCSRMC_INVALID_ARG, "NULL CSR array");
        vcsrmc_upload_options o{};
        if (opts) o = *opts;
        for (int r : o.reserved)
            if (r != 0) throw StatusError(VCSRMC_INVALID_ARG, "reserved upload options must be 0");
        int plans = o.plans == 0 ? ((1 << VCSRMC_PLAN_SEGMENT) | (1 << VCSRMC_PLAN_ROWS)) : o.plans;
        constexpr int kTensorPlans = (1 << VCSRMC_PLAN_BAND) | (1 << VCSRMC_PLAN_HYBRID);
        if (plans & ~((1 << VCSRMC_PLAN_SEGMENT) | (1 << VCSRMC_PLAN_ROWS) | kTensorPlans))
            throw StatusError(VCSRMC_INVALID_ARG, "unknown plan bits");
        if ((plans & kTensorPlans) && fp32)
            throw StatusError(VCSRMC_INVALID_ARG,
                              "the BAND and HYBRID plans run on the tensor cores and need the FP16 format");
        int unit_nnz = o.rows_unit_nnz;
        if (unit_nnz != 0 && (unit_nnz < 16 || unit_nnz > dev::kUnitNnzMax || (unit_nnz & (unit_nnz - 1))))
            throw StatusError(VCSRMC_INVALID_ARG, "rows_unit_nnz must be 0 or a power of two in [16, 1024]");
        if (o.band_rows < 0 || o.band_rows > dev::kBandRows)
            throw StatusError(VCSRMC_INVALID_ARG, "band_rows must be 0 or in [1, 128]");
        check_hot_options(o);
        if (device < 0) cuda_check(cudaGetDevice(&device), "cudaGetDevice");
        DeviceGuard guard(device);
        cudaStream_t st = static_cast<cudaStream_t>(stream);
        if (!dev::device_csr_rows_sorted(row_ptr, col, M, N, nnz, st))
            throw StatusError(VCSRMC_INVALID_ARG,
                              "the device builder needs row_ptr from 0 to nnz and rows with strictly ascending "
                              "columns in [0, N) (vcsrmc_build_host sorts other rows)");
        const float scale = fp32 ? 1.0f : half_scale_from_absmax(dev::device_abs_max(val, nnz, st));
        // The band height, and for the default plans whether BAND joins them (as for an upload).
        int band_rows = o.band_rows;
        if ((band_rows == 0 && (plans & kTensorPlans)) || (o.plans == 0 && !fp32)) {
            const dev::BandChoice bc = dev::choose_band_device(row_ptr, col, M, st);
            if (band_rows == 0) band_rows = bc.band_rows;
            if (o.plans == 0 && !fp32 && bc.entries_per_tile >= dev::kBandMinEntriesPerTile)
                plans |= 1 << VCSRMC_PLAN_BAND;
            else if (o.plans == 0 && !fp32 && bc.dense_fraction >= dev::kHybridMinDenseFraction)
                plans |= 1 << VCSRMC_PLAN_HYBRID;
        }
        auto* d = new vcsrmc_device_format;
        d->device = device;
        d->M = M;
        d->N = N;
        d->segw = segw;
        d->num_segments = (N + segw - 1) / segw;
        d->fp32 = fp32 ? 1 : 0;
        d->scale = scale;
        try {
            dev::SegmentLayout seg;
            dev::RowsLayout rows;
            if (plans & (1 << VCSRMC_PLAN_SEGMENT)) {
                seg = dev::build_segment_layout(row_ptr, col, val, M, N, nnz, segw, fp32 != 0, scale, st);
                d->items = seg.items;
                d->gmeta = seg.gmeta;
                d->grows = seg.grows;
                d->lcol = seg.lcol;
                d->val = seg.val;
                d->n_groups = seg.n_groups;
                d->n_slots = seg.n_slots;
                d->n_items = seg.n_items;
                d->has_segment = true;
            }
            if (plans & (1 << VCSRMC_PLAN_ROWS)) {
                if (unit_nnz == 0) {
                    int sms = 0;
                    cuda_check(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device),
                               "cudaDeviceGetAttribute");
                    unit_nnz = dev::choose_unit_nnz(nnz, sms);
                }
                rows = dev::build_rows_layout(row_ptr, col, val, M, nnz, fp32 != 0, scale, unit_nnz, st);
                d->rp = rows.rp;
                d->cols = rows.cols;
                d->rvals = rows.vals;
                d->units = rows.units;
                d->n_units = rows.n_units;
                d->split_rows = rows.split_rows;
                d->n_split_rows = rows.n_split_rows;
                d->unit_nnz = unit_nnz;
                d->has_rows = true;
            }
            if (!dev::device_validate(d->has_segment ? &seg : nullptr, d->has_rows ? &rows : nullptr, M, N, segw, st))
                throw StatusError(VCSRMC_INTERNAL, "device-built format failed its index checks");
            make_hot_columns(d, nnz, o, st);
            if (plans & kTensorPlans) {
                dev::BandLayout band = dev::build_band_layout(row_ptr, col, val, M, nnz, scale, band_rows, st);
                // the handle owns the full band layout from here (freed with it if BAND is not kept)
                d->band_rows = band.band_rows;
                d->n_bands = band.n_bands;
                d->n_tiles = band.n_tiles;
                d->tile_ptr = band.tile_ptr;
                d->tile_col = band.tile_col;
                d->tile_eptr = band.tile_eptr;
                d->ents = band.ents;
                if (plans & (1 << VCSRMC_PLAN_HYBRID)) {
                    if (unit_nnz == 0) {
                        int sms = 0;
                        cuda_check(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device),
                                   "cudaDeviceGetAttribute");
                        unit_nnz = dev::choose_unit_nnz(nnz, sms);
                    }
                    dev::HybridLayout h = dev::build_hybrid_layout(band, M, N, nnz, int(dev::kBandMinEntriesPerTile),
                                                                   unit_nnz, st);
                    d->hb_rows = h.dense.band_rows;
                    d->hb_bands = h.dense.n_bands;
                    d->hb_tiles = h.dense.n_tiles;
                    d->hb_nnz = h.dense_nnz;
                    d->hb_tile_ptr = h.dense.tile_ptr;
                    d->hb_tile_col = h.dense.tile_col;
                    d->hb_tile_eptr = h.dense.tile_eptr;
                    d->hb_ents = h.dense.ents;
                    d->hr_nnz = h.resid_nnz;
                    d->hr_rp = h.resid.rp;
                    d->hr_cols = h.resid.cols;
                    d->hr_vals = h.resid.vals;
                    d->hr_units = h.resid.units;
                    d->hr_n_units = h.resid.n_units;
                    d->hr_split = h.resid.split_rows;
                    d->hr_n_split = h.resid.n_split_rows;
                    d->has_hybrid = true;
                }
                if (plans & (1 << VCSRMC_PLAN_BAND)) {
                    d->has_band = true;
                } else {
                    cudaFree(d->tile_ptr);
                    cudaFree(d->tile_col);
                    cudaFree(d->tile_eptr);
                    cudaFree(d->ents);
                    d->tile_ptr = d->tile_col = d->tile_eptr = nullptr;
                    d->ents = nullptr;
                    d->band_rows = d->n_bands = 0;
                    d->n_tiles = 0;
                }
            }
            cuda_check(cudaMalloc(&d->status, sizeof(uint32_t)), "cudaMalloc");
            cuda_check(cudaMemsetAsync(d->status, 0, sizeof(uint32_t), st), "cudaMemsetAsync");
            cuda_check(cudaStreamSynchronize(st), "cudaStreamSynchronize");
        } catch (...) {
            free_device(d);
            throw;
        }
        *out = d;
    });
}

VCSRMC_EXPORT int vcsrmc_device_download(const vcsrmc_device_format* d, vcsrmc_format** out) {
    return guarded([&] {
        if (!d || !out) throw StatusError(VCSRMC_INVALID_ARG, "NULL argument");
        if (!d->has_segment) throw StatusError(VCSRMC_INVALID_ARG, "the SEGMENT plan layout is not resident");
        DeviceGuard guard(d->device);
        const int64_t G = d->n_groups, S = d->n_slots, I = d->n_items;
        std::vector<int4> gmeta(static_cast<size_t>(G));
        std::vector<int2> items(static_cast<size_t>(I));
        std::vector<int8_t> lcol(static_cast<size_t>(S));
        auto* f = new vcsrmc_format;
        try {
            VCSRMC& v = f->v;
            v.M = d->M;
            v.N = d->N;
            v.segw = d->segw;
            v.bundle = 16;
            v.num_segments = d->num_segments;
            v.fp32 = d->fp32 != 0;
            v.scale = d->scale;
            v.group_rows.resize(size_t(G) * 16);
            v.val.resize(size_t(S));
            if (G) {
                cuda_check(cudaMemcpy(gmeta.data(), d->gmeta, sizeof(int4) * size_t(G), cudaMemcpyDeviceToHost), "cudaMemcpy");
                cuda_check(cudaMemcpy(v.group_rows.data(), d->grows, sizeof(int) * size_t(G) * 16, cudaMemcpyDeviceToHost),
                           "cudaMemcpy");
            }
            if (I) cuda_check(cudaMemcpy(items.data(), d->items, sizeof(int2) * size_t(I), cudaMemcpyDeviceToHost), "cudaMemcpy");
            if (S) {
                cuda_check(cudaMemcpy(lcol.data(), d->lcol, size_t(S), cudaMemcpyDeviceToHost), "cudaMemcpy");
                if (d->fp32) {
                    cuda_check(cudaMemcpy(v.val.data(), d->val, sizeof(float) * size_t(S), cudaMemcpyDeviceToHost), "cudaMemcpy");
                } else {
                    std::vector<__half> h(static_cast<size_t>(S));
                    cuda_check(cudaMemcpy(h.data(), d->val, sizeof(__half) * size_t(S), cudaMemcpyDeviceToHost), "cudaMemcpy");
                    for (int64_t i = 0; i < S; ++i) v.val[size_t(i)] = __half2float(h[size_t(i)]);
                }
            }
            v.group_ptr.resize(size_t(G) + 1);
            v.group_depth.resize(size_t(G));
            v.group_seg_base.resize(size_t(G));
            for (int64_t g = 0; g < G; ++g) {
                v.group_ptr[size_t(g)] = gmeta[size_t(g)].x;
                v.group_depth[size_t(g)] = gmeta[size_t(g)].y;
                v.group_seg_base[size_t(g)] = gmeta[size_t(g)].z;
            }
            v.group_ptr[size_t(G)] = int(S);
            v.lcol.assign(lcol.begin(), lcol.end());
            v.item_gbeg.resize(size_t(I));
            v.item_gend.resize(size_t(I));
            for (int64_t i = 0; i < I; ++i) {
                v.item_gbeg[size_t(i)] = items[size_t(i)].x;
                v.item_gend[size_t(i)] = items[size_t(i)].y;
            }
        } catch (...) {
            delete f;
            throw;
        }
        *out = f;
    });
}

VCSRMC_EXPORT int vcsrmc_half_scale_device(const float* val, int64_t nnz, void* stream, float* scale) {
    return guarded([&] {
        if (!scale || nnz < 0 || (nnz > 0 && !val)) throw StatusError(VCSRMC_INVALID_ARG, "bad arguments");
        static std::mutex scratch_mu;  // one scratch word per device: calls do not overlap
        std::lock_guard<std::mutex> lock(scratch_mu);
        *scale = half_scale_from_absmax(dev::device_abs_max_noalloc(val, nnz, static_cast<cudaStream_t>(stream)));
    });
}
