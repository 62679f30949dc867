// Comparison-only library (libvcsrmc_cusparse.so): times NVIDIA cuSPARSE's CSR SpMM on the same
// device buffers, for the "next to a cuSPARSE SpMM number" rows of the benchmark and driver.
// Mirrors the reference's hipSPARSE baseline (src/kernels.cu:60-206): FP32 A/B/C, and FP16 A/B
// with FP32 compute and C (alpha = half_scale factor). Not part of the product path.
#include <cuda_runtime.h>
#include <cusparse.h>

#include <algorithm>
#include <cstdint>
#include <cstdio>
#include <vector>

#define CMP_API extern "C" __attribute__((visibility("default")))

namespace {
int g_last = 0;
char g_msg[256] = {0};
int failed(int code, const char* what) {
    g_last = code;
    std::snprintf(g_msg, sizeof g_msg, "%s (status %d)", what, code);
    return code;
}
}  // namespace

CMP_API const char* vcsrmc_cusparse_last_error(void) { return g_msg; }

// C[M x O] = alpha * A * B with cusparseSpMM (default algorithm); val_f16 / b_f16 select fp16 A
// values / B. Runs `warmup` untimed and `reps` timed launches on `stream`; returns the median
// launch time in *ms_median. Descriptor creation, buffer sizing and preprocessing are outside
// the timed launches (as in the reference's setup_ms).
CMP_API int vcsrmc_cusparse_spmm(int32_t M, int32_t N, int64_t nnz, const int32_t* d_rowptr, const int32_t* d_col,
                                 const void* d_val, int val_f16, const void* d_B, int b_f16, int32_t O, float* d_C,
                                 float alpha, int warmup, int reps, void* stream, float* ms_median) {
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    cusparseHandle_t h = nullptr;
    cusparseSpMatDescr_t A = nullptr;
    cusparseDnMatDescr_t Bd = nullptr, Cd = nullptr;
    void* buf = nullptr;
    int rc = 0;
    cusparseStatus_t s;
    size_t bytes = 0;
    const float beta = 0.f;
    std::vector<float> times;
    cudaEvent_t e0 = nullptr, e1 = nullptr;
#define CK(x, what)                                  \
    if ((s = (x)) != CUSPARSE_STATUS_SUCCESS) {      \
        rc = failed(int(s), what);                   \
        goto done;                                   \
    }
    CK(cusparseCreate(&h), "cusparseCreate");
    CK(cusparseSetStream(h, st), "cusparseSetStream");
    CK(cusparseCreateCsr(&A, M, N, nnz, const_cast<int32_t*>(d_rowptr), const_cast<int32_t*>(d_col),
                         const_cast<void*>(d_val), CUSPARSE_INDEX_32I, CUSPARSE_INDEX_32I, CUSPARSE_INDEX_BASE_ZERO,
                         val_f16 ? CUDA_R_16F : CUDA_R_32F),
       "cusparseCreateCsr");
    CK(cusparseCreateDnMat(&Bd, N, O, O, const_cast<void*>(d_B), b_f16 ? CUDA_R_16F : CUDA_R_32F, CUSPARSE_ORDER_ROW),
       "cusparseCreateDnMat(B)");
    CK(cusparseCreateDnMat(&Cd, M, O, O, d_C, CUDA_R_32F, CUSPARSE_ORDER_ROW), "cusparseCreateDnMat(C)");
    CK(cusparseSpMM_bufferSize(h, CUSPARSE_OPERATION_NON_TRANSPOSE, CUSPARSE_OPERATION_NON_TRANSPOSE, &alpha, A, Bd,
                               &beta, Cd, CUDA_R_32F, CUSPARSE_SPMM_ALG_DEFAULT, &bytes),
       "cusparseSpMM_bufferSize");
    if (bytes && cudaMalloc(&buf, bytes) != cudaSuccess) {
        rc = failed(-1, "cudaMalloc(workspace)");
        goto done;
    }
    CK(cusparseSpMM_preprocess(h, CUSPARSE_OPERATION_NON_TRANSPOSE, CUSPARSE_OPERATION_NON_TRANSPOSE, &alpha, A, Bd,
                               &beta, Cd, CUDA_R_32F, CUSPARSE_SPMM_ALG_DEFAULT, buf),
       "cusparseSpMM_preprocess");
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    for (int i = 0; i < warmup + reps; ++i) {
        cudaEventRecord(e0, st);
        CK(cusparseSpMM(h, CUSPARSE_OPERATION_NON_TRANSPOSE, CUSPARSE_OPERATION_NON_TRANSPOSE, &alpha, A, Bd, &beta, Cd,
                        CUDA_R_32F, CUSPARSE_SPMM_ALG_DEFAULT, buf),
           "cusparseSpMM");
        cudaEventRecord(e1, st);
        cudaEventSynchronize(e1);
        float ms = 0.f;
        cudaEventElapsedTime(&ms, e0, e1);
        if (i >= warmup) times.push_back(ms);
    }
    std::sort(times.begin(), times.end());
    *ms_median = times.empty() ? 0.f : times[times.size() / 2];
done:
#undef CK
    if (e0) cudaEventDestroy(e0);
    if (e1) cudaEventDestroy(e1);
    if (buf) cudaFree(buf);
    if (Cd) cusparseDestroyDnMat(Cd);
    if (Bd) cusparseDestroyDnMat(Bd);
    if (A) cusparseDestroySpMat(A);
    if (h) cusparseDestroy(h);
    if (rc == 0 && cudaGetLastError() != cudaSuccess) rc = failed(-2, "CUDA error");
    return rc;
}
