// Host side of the TMA loads: the driver's tensor-map encoder (looked up once through the
// runtime) and the map for a row-major fp16 B read as boxes of `box_rows` rows x 64 columns with
// the 128-byte swizzle (the tcgen05 B operand, MN-major).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cstdint>
#include <cstring>
#include <mutex>

namespace vcsrmc {
namespace dev {

inline PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

// B: rows x O fp16, row pitch ldb elements. False when the layout cannot be read by TMA (base
// not 16-byte aligned, pitch not a multiple of 16 bytes, fewer than 64 columns or fewer rows
// than one box) or the encoder is unavailable; the kernels then stage B with plain loads.
// Boxes start at column multiples of 64 (128 bytes) only, which keeps the innermost TMA
// coordinate 16-byte aligned. Rows >= `rows` and columns >= O read as zero.
inline bool encode_b_tmap_f16(CUtensorMap* tmap, const void* B, int64_t ldb, int O, int64_t rows, int box_rows) {
    std::memset(tmap, 0, sizeof(*tmap));
    const bool ok = (reinterpret_cast<uintptr_t>(B) & 15) == 0 && ((ldb * 2) & 15) == 0 && ldb >= O && O >= 64 &&
                    rows >= box_rows;
    if (!ok) return false;
    PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
    if (!enc) return false;
    const cuuint64_t dims[2] = {cuuint64_t(O), cuuint64_t(rows)};
    const cuuint64_t strides[1] = {cuuint64_t(ldb) * 2};
    const cuuint32_t box[2] = {64u, cuuint32_t(box_rows)};
    const cuuint32_t estr[2] = {1u, 1u};
    const CUresult r = enc(tmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(B), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

}  // namespace dev
}  // namespace vcsrmc
