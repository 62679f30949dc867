// The reference's device entry points, same names and semantics, over the C ABI (vcsrmc.h):
//   upload_vcsr_mc_device(V)                          src/vcsr_mc.cu:332-349
//   run_vcsr_mc_spmm_gpu(V, dB, O, tileK, dC, st, ms) src/vcsr_mc.cu:352-394
//   destroy_vcsr_mc_device(st)                        src/vcsr_mc.cu:397-404
// As in the reference there is one uploaded format per process at a time (these functions keep
// it in a file-local handle, are not thread-safe, and upload lazily on the first launch), C is
// accumulated (C += A*B, the caller zeroes it), B and C are fp32 with ldb = ldc = O, the launch
// is timed with events and blocks. Errors throw std::runtime_error instead of exiting.
// New code should call the C ABI directly (handles, streams, plans, fp16 B).
#pragma once
#include <cstdint>
#include <stdexcept>
#include <string>

#include "../vcsrmc.h"
#include "vcsr_formats.hpp"

typedef struct CUstream_st* cudaStream_t;

namespace vcsrmc {
namespace compat_detail {
inline vcsrmc_format*& host_handle() {
    static vcsrmc_format* h = nullptr;
    return h;
}
inline vcsrmc_device_format*& device_handle() {
    static vcsrmc_device_format* h = nullptr;
    return h;
}
inline void check(int status) {
    if (status != VCSRMC_OK) {
        char msg[512];
        vcsrmc_last_error(msg, sizeof msg);
        throw std::runtime_error(std::string("vcsrmc: ") + msg);
    }
}
}  // namespace compat_detail

inline void upload_vcsr_mc_device(const VCSRMC& V) {
    using namespace compat_detail;
    if (device_handle()) return;  // already uploaded (the reference keeps the first upload too)
    vcsrmc_format_view v{};
    v.M = V.M;
    v.N = V.N;
    v.segw = V.segw;
    v.bundle = V.bundle;
    v.num_segments = V.num_segments;
    v.fp32 = V.fp32 ? 1 : 0;
    v.scale = V.scale;
    v.n_groups = int64_t(V.group_depth.size());
    v.n_slots = int64_t(V.lcol.size());
    v.n_items = int64_t(V.item_gbeg.size());
    v.group_ptr = V.group_ptr.data();
    v.group_depth = V.group_depth.data();
    v.group_seg_base = V.group_seg_base.data();
    v.group_rows = V.group_rows.data();
    v.lcol = V.lcol.data();
    v.val = V.val.data();
    v.item_gbeg = V.item_gbeg.data();
    v.item_gend = V.item_gend.data();
    check(vcsrmc_format_from_view(&v, &host_handle()));
    // -1: the caller's current device, which is where the reference's hipMalloc allocates
    check(vcsrmc_upload(host_handle(), -1, nullptr, &device_handle()));
}

inline void run_vcsr_mc_spmm_gpu(const VCSRMC& V, const float* dB, int O, int tileK, float* dC, cudaStream_t st,
                                 float& ms) {
    using namespace compat_detail;
    if (V.item_gbeg.empty()) { ms = 0.f; return; }
    if (!device_handle()) upload_vcsr_mc_device(V);
    check(vcsrmc_spmm_timed(device_handle(), dB, VCSRMC_F32, O, O, tileK, dC, O, 1, st, &ms));
}

inline void destroy_vcsr_mc_device(cudaStream_t) {
    using namespace compat_detail;
    if (device_handle()) check(vcsrmc_device_free(device_handle()));
    device_handle() = nullptr;
    vcsrmc_format_free(host_handle());
    host_handle() = nullptr;
}

}  // namespace vcsrmc
