// TEST INFRASTRUCTURE — BASELINE ONLY. Not part of the product library (vcsr_mc_b200).
//
// Times the reference's own CUDA tensor-core kernel (reference/vcsr_tc.cu: csr_to_vcsr_tc,
// vcsr_tc_kernel, run_vcsr_tc_spmm_gpu; WMMA 16x16x16, segment width 16, fp32 B converted to
// half in shared memory, atomic adds into C) on this GPU, as a GPU-side baseline next to the
// library's kernels. The reference file is compiled from where it lies in the reference checkout
// (oracle/Makefile); nothing of it is copied here.
//
//   oracle/_ref/ref_tc_bench A.csr [O=128] [repeat=10] [warmup=3]
// A.csr is a binary CSR written by vcsrmc_csr_save / vm.CSR.save. B is U(-1,1) fp32 from a
// fixed LCG; C is zeroed before every launch (the kernel accumulates). Prints the median of the
// kernel times the reference's own run function reports, and the largest error of 256 sampled
// rows against an fp64 CPU product, scaled by sum |a||b| (the FP16 tolerance is 2e-2).
#include "vcsr_tc.cu"

#include <cmath>
#include <cstdint>
#include <cstring>
#include <string>

namespace {

bool load_csr(const char* path, CSR& A) {
    FILE* f = std::fopen(path, "rb");
    if (!f) return false;
    char magic[8];
    int64_t hdr[3];
    bool ok = std::fread(magic, 1, 8, f) == 8 && std::memcmp(magic, "VCSRMC1", 8) == 0 &&
              std::fread(hdr, 8, 3, f) == 3 && hdr[0] >= 0 && hdr[1] >= 0 && hdr[2] >= 0 && hdr[0] < INT32_MAX &&
              hdr[1] < INT32_MAX && hdr[2] <= INT32_MAX;
    if (ok) {
        A.M = int(hdr[0]);
        A.N = int(hdr[1]);
        A.nnz = int(hdr[2]);
        A.row_ptr.resize(size_t(A.M) + 1);
        A.col.resize(size_t(A.nnz));
        A.val.resize(size_t(A.nnz));
        ok = std::fread(A.row_ptr.data(), 4, A.row_ptr.size(), f) == A.row_ptr.size() &&
             std::fread(A.col.data(), 4, A.col.size(), f) == A.col.size() &&
             std::fread(A.val.data(), 4, A.val.size(), f) == A.val.size();
    }
    std::fclose(f);
    if (!ok || A.row_ptr[0] != 0 || A.row_ptr[size_t(A.M)] != A.nnz) return false;
    for (int r = 0; r < A.M; ++r)
        if (A.row_ptr[size_t(r) + 1] < A.row_ptr[size_t(r)]) return false;
    for (const int c : A.col)
        if (c < 0 || c >= A.N) return false;
    return true;
}

}  // namespace

int main(int argc, char** argv) {
    if (argc < 2) {
        std::fprintf(stderr, "usage: %s A.csr [O] [repeat] [warmup]\n", argv[0]);
        return 2;
    }
    const int O = argc > 2 ? std::atoi(argv[2]) : 128;
    const int repeat = argc > 3 ? std::atoi(argv[3]) : 10;
    const int warmup = argc > 4 ? std::atoi(argv[4]) : 3;
    CSR A;
    if (O < 1 || repeat < 1 || warmup < 0 || !load_csr(argv[1], A)) {
        std::fprintf(stderr, "bad arguments or CSR file\n");
        return 2;
    }
    if (int64_t(A.N) * O >= INT32_MAX || int64_t(A.M) * O >= INT32_MAX) {
        std::fprintf(stderr, "the reference kernel indexes B and C with 32-bit ints: N*O and M*O must fit\n");
        return 2;
    }
    VCSRTC V = csr_to_vcsr_tc(A, 16);
    std::vector<float> hB(size_t(A.N) * O);
    uint64_t s = 0x9e3779b97f4a7c15ull;
    for (float& x : hB) {
        s = s * 6364136223846793005ull + 1442695040888963407ull;
        x = float(double(s >> 11) / double(1ull << 53) * 2.0 - 1.0);
    }
    float *dB = nullptr, *dC = nullptr;
    const size_t cbytes = sizeof(float) * size_t(A.M) * O;
    if (cudaMalloc(&dB, sizeof(float) * hB.size()) != cudaSuccess || cudaMalloc(&dC, cbytes) != cudaSuccess) {
        std::fprintf(stderr, "device allocation failed\n");
        return 1;
    }
    cudaMemcpy(dB, hB.data(), sizeof(float) * hB.size(), cudaMemcpyHostToDevice);
    std::vector<float> times;
    for (int i = 0; i < warmup + repeat; ++i) {
        cudaMemset(dC, 0, cbytes);
        float ms = 0.f;
        run_vcsr_tc_spmm_gpu(V, dB, O, dC, 0, ms);
        if (i >= warmup) times.push_back(ms);
    }
    const cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        std::fprintf(stderr, "CUDA error: %s\n", cudaGetErrorString(e));
        return 1;
    }
    std::vector<float> hC(size_t(A.M) * O);
    cudaMemcpy(hC.data(), dC, cbytes, cudaMemcpyDeviceToHost);
    destroy_vcsr_tc_device(0);
    cudaFree(dB);
    cudaFree(dC);
    std::sort(times.begin(), times.end());
    const double med = times[times.size() / 2];
    double worst = 0.0;
    for (int k = 0; k < 256 && A.M > 0; ++k) {
        const int r = int((int64_t(k) * 2654435761ll) % A.M);
        for (int j = 0; j < O; ++j) {
            double ref = 0.0, mag = 0.0;
            for (int p = A.row_ptr[size_t(r)]; p < A.row_ptr[size_t(r) + 1]; ++p) {
                const double t = double(A.val[size_t(p)]) * double(hB[size_t(A.col[size_t(p)]) * O + j]);
                ref += t;
                mag += std::fabs(t);
            }
            const double err = std::fabs(double(hC[size_t(r) * O + j]) - ref) / (mag > 0 ? mag : 1.0);
            worst = std::max(worst, err);
        }
    }
    std::printf("ref_tc M=%d N=%d nnz=%d O=%d groups=%zu median_ms=%.4f gflops=%.1f max_scaled_err=%.3e\n", A.M, A.N,
                A.nnz, O, V.group_depth.size(), med, 2.0 * A.nnz * O / (med * 1e6), worst);
    return 0;
}
