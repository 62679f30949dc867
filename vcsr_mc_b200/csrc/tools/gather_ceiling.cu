// gather_ceiling: the achievable rate of random 256-byte row gathers on this GPU (the memory
// pattern of the ROWS SpMM plan, without its sparse bookkeeping). B = 2^24 rows x 128 fp16
// (4.3 GB); 2^26 row indices drawn uniformly from the first `span` rows (mode 0: all rows,
// 1: 2^20 rows = 268 MB, 2: 2^17 rows = 34 MB, i.e. L2-resident). A 16-lane group loads 16
// indices coalesced and gathers them in rounds of 8 rows whose loads are issued together; each
// lane sums its 16 bytes of each row. Reports rows/s and gathered TB/s per launch shape.
//   vcsr_mc_b200/gather_ceiling [mode]
#include <cuda_fp16.h>
#include <cstdio>
#include <cstdint>
#include <cstdlib>
#include <vector>
#include <random>

__device__ __forceinline__ void ld8(const uint4* p0, const uint4* p1, const uint4* p2, const uint4* p3,
                                    const uint4* p4, const uint4* p5, const uint4* p6, const uint4* p7, uint4 (&r)[8]) {
    asm volatile(
        "ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%32];\n\t"
        "ld.global.nc.v4.u32 {%4,%5,%6,%7}, [%33];\n\t"
        "ld.global.nc.v4.u32 {%8,%9,%10,%11}, [%34];\n\t"
        "ld.global.nc.v4.u32 {%12,%13,%14,%15}, [%35];\n\t"
        "ld.global.nc.v4.u32 {%16,%17,%18,%19}, [%36];\n\t"
        "ld.global.nc.v4.u32 {%20,%21,%22,%23}, [%37];\n\t"
        "ld.global.nc.v4.u32 {%24,%25,%26,%27}, [%38];\n\t"
        "ld.global.nc.v4.u32 {%28,%29,%30,%31}, [%39];\n\t"
        : "=r"(r[0].x), "=r"(r[0].y), "=r"(r[0].z), "=r"(r[0].w), "=r"(r[1].x), "=r"(r[1].y), "=r"(r[1].z), "=r"(r[1].w),
          "=r"(r[2].x), "=r"(r[2].y), "=r"(r[2].z), "=r"(r[2].w), "=r"(r[3].x), "=r"(r[3].y), "=r"(r[3].z), "=r"(r[3].w),
          "=r"(r[4].x), "=r"(r[4].y), "=r"(r[4].z), "=r"(r[4].w), "=r"(r[5].x), "=r"(r[5].y), "=r"(r[5].z), "=r"(r[5].w),
          "=r"(r[6].x), "=r"(r[6].y), "=r"(r[6].z), "=r"(r[6].w), "=r"(r[7].x), "=r"(r[7].y), "=r"(r[7].z), "=r"(r[7].w)
        : "l"(p0), "l"(p1), "l"(p2), "l"(p3), "l"(p4), "l"(p5), "l"(p6), "l"(p7));
}

// R rounds of 8 per batch of 16 indices; kDouble: issue round r+1 before consuming round r
template <int WPB, bool kDouble>
__global__ void __launch_bounds__(WPB * 32) gather16(const uint4* __restrict__ B, const unsigned* __restrict__ idx,
                                                     long long n, float* __restrict__ out, int per_group) {
    const int lane = threadIdx.x & 31, sub = lane >> 4, sl = lane & 15;
    const unsigned gmask = 0xffffu << (16 * sub);
    const long long g = (long long)(blockIdx.x * WPB + (threadIdx.x >> 5)) * 2 + sub;
    const long long p0 = g * per_group;
    if (p0 >= n) return;
    const long long p1 = p0 + per_group < n ? p0 + per_group : n;
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    auto consume = [&](const uint4 (&r)[8]) {
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const __half2* h = reinterpret_cast<const __half2*>(&r[k]);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                float2 f = __half22float2(h[i]);
                acc[2 * i] += f.x;
                acc[2 * i + 1] += f.y;
            }
        }
    };
    for (long long p = p0; p < p1; p += 16) {
        const unsigned myrow = (p + sl < p1) ? __ldcs(idx + p + sl) : 0u;
        const uint4* a[16];
#pragma unroll
        for (int k = 0; k < 16; ++k) a[k] = B + (size_t)__shfl_sync(gmask, myrow, k, 16) * 16 + sl;
        uint4 r0[8], r1[8];
        ld8(a[0], a[1], a[2], a[3], a[4], a[5], a[6], a[7], r0);
        if (kDouble) {
            ld8(a[8], a[9], a[10], a[11], a[12], a[13], a[14], a[15], r1);
            consume(r0);
            consume(r1);
        } else {
            consume(r0);
            ld8(a[8], a[9], a[10], a[11], a[12], a[13], a[14], a[15], r1);
            consume(r1);
        }
    }
    float s = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) s += acc[i];
    if (s == 12345.f) out[g] = s;  // keep the loads alive
}

template <int WPB, bool kDouble>
void run(const uint4* B, const unsigned* idx, long long n, float* out, const char* name) {
    const int per_group = 256;
    const long long groups = (n + per_group - 1) / per_group;
    const long long blocks = (groups + 2 * WPB - 1) / (2 * WPB);
    cudaEvent_t a, b; cudaEventCreate(&a); cudaEventCreate(&b);
    for (int w = 0; w < 2; ++w) gather16<WPB, kDouble><<<blocks, WPB * 32>>>(B, idx, n, out, per_group);
    cudaEventRecord(a);
    const int reps = 5;
    for (int w = 0; w < reps; ++w) gather16<WPB, kDouble><<<blocks, WPB * 32>>>(B, idx, n, out, per_group);
    cudaEventRecord(b); cudaEventSynchronize(b);
    float ms; cudaEventElapsedTime(&ms, a, b);
    int nb = 0; cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, gather16<WPB, kDouble>, WPB * 32, 0);
    cudaFuncAttributes fa; cudaFuncGetAttributes(&fa, gather16<WPB, kDouble>);
    ms /= reps;
    printf("%-8s WPB=%2d regs=%3d warps/SM=%2d : %.3f ms  %6.2f G rows/s  %.2f TB/s\n", name, WPB, fa.numRegs, nb * WPB, ms,
           n / (ms * 1e6), n * 256.0 / (ms * 1e9));
}

int main(int argc, char** argv) {
    const long long nrows = 1LL << 24;  // 16.8M rows x 256 B = 4.3 GB
    const long long n = 1LL << 26;      // gathers
    const int mode = argc > 1 ? atoi(argv[1]) : 0;
    uint4* B; unsigned* idx; float* out;
    if (cudaMalloc(&B, nrows * 256) != cudaSuccess) { printf("oom\n"); return 1; }
    cudaMemset(B, 0, nrows * 256);
    cudaMalloc(&idx, n * 4); cudaMalloc(&out, 1 << 24);
    std::vector<unsigned> h(n);
    std::mt19937_64 rng(1);
    const long long span = mode == 0 ? nrows : (mode == 1 ? (1LL << 20) : (1LL << 17));
    for (auto& x : h) x = unsigned(rng() % span);
    cudaMemcpy(idx, h.data(), n * 4, cudaMemcpyHostToDevice);
    printf("mode %d: rows uniform over %lld (%.0f MB)\n", mode, span, span * 256.0 / 1e6);
    run<8, false>(B, idx, n, out, "single");
    run<8, true>(B, idx, n, out, "double");
    run<4, true>(B, idx, n, out, "double");
    run<16, true>(B, idx, n, out, "double");
    run<16, false>(B, idx, n, out, "single");
    cudaError_t e = cudaDeviceSynchronize();
    printf("status %s\n", cudaGetErrorString(e));
    return e == cudaSuccess ? 0 : 1;
}
