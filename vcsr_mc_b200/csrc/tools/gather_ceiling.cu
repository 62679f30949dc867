// gather_ceiling: the achievable rate of random 256-byte row gathers on this GPU (the memory
// pattern of the ROWS SpMM plan, without its sparse bookkeeping). B = 2^24 rows x 128 fp16
// (4.3 GB); 2^26 row indices drawn uniformly from the first `span` rows (mode 0: all rows,
// 1: 2^20 rows = 268 MB, 2: 2^17 rows = 34 MB, i.e. L2-resident). Two ways to gather:
//   * registers: a 16-lane group loads 16 indices coalesced (one round ahead) and gathers them in
//     rounds of 8 rows whose loads are issued together; each lane sums its 16 bytes of each row;
//   * TMA tile::gather4: each warp keeps a ring of kDepth 1-KB slots in shared memory, lane 0
//     fills a slot with four B rows per instruction (completion on the slot's mbarrier) and the
//     warp sums the slot, so the rows in flight per SM are set by shared memory, not registers.
// B holds ((r % 61) + (c % 3)) / 64, so the exact sum of every gathered row is known on the host
// and the TMA path's result is checked against it. A hybrid CTA runs both kinds of warps on
// chunks of indices taken from a shared counter, to see whether the two paths add up. Reports
// rows/s and gathered TB/s per shape.
// Mode 3 gathers a given index stream instead, in its order: an int32 .npy file of row indices
// below 2^24 (e.g. the column array of a CSR, as the ROWS plan walks it), register gathers only.
//   vcsr_mc_b200/gather_ceiling [mode] [indices.npy]
#include <cuda_fp16.h>
#include <cuda.h>
#include <cstdio>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>
#include <random>

#include "../cuda/common.cuh"
#include "../cuda/tma_host.hpp"

using namespace vcsrmc::dev;

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

// R rounds of 8 per batch of 16 indices; kDouble: issue round r+1 before consuming round r.
// kWriteRows: after each batch of 16 the group also stores its 16 x 8 fp32 sums as one 512-byte
// row of `rows_out` (row p / 16, streaming stores), the C stream of the SpMM.
template <int WPB, bool kDouble, bool kWriteRows = false>
__global__ void __launch_bounds__(WPB * 32) gather16(const uint4* __restrict__ B, const unsigned* __restrict__ idx,
                                                     long long n, float* __restrict__ out, int per_group,
                                                     float* __restrict__ rows_out = nullptr) {
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
    unsigned nextrow = (p0 + sl < p1) ? __ldcs(idx + p0 + sl) : 0u;
    for (long long p = p0; p < p1; p += 16) {
        const unsigned myrow = nextrow;  // loaded one round ahead
        nextrow = (p + 16 + sl < p1) ? __ldcs(idx + p + 16 + sl) : 0u;
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
        if (kWriteRows) {
            float4* dst = reinterpret_cast<float4*>(rows_out + (size_t)(p >> 4) * 128 + sl * 8);
            __stcs(dst, make_float4(acc[0], acc[1], acc[2], acc[3]));
            __stcs(dst + 1, make_float4(acc[4], acc[5], acc[6], acc[7]));
#pragma unroll
            for (int i = 0; i < 8; ++i) acc[i] = 0.f;
        }
    }
    float s = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) s += acc[i];
    if (s == 12345.f) out[g] = s;  // keep the loads alive
}

template <int WPB, bool kDouble, bool kWriteRows = false>
void run(const uint4* B, const unsigned* idx, long long n, float* out, const char* name, float* rows_out = nullptr) {
    const int per_group = 256;
    const long long groups = (n + per_group - 1) / per_group;
    const long long blocks = (groups + 2 * WPB - 1) / (2 * WPB);
    auto k = gather16<WPB, kDouble, kWriteRows>;
    cudaEvent_t a, b; cudaEventCreate(&a); cudaEventCreate(&b);
    for (int w = 0; w < 2; ++w) k<<<blocks, WPB * 32>>>(B, idx, n, out, per_group, rows_out);
    cudaEventRecord(a);
    const int reps = 5;
    for (int w = 0; w < reps; ++w) k<<<blocks, WPB * 32>>>(B, idx, n, out, per_group, rows_out);
    cudaEventRecord(b); cudaEventSynchronize(b);
    float ms; cudaEventElapsedTime(&ms, a, b);
    int nb = 0; cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, k, WPB * 32, 0);
    cudaFuncAttributes fa; cudaFuncGetAttributes(&fa, k);
    ms /= reps;
    printf("%-8s WPB=%2d regs=%3d warps/SM=%2d : %.3f ms  %6.2f G rows/s  %.2f TB/s\n", name, WPB, fa.numRegs, nb * WPB, ms,
           n / (ms * 1e6), n * 256.0 / (ms * 1e9));
}

__global__ void fill_b(__half* B, long long nrows) {
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < nrows * 128; i += (long long)gridDim.x * blockDim.x)
        B[i] = __float2half(float((i / 128) % 61 + (i % 128) % 3) / 64.f);
}

// kWarps warps per CTA, each with its own ring of kDepth slots; warp w of CTA b gathers indices
// [p0, p0 + per_warp), p0 = (b * kWarps + w) * per_warp, four per slot. Every wait is bounded: on
// expiry the warp drains what it issued (bounded), sets *err and stops.
template <int kWarps, int kDepth>
__global__ void __launch_bounds__(kWarps * 32) gather4_tma(const __grid_constant__ CUtensorMap tmap,
                                                           const uint4* __restrict__ idx4, long long n, int per_warp,
                                                           double* __restrict__ out, int* err) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    uint8_t* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint8_t* ring = smem + warp * kDepth * 1024;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kWarps * kDepth * 1024) + warp * kDepth;
    const long long gw = (long long)blockIdx.x * kWarps + warp;
    const long long p0 = gw * per_warp;
    if (p0 >= n) return;
    const long long p1 = p0 + per_warp < n ? p0 + per_warp : n;
    const int nq = int((p1 - p0) / 4);
    const long long g0 = p0 / 4;
    if (lane == 0) {
        for (int s = 0; s < kDepth; ++s) mbar_init(&bars[s], 1);
        fence_mbar_init();
        prefetch_tmap(&tmap);
    }
    __syncwarp();
    // Indices are loaded a batch of 32 slots at a time, one uint4 (four rows) per lane, one batch
    // ahead of use: ya holds batch q / 32, yb the next one.
    uint4 ya = lane < nq ? __ldg(idx4 + g0 + lane) : make_uint4(0, 0, 0, 0);
    uint4 yb = 32 + lane < nq ? __ldg(idx4 + g0 + 32 + lane) : make_uint4(0, 0, 0, 0);
    auto issue = [&](int j, uint4 y) {
        const int s = j % kDepth;
        fence_proxy_async_smem();
        mbar_arrive_expect_tx(&bars[s], 1024u);
        tma_gather4_2d(ring + s * 1024, &tmap, &bars[s], 0, int(y.x), int(y.y), int(y.z), int(y.w));
    };
    const int pre = nq < kDepth ? nq : kDepth;  // kDepth <= 32: the first slots are all in batch 0
    for (int j = 0; j < pre; ++j) {
        uint4 y;
        y.x = __shfl_sync(0xffffffffu, ya.x, j);
        y.y = __shfl_sync(0xffffffffu, ya.y, j);
        y.z = __shfl_sync(0xffffffffu, ya.z, j);
        y.w = __shfl_sync(0xffffffffu, ya.w, j);
        if (lane == 0) issue(j, y);
    }
    float acc = 0.f;
    int q = 0;
    for (; q < nq; ++q) {
        if (q > 0 && (q & 31) == 0) {  // entering batch q / 32: shift, and load the one after
            ya = yb;
            const int nxt = q + 32 + lane;
            yb = nxt < nq ? __ldg(idx4 + g0 + nxt) : make_uint4(0, 0, 0, 0);
        }
        const int s = q % kDepth;
        const bool ok = mbar_wait_bounded(&bars[s], uint32_t(q / kDepth) & 1u);
        if (!__all_sync(0xffffffffu, ok)) break;
        const uint4* src = reinterpret_cast<const uint4*>(ring + s * 1024) + lane * 2;
        const uint4 a = src[0], b = src[1];
        const __half2* h0 = reinterpret_cast<const __half2*>(&a);
        const __half2* h1 = reinterpret_cast<const __half2*>(&b);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 f0 = __half22float2(h0[i]), f1 = __half22float2(h1[i]);
            acc += (f0.x + f0.y) + (f1.x + f1.y);
        }
        __syncwarp();  // every lane has read slot s before it is refilled
        const int j = q + kDepth;
        if (j < nq) {
            const uint4 from = (j >> 5) == (q >> 5) ? ya : yb;
            uint4 y;
            y.x = __shfl_sync(0xffffffffu, from.x, j & 31);
            y.y = __shfl_sync(0xffffffffu, from.y, j & 31);
            y.z = __shfl_sync(0xffffffffu, from.z, j & 31);
            y.w = __shfl_sync(0xffffffffu, from.w, j & 31);
            if (lane == 0) issue(j, y);
        }
    }
    const int issued = q + kDepth < nq ? q + kDepth : nq;
    if (q < nq) {  // a wait expired: let the loads already issued land, then report
        if (lane == 0) {
            for (int r = q; r < issued; ++r) mbar_wait_bounded(&bars[r % kDepth], uint32_t(r / kDepth) & 1u);
            atomicOr(err, 1);
        }
        return;
    }
    double d = acc;
    for (int o = 16; o; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
    if (lane == 0) out[gw] = d;
}

// Register-gather warps and gather4 warps in one CTA, each warp taking chunks of `chunk` indices
// from a global counter until none are left. The gather4 warps keep their slot phases across
// chunks and drain their ring at the end of each chunk. Sums are exact in double.
template <int kLdgWarps, int kTmaWarps, int kDepth>
__global__ void __launch_bounds__((kLdgWarps + kTmaWarps) * 32) gather_hybrid(
    const __grid_constant__ CUtensorMap tmap, const uint4* __restrict__ B, const unsigned* __restrict__ idx, long long n,
    int chunk, unsigned long long* counter, double* out, int* err) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    uint8_t* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    double total = 0.0;
    if (warp < kLdgWarps) {
        const int sub = lane >> 4, sl = lane & 15;
        const unsigned gmask = 0xffffu << (16 * sub);
        for (;;) {
            unsigned long long start = 0;
            if (lane == 0) start = atomicAdd(counter, (unsigned long long)chunk);
            start = __shfl_sync(0xffffffffu, start, 0);
            if ((long long)start >= n) break;
            const long long c1 = (long long)start + chunk < n ? (long long)start + chunk : n;
            const long long half = (c1 - (long long)start + 1) / 2;
            const long long p0 = (long long)start + sub * half;
            const long long p1 = sub == 0 ? (long long)start + half : c1;
            float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
            unsigned nextrow = (p0 + sl < p1) ? __ldcs(idx + p0 + sl) : 0u;
            for (long long p = p0; p < p1; p += 16) {  // both halves take the same number of rounds
                const unsigned myrow = nextrow;
                nextrow = (p + 16 + sl < p1) ? __ldcs(idx + p + 16 + sl) : 0u;
                const uint4* a[16];
                bool v[16];
#pragma unroll
                for (int k = 0; k < 16; ++k) {
                    a[k] = B + (size_t)__shfl_sync(gmask, myrow, k, 16) * 16 + sl;
                    v[k] = p + k < p1;
                }
                uint4 r0[8], r1[8];
                ld8(a[0], a[1], a[2], a[3], a[4], a[5], a[6], a[7], r0);
                ld8(a[8], a[9], a[10], a[11], a[12], a[13], a[14], a[15], r1);
#pragma unroll
                for (int k = 0; k < 16; ++k) {
                    if (!v[k]) continue;
                    const __half2* h = reinterpret_cast<const __half2*>(k < 8 ? &r0[k] : &r1[k - 8]);
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const float2 f = __half22float2(h[i]);
                        acc[2 * i] += f.x;
                        acc[2 * i + 1] += f.y;
                    }
                }
            }
            for (int i = 0; i < 8; ++i) total += acc[i];
        }
    } else {
        const int tw = warp - kLdgWarps;
        uint8_t* ring = smem + tw * kDepth * 1024;
        uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kTmaWarps * kDepth * 1024) + tw * kDepth;
        if (lane == 0) {
            for (int s = 0; s < kDepth; ++s) mbar_init(&bars[s], 1);
            fence_mbar_init();
        }
        __syncwarp();
        const uint4* idx4 = reinterpret_cast<const uint4*>(idx);
        uint32_t u = 0;  // slots used so far (phase = (u / kDepth) & 1)
        float acc = 0.f;
        bool failed = false;
        for (; !failed;) {
            unsigned long long start = 0;
            if (lane == 0) start = atomicAdd(counter, (unsigned long long)chunk);
            start = __shfl_sync(0xffffffffu, start, 0);
            if ((long long)start >= n) break;
            const long long c1 = (long long)start + chunk < n ? (long long)start + chunk : n;
            const int nq = int((c1 - (long long)start) / 4);  // n and chunk are multiples of 4
            const long long g0 = (long long)start / 4;
            uint4 ya = lane < nq ? __ldg(idx4 + g0 + lane) : make_uint4(0, 0, 0, 0);
            uint4 yb = 32 + lane < nq ? __ldg(idx4 + g0 + 32 + lane) : make_uint4(0, 0, 0, 0);
            auto issue = [&](int j, const uint4& from) {
                uint4 y;
                y.x = __shfl_sync(0xffffffffu, from.x, j & 31);
                y.y = __shfl_sync(0xffffffffu, from.y, j & 31);
                y.z = __shfl_sync(0xffffffffu, from.z, j & 31);
                y.w = __shfl_sync(0xffffffffu, from.w, j & 31);
                if (lane == 0) {
                    const int s = int((u + uint32_t(j)) % kDepth);
                    fence_proxy_async_smem();
                    mbar_arrive_expect_tx(&bars[s], 1024u);
                    tma_gather4_2d(ring + s * 1024, &tmap, &bars[s], 0, int(y.x), int(y.y), int(y.z), int(y.w));
                }
            };
            const int pre = nq < kDepth ? nq : kDepth;
            for (int j = 0; j < pre; ++j) issue(j, ya);
            int q = 0;
            for (; q < nq; ++q) {
                if (q > 0 && (q & 31) == 0) {
                    ya = yb;
                    const int nxt = q + 32 + lane;
                    yb = nxt < nq ? __ldg(idx4 + g0 + nxt) : make_uint4(0, 0, 0, 0);
                }
                const uint32_t w = u + uint32_t(q);
                const int s = int(w % kDepth);
                const bool ok = mbar_wait_bounded(&bars[s], (w / kDepth) & 1u);
                if (!__all_sync(0xffffffffu, ok)) break;
                const uint4* src = reinterpret_cast<const uint4*>(ring + s * 1024) + lane * 2;
                const uint4 a = src[0], b = src[1];
                const __half2* h0 = reinterpret_cast<const __half2*>(&a);
                const __half2* h1 = reinterpret_cast<const __half2*>(&b);
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const float2 f0 = __half22float2(h0[i]), f1 = __half22float2(h1[i]);
                    acc += (f0.x + f0.y) + (f1.x + f1.y);
                }
                __syncwarp();
                const int j = q + kDepth;
                if (j < nq) issue(j, (j >> 5) == (q >> 5) ? ya : yb);
            }
            if (q < nq) {  // a wait expired: drain what was issued, report, stop
                const int issued = q + kDepth < nq ? q + kDepth : nq;
                if (lane == 0) {
                    for (int r = q; r < issued; ++r) {
                        const uint32_t w = u + uint32_t(r);
                        mbar_wait_bounded(&bars[w % kDepth], (w / kDepth) & 1u);
                    }
                    atomicOr(err, 1);
                }
                failed = true;
            }
            u += uint32_t(nq);
            total += acc;  // acc < 2^18 per chunk: exact in fp32
            acc = 0.f;
        }
    }
    for (int o = 16; o; o >>= 1) total += __shfl_xor_sync(0xffffffffu, total, o);
    if (lane == 0) atomicAdd(out, total);
}

template <int kLdgWarps, int kTmaWarps, int kDepth>
void run_hybrid(const CUtensorMap& tmap, const uint4* B, const unsigned* idx, long long n, double* out,
                unsigned long long* counter, int* err, double expect, int sms) {
    const int threads = (kLdgWarps + kTmaWarps) * 32;
    const int smem = kTmaWarps * kDepth * 1024 + kTmaWarps * kDepth * 8 + 1024;
    auto k = gather_hybrid<kLdgWarps, kTmaWarps, kDepth>;
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) return;
    int nb = 0;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, k, threads, smem);
    if (nb == 0) {
        printf("hybrid   L=%2d T=%2d D=%2d: does not fit\n", kLdgWarps, kTmaWarps, kDepth);
        return;
    }
    cudaFuncAttributes fa; cudaFuncGetAttributes(&fa, k);
    const int chunk = 4096;
    cudaEvent_t a, b; cudaEventCreate(&a); cudaEventCreate(&b);
    float total_ms = 0.f;
    double sum = 0.0;
    const int reps = 6;
    for (int w = 0; w < reps; ++w) {  // first launch is warm-up
        cudaMemset(counter, 0, sizeof(unsigned long long));
        cudaMemset(out, 0, sizeof(double));
        cudaEventRecord(a);
        k<<<sms * nb, threads, smem>>>(tmap, B, idx, n, chunk, counter, out, err);
        cudaEventRecord(b);
        cudaEventSynchronize(b);
        float ms; cudaEventElapsedTime(&ms, a, b);
        if (w > 0) total_ms += ms;
        cudaMemcpy(&sum, out, sizeof(double), cudaMemcpyDeviceToHost);
    }
    int herr = 0;
    cudaMemcpy(&herr, err, sizeof(int), cudaMemcpyDeviceToHost);
    const float ms = total_ms / (reps - 1);
    printf("hybrid   L=%2d T=%2d D=%2d regs=%3d CTAs/SM=%d : %.3f ms  %6.2f G rows/s  %.2f TB/s  sum %s%s\n", kLdgWarps,
           kTmaWarps, kDepth, fa.numRegs, nb, ms, n / (ms * 1e6), n * 256.0 / (ms * 1e9),
           sum == expect ? "exact" : "WRONG", herr ? " (a wait expired)" : "");
}

template <int kWarps, int kDepth>
void run_tma(const CUtensorMap& tmap, const unsigned* idx, long long n, double* out, int* err, double expect) {
    const int per_warp = 4096;
    const long long warps = (n + per_warp - 1) / per_warp;
    const long long blocks = (warps + kWarps - 1) / kWarps;
    const int smem = kWarps * kDepth * 1024 + kWarps * kDepth * 8 + 1024;
    auto k = gather4_tma<kWarps, kDepth>;
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) {
        printf("tma      W=%2d D=%2d: shared memory %d B not available\n", kWarps, kDepth, smem);
        return;
    }
    cudaMemset(out, 0, warps * sizeof(double));
    cudaEvent_t a, b; cudaEventCreate(&a); cudaEventCreate(&b);
    for (int w = 0; w < 2; ++w) k<<<blocks, kWarps * 32, smem>>>(tmap, reinterpret_cast<const uint4*>(idx), n, per_warp, out, err);
    cudaEventRecord(a);
    const int reps = 5;
    for (int w = 0; w < reps; ++w) k<<<blocks, kWarps * 32, smem>>>(tmap, reinterpret_cast<const uint4*>(idx), n, per_warp, out, err);
    cudaEventRecord(b); cudaEventSynchronize(b);
    float ms; cudaEventElapsedTime(&ms, a, b);
    ms /= reps;
    std::vector<double> h(warps);
    cudaMemcpy(h.data(), out, warps * sizeof(double), cudaMemcpyDeviceToHost);
    int herr = 0;
    cudaMemcpy(&herr, err, sizeof(int), cudaMemcpyDeviceToHost);
    double sum = 0;
    for (double x : h) sum += x;
    int nb = 0; cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, k, kWarps * 32, smem);
    printf("tma      W=%2d D=%2d warps/SM=%2d rows in flight/SM=%4d : %.3f ms  %6.2f G rows/s  %.2f TB/s  sum %s%s\n",
           kWarps, kDepth, nb * kWarps, nb * kWarps * kDepth * 4, ms, n / (ms * 1e6), n * 256.0 / (ms * 1e9),
           sum == expect ? "exact" : "WRONG", herr ? " (a wait expired)" : "");
}

// An int32 (little-endian '<i4') one-dimensional .npy file; false unless every value is in [0, limit).
bool read_npy_indices(const char* path, long long limit, std::vector<unsigned>& out) {
    FILE* f = std::fopen(path, "rb");
    if (!f) return false;
    unsigned char pre[10];
    bool ok = std::fread(pre, 1, 10, f) == 10 && std::memcmp(pre, "\x93NUMPY", 6) == 0;
    long long hlen = 0, hstart = 10;
    if (ok && pre[6] == 1) {
        hlen = pre[8] | (pre[9] << 8);
    } else if (ok && (pre[6] == 2 || pre[6] == 3)) {
        unsigned char b[2];
        ok = std::fread(b, 1, 2, f) == 2;
        hlen = pre[8] | (pre[9] << 8) | ((long long)b[0] << 16) | ((long long)b[1] << 24);
        hstart = 12;
    } else {
        ok = false;
    }
    std::string hdr(size_t(ok ? hlen : 0), ' ');
    ok = ok && std::fread(&hdr[0], 1, size_t(hlen), f) == size_t(hlen) && hdr.find("'<i4'") != std::string::npos &&
         hdr.find("'fortran_order': False") != std::string::npos;
    if (ok) {
        std::fseek(f, 0, SEEK_END);
        const long long bytes = std::ftell(f) - hstart - hlen;
        ok = bytes >= 0 && bytes % 4 == 0;
        if (ok) {
            out.resize(size_t(bytes / 4));
            std::fseek(f, long(hstart + hlen), SEEK_SET);
            ok = std::fread(out.data(), 4, out.size(), f) == out.size();
        }
    }
    std::fclose(f);
    if (!ok) return false;
    for (const unsigned x : out)
        if ((long long)x >= limit) return false;
    return !out.empty();
}

int main(int argc, char** argv) {
    const long long nrows = 1LL << 24;  // 16.8M rows x 256 B = 4.3 GB
    long long n = 1LL << 26;            // gathers
    const int mode = argc > 1 ? atoi(argv[1]) : 0;
    std::vector<unsigned> given;
    if (mode == 3) {
        if (argc < 3 || !read_npy_indices(argv[2], nrows, given)) {
            printf("mode 3 needs an int32 .npy of indices below %lld\n", nrows);
            return 1;
        }
        n = (long long)given.size();
    }
    uint4* B; unsigned* idx; float* out; double* dout; int* err;
    if (cudaMalloc(&B, nrows * 256) != cudaSuccess) { printf("oom\n"); return 1; }
    fill_b<<<148 * 16, 256>>>(reinterpret_cast<__half*>(B), nrows);
    cudaMalloc(&idx, n * 4); cudaMalloc(&out, 1 << 24); cudaMalloc(&dout, (n / 4096 + 1) * sizeof(double));
    cudaMalloc(&err, sizeof(int)); cudaMemset(err, 0, sizeof(int));
    std::vector<unsigned> h;
    if (mode == 3) {
        h.swap(given);
        printf("mode 3: %lld given indices from %s\n", n, argv[2]);
    } else {
        h.resize(n);
        std::mt19937_64 rng(1);
        const long long span = mode == 0 ? nrows : (mode == 1 ? (1LL << 20) : (1LL << 17));
        for (auto& x : h) x = unsigned(rng() % span);
        printf("mode %d: rows uniform over %lld (%.0f MB)\n", mode, span, span * 256.0 / 1e6);
    }
    double expect = 0;
    for (const unsigned x : h) expect += 2.0 * (x % 61) + 127.0 / 64.0;  // sum of row x of B
    cudaMemcpy(idx, h.data(), n * 4, cudaMemcpyHostToDevice);
    if (mode == 3) {
        run<8, true>(B, idx, n, out, "double");
        run<4, true>(B, idx, n, out, "double");
        run<8, false>(B, idx, n, out, "single");
        // the same gathers plus one 512-byte fp32 row stored per 16 entries (a C stream)
        float* rows_out = nullptr;
        const long long nrows_out = (n + 15) / 16;
        if (cudaMalloc(&rows_out, nrows_out * 512) == cudaSuccess) {
            printf("with a 512-byte row stored per 16 gathers (%.2f GB written):\n", nrows_out * 512.0 / 1e9);
            run<4, true, true>(B, idx, n, out, "double+C", rows_out);
            run<8, false, true>(B, idx, n, out, "single+C", rows_out);
            cudaFree(rows_out);
        } else {
            cudaGetLastError();
            printf("no room for the row stream\n");
        }
        cudaError_t e = cudaDeviceSynchronize();
        printf("status %s\n", cudaGetErrorString(e));
        return e == cudaSuccess ? 0 : 1;
    }
    run<8, false>(B, idx, n, out, "single");
    run<8, true>(B, idx, n, out, "double");
    run<4, true>(B, idx, n, out, "double");
    run<16, true>(B, idx, n, out, "double");
    run<16, false>(B, idx, n, out, "single");
    CUtensorMap tmap;
    std::memset(&tmap, 0, sizeof tmap);
    PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
    const cuuint64_t dims[2] = {128u, cuuint64_t(nrows)};
    const cuuint64_t strides[1] = {256u};
    const cuuint32_t box[2] = {128u, 1u};  // gather4: one row high
    const cuuint32_t estr[2] = {1u, 1u};
    if (!enc || enc(&tmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, B, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS) {
        printf("tensor map for gather4 not available\n");
    } else {
        run_tma<8, 12>(tmap, idx, n, dout, err, expect);
        run_tma<16, 12>(tmap, idx, n, dout, err, expect);
        run_tma<8, 24>(tmap, idx, n, dout, err, expect);
        run_tma<16, 6>(tmap, idx, n, dout, err, expect);
        int sms = 0;
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, 0);
        unsigned long long* counter;
        cudaMalloc(&counter, sizeof(unsigned long long));
        run_hybrid<8, 4, 12>(tmap, B, idx, n, dout, counter, err, expect, sms);
        run_hybrid<8, 2, 16>(tmap, B, idx, n, dout, counter, err, expect, sms);
        run_hybrid<16, 8, 12>(tmap, B, idx, n, dout, counter, err, expect, sms);
        run_hybrid<8, 0, 1>(tmap, B, idx, n, dout, counter, err, expect, sms);
        run_hybrid<0, 8, 12>(tmap, B, idx, n, dout, counter, err, expect, sms);
    }
    cudaError_t e = cudaDeviceSynchronize();
    printf("status %s\n", cudaGetErrorString(e));
    return e == cudaSuccess ? 0 : 1;
}
