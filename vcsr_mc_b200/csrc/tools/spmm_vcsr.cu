// spmm_vcsr: the benchmark driver, with the reference's command-line surface (src/main.cpp:33-372):
//   --mtx FILE | --gen c1|c2|c3|rmat[:scale]  --O 128 --segw 16 --tileK 64 --repeat 10 --warmup 3
//   --stat mean|median --reorder none|rcm --algo vcsr_mc,vcsr_mc_fp32,cusparse,cusparse_fp16|all
//   --check cpu|none --csv --bdist pattern|normal|uniform|wide --lenient
// plus: --gen (seeded synthetic configurations, no download needed), --seed, --plan auto|rows|segment|band,
// --b16 (the FP16 path reads fp16 B instead of converting fp32 B).
// Same B fill (fixed seed 20260923), same fp64 CPU check and acceptance bounds, same CSV schema.
// Host work uses the library's C++ surface (vcsrmc/*.hpp); every GPU call goes through the C ABI
// (vcsrmc.h). "vcsr_mc"/"vcsr_mc_fp32" with --plan auto and fp32 B run exactly like the reference
// through upload_vcsr_mc_device / run_vcsr_mc_spmm_gpu / destroy_vcsr_mc_device.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <getopt.h>

#include <algorithm>
#include <chrono>
#include <climits>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <functional>
#include <numeric>
#include <random>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

#include "vcsrmc.h"
#include "vcsrmc/csr.hpp"
#include "vcsrmc/gen.hpp"
#include "vcsrmc/reorder.hpp"
#include "vcsrmc/vcsr_formats.hpp"
#include "vcsrmc/vcsr_mc_device.hpp"

extern "C" int vcsrmc_cusparse_spmm(int32_t M, int32_t N, int64_t nnz, const int32_t* d_rowptr, const int32_t* d_col,
                                    const void* d_val, int val_f16, const void* d_B, int b_f16, int32_t O, float* d_C,
                                    float alpha, int warmup, int reps, void* stream, float* ms_median);
extern "C" const char* vcsrmc_cusparse_last_error(void);

using namespace vcsrmc;

namespace {

void cuda_ok(cudaError_t e, const char* what) {
    if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}
void abi_ok(int st) {
    if (st != VCSRMC_OK) {
        char msg[512];
        vcsrmc_last_error(msg, sizeof msg);
        throw std::runtime_error(std::string("vcsrmc: ") + msg);
    }
}

void usage() {
    std::printf(
        "Usage: spmm_vcsr (--mtx file.mtx | --gen c1|c2|c3|rmat[:scale]) --O 128 [options]\n"
        "Algorithms: vcsr_mc (FP16 A/B, FP32 accumulate), vcsr_mc_fp32, cusparse (FP32),\n"
        "            cusparse_fp16 (FP16 A and B, FP32 compute and C), all\n"
        "Options: --segw 16 --tileK 64 --repeat 10 --warmup 3 --stat mean|median\n"
        "         --reorder none|rcm --check cpu|none --csv --bdist pattern|normal|uniform|wide\n"
        "         --lenient --seed 0 --plan auto|rows|segment|band --b16\n"
        "tileK must be one of 16, 32, 64, 128, 256; segw one of 16, 32, 48, 64.\n");
}

int int_at_least(const char* text, long minimum) {
    char* end = nullptr;
    const long v = std::strtol(text, &end, 10);
    if (end == text || *end || v < minimum || v > INT_MAX)
        throw std::runtime_error(std::string("Expected integer >= ") + std::to_string(minimum) + ", got: " + text);
    return int(v);
}

std::string csv_quote(const std::string& value) {
    std::string out = "\"";
    for (char c : value) {
        if (c == '"') out += '"';
        out += c;
    }
    return out + '"';
}

CSR generate(const std::string& spec, uint64_t seed) {
    if (spec == "c1") return gen_uniform_poisson(4096, 4096, 16.0, seed);
    if (spec == "c2") return gen_zipf_rows(262144, 262144, 1.8, 8192, 10.0, seed);
    if (spec == "c3") return gen_stencil27(100, 100, 100, seed);
    if (spec.rfind("rmat", 0) == 0) {
        const int scale = spec.size() > 5 ? int_at_least(spec.c_str() + 5, 1) : 24;
        return gen_rmat(scale, int64_t(1) << (scale + 4), 0.57, 0.19, 0.19, seed);
    }
    throw std::runtime_error("Unknown --gen: " + spec + " (c1|c2|c3|rmat[:scale])");
}

// fp64 CSR SpMM, row blocks on all host threads; per-row accumulation order of the reference.
std::vector<double> cpu_reference(const CSR& csr, const std::vector<float>& hB, int O) {
    std::vector<double> ref(size_t(csr.M) * O, 0.0);
    const int T = std::max(1u, std::thread::hardware_concurrency());
    std::vector<std::thread> th;
    for (int t = 0; t < T; ++t)
        th.emplace_back([&, t] {
            for (int r = int(int64_t(csr.M) * t / T); r < int(int64_t(csr.M) * (t + 1) / T); ++r)
                for (int p = csr.row_ptr[r]; p < csr.row_ptr[r + 1]; ++p)
                    for (int k = 0; k < O; ++k)
                        ref[size_t(r) * O + k] += double(csr.val[p]) * hB[size_t(csr.col[p]) * O + k];
        });
    for (auto& x : th) x.join();
    return ref;
}

}  // namespace

static int benchmark_main(int argc, char** argv) {
    std::string mtx, gen, algo = "all", check = "cpu", reorder = "none", bdist = "pattern", stat = "mean",
                         plan = "auto";
    int O = 128, segw = 16, tileK = 64, repeat = 10, warmup = 3;
    uint64_t seed = 0;
    bool csv = false, lenient = false, b16 = false;
    constexpr int bundle = 16;
    static option opts[] = {
        {"mtx", required_argument, nullptr, 'm'},    {"gen", required_argument, nullptr, 'g'},
        {"O", required_argument, nullptr, 'o'},      {"segw", required_argument, nullptr, 's'},
        {"tileK", required_argument, nullptr, 't'},  {"repeat", required_argument, nullptr, 'r'},
        {"warmup", required_argument, nullptr, 'w'}, {"reorder", required_argument, nullptr, 'R'},
        {"algo", required_argument, nullptr, 'a'},   {"check", required_argument, nullptr, 'c'},
        {"csv", no_argument, nullptr, 'j'},          {"help", no_argument, nullptr, 'h'},
        {"bdist", required_argument, nullptr, 'D'},  {"lenient", no_argument, nullptr, 'L'},
        {"stat", required_argument, nullptr, 'S'},   {"seed", required_argument, nullptr, 'e'},
        {"plan", required_argument, nullptr, 'p'},   {"b16", no_argument, nullptr, 'b'},
        {nullptr, 0, nullptr, 0}};
    int opt;
    while ((opt = getopt_long(argc, argv, "", opts, nullptr)) != -1) {
        switch (opt) {
            case 'm': mtx = optarg; break;
            case 'g': gen = optarg; break;
            case 'o': O = int_at_least(optarg, 1); break;
            case 's': segw = int_at_least(optarg, 1); break;
            case 't': tileK = int_at_least(optarg, 1); break;
            case 'r': repeat = int_at_least(optarg, 1); break;
            case 'w': warmup = int_at_least(optarg, 0); break;
            case 'R': reorder = optarg; break;
            case 'a': algo = optarg; break;
            case 'c': check = optarg; break;
            case 'D': bdist = optarg; break;
            case 'L': lenient = true; break;
            case 'S': stat = optarg; break;
            case 'e': seed = std::strtoull(optarg, nullptr, 10); break;
            case 'p': plan = optarg; break;
            case 'b': b16 = true; break;
            case 'j': csv = true; break;
            case 'h': usage(); return 0;
            default: usage(); return 2;
        }
    }
    const std::vector<std::string> algorithms = {"all", "vcsr_mc", "vcsr_mc_fp32", "cusparse", "cusparse_fp16"};
    std::vector<std::string> requested;
    for (size_t pos = 0;;) {
        const size_t comma = algo.find(',', pos);
        const std::string one = algo.substr(pos, comma == std::string::npos ? std::string::npos : comma - pos);
        if (one.empty() || std::find(algorithms.begin(), algorithms.end(), one) == algorithms.end())
            throw std::runtime_error("Unknown algorithm: " + one);
        requested.push_back(one);
        if (comma == std::string::npos) break;
        pos = comma + 1;
    }
    auto selected = [&](const char* name) {
        return std::find(requested.begin(), requested.end(), "all") != requested.end() ||
               std::find(requested.begin(), requested.end(), name) != requested.end();
    };
    if (check != "cpu" && check != "none") throw std::runtime_error("Unknown reference: " + check);
    if ((mtx.empty() == gen.empty()) || optind != argc) { usage(); return 2; }
    if (reorder != "none" && reorder != "rcm") throw std::runtime_error("Unknown reordering: " + reorder);
    if (stat != "mean" && stat != "median") throw std::runtime_error("Unknown --stat: " + stat + " (mean|median)");
    if (plan != "auto" && plan != "rows" && plan != "segment" && plan != "band")
        throw std::runtime_error("Unknown --plan: " + plan);
    const int plan_id = plan == "rows"      ? VCSRMC_PLAN_ROWS
                        : plan == "segment" ? VCSRMC_PLAN_SEGMENT
                        : plan == "band"    ? VCSRMC_PLAN_BAND
                                            : VCSRMC_PLAN_AUTO;

    CSR csr = mtx.empty() ? generate(gen, seed) : coo_to_csr(read_matrix_market_coo(mtx));
    const std::string source = mtx.empty() ? "gen:" + gen : mtx;
    const size_t elementsB = size_t(csr.N) * O, elementsC = size_t(csr.M) * O;
    std::vector<float> hB(elementsB);
    if (bdist == "pattern") {
        for (size_t i = 0; i < hB.size(); ++i) hB[i] = float(int(i % 13) - 6) / 7.f;
    } else {
        std::mt19937_64 rng(20260923);
        if (bdist == "normal") {
            std::normal_distribution<float> d(0.f, 1.f);
            for (float& x : hB) x = d(rng);
        } else if (bdist == "uniform") {
            std::uniform_real_distribution<float> d(-1.f, 1.f);
            for (float& x : hB) x = d(rng);
        } else if (bdist == "wide") {
            std::uniform_real_distribution<float> e(-3.f, 3.f);
            std::bernoulli_distribution sign(0.5);
            for (float& x : hB) x = (sign(rng) ? -1.f : 1.f) * std::pow(10.f, e(rng));
        } else {
            throw std::runtime_error("Unknown --bdist: " + bdist + " (pattern|normal|uniform|wide)");
        }
    }
    if (reorder == "rcm" && csr.nnz) apply_column_permutation(csr, hB, O, rcm_column_order(csr));

    cudaDeviceProp device{};
    int device_id = 0;
    cuda_ok(cudaGetDevice(&device_id), "cudaGetDevice");
    cuda_ok(cudaGetDeviceProperties(&device, device_id), "cudaGetDeviceProperties");
    float *dB = nullptr, *dC = nullptr, *d_val = nullptr;
    __half *dB16 = nullptr, *d_val16 = nullptr;
    int *d_rowptr = nullptr, *d_col = nullptr;
    cuda_ok(cudaMalloc(&dB, elementsB * sizeof(float)), "cudaMalloc");
    cuda_ok(cudaMalloc(&dC, std::max<size_t>(elementsC, 1) * sizeof(float)), "cudaMalloc");
    cuda_ok(cudaMemcpy(dB, hB.data(), elementsB * sizeof(float), cudaMemcpyHostToDevice), "cudaMemcpy");
    cudaStream_t st;
    cuda_ok(cudaStreamCreate(&st), "cudaStreamCreate");

    std::vector<double> reference;
    if (check == "cpu") reference = cpu_reference(csr, hB, O);
    if (csv)
        std::printf("gpu,sm,mtx,O,segw,bundle,tileK,repeat,algo,ms,gflops,validation,rel_l2,setup_ms,ms_mean,ms_median,"
                    "convert_ms,upload_ms,plan\n");
    else
        std::printf("Matrix: %d x %d, nnz=%d; O=%d segw=%d bundle=%d tileK=%d repeat=%d warmup=%d reorder=%s; "
                    "reference=%s\nKernel                Time (ms)      GFLOP/s   Validation\n",
                    csr.M, csr.N, csr.nnz, O, segw, bundle, tileK, repeat, warmup, reorder.c_str(), check.c_str());
    auto wall_ms = [](auto&& f) {
        const auto t0 = std::chrono::steady_clock::now();
        f();
        return std::chrono::duration<float, std::milli>(std::chrono::steady_clock::now() - t0).count();
    };
    auto measure = [&](const char* name, const std::function<float()>& run, float setup_ms, float convert_ms,
                       float upload_ms, const char* plan_used) {
        auto iterate = [&]() {
            cuda_ok(cudaMemsetAsync(dC, 0, elementsC * sizeof(float), st), "cudaMemsetAsync");
            cuda_ok(cudaStreamSynchronize(st), "cudaStreamSynchronize");
            const float ms = csr.nnz ? run() : 0.f;
            cuda_ok(cudaStreamSynchronize(st), "cudaStreamSynchronize");
            if (!std::isfinite(ms) || ms < 0) throw std::runtime_error("Invalid kernel timing");
            return double(ms);
        };
        for (int it = 0; it < warmup; ++it) iterate();
        std::vector<double> times(repeat);
        for (double& t : times) t = iterate();
        double rel_l2 = 0;
        bool failed = false;
        if (check != "none") {
            std::vector<float> result(elementsC);
            cuda_ok(cudaMemcpy(result.data(), dC, elementsC * sizeof(float), cudaMemcpyDeviceToHost), "cudaMemcpy");
            double e2 = 0, r2 = 0;
            bool nonfinite = false;
            for (size_t i = 0; i < result.size(); ++i) {
                if (!std::isfinite(result[i])) {
                    if (!lenient) throw std::runtime_error(std::string(name) + ": non-finite output");
                    nonfinite = true;
                    break;
                }
                const double e = double(result[i]) - reference[i];
                e2 += e * e;
                r2 += reference[i] * reference[i];
            }
            const double err = std::sqrt(e2), norm = std::sqrt(r2);
            rel_l2 = norm > 0 ? err / norm : err;
            if (nonfinite) { rel_l2 = INFINITY; failed = true; }
            const std::string kname(name);
            const bool half = kname == "vcsr_mc" || kname == "cusparse_fp16";
            const double tolerance = (half ? 3e-3 : 1e-4) * norm + 1e-5 * std::sqrt(double(elementsC));
            if (!nonfinite && (err > tolerance || rel_l2 > (half ? 1e-1 : 1e-2))) {
                if (!lenient)
                    throw std::runtime_error(std::string(name) + ": correctness check failed, rel_l2=" +
                                             std::to_string(rel_l2));
                failed = true;
            }
        }
        const double ms_mean = std::accumulate(times.begin(), times.end(), 0.0) / repeat;
        std::sort(times.begin(), times.end());
        const double ms_median =
            repeat % 2 ? times[repeat / 2] : 0.5 * (times[repeat / 2 - 1] + times[repeat / 2]);
        const double ms = stat == "median" ? ms_median : ms_mean;
        const double gflops = ms > 0 ? (2.0 * csr.nnz * O) / (ms * 1e6) : 0;
        const char* validation = check == "none" ? "unchecked" : failed ? "FAIL" : "pass";
        if (csv)
            std::printf("%s,%d,%s,%d,%d,%d,%d,%d,%s,%.9g,%.9g,%s,%.9g,%.6g,%.9g,%.9g,%.6g,%.6g,%s\n",
                        csv_quote(device.name).c_str(), device.major * 10 + device.minor, csv_quote(source).c_str(), O,
                        segw, bundle, tileK, repeat, name, ms, gflops, validation, rel_l2, setup_ms, ms_mean, ms_median,
                        convert_ms, upload_ms, plan_used);
        else
            std::printf("%-20s %10.6f %12.2f   %s (rel_l2=%.3g, setup %.3f ms, plan %s)\n", name, ms, gflops, validation,
                        rel_l2, setup_ms, plan_used);
        std::fflush(stdout);
    };

    for (const bool fp32 : {false, true}) {
        const char* name = fp32 ? "vcsr_mc_fp32" : "vcsr_mc";
        if (!selected(name)) continue;
        VCSRMC V;
        const float convert = wall_ms([&] { V = csr_to_vcsr_mc(csr, fp32, segw); });
        const bool use_b16 = b16 && !fp32;
        if (use_b16 && !dB16) {
            std::vector<__half> h(elementsB);
            for (size_t i = 0; i < elementsB; ++i) h[i] = __float2half_rn(hB[i]);
            cuda_ok(cudaMalloc(&dB16, elementsB * sizeof(__half)), "cudaMalloc");
            cuda_ok(cudaMemcpy(dB16, h.data(), elementsB * sizeof(__half), cudaMemcpyHostToDevice), "cudaMemcpy");
        }
        if (plan_id == VCSRMC_PLAN_AUTO && !use_b16) {
            // the reference's own call sequence (src/main.cpp:356-361)
            const float upload = wall_ms([&] { upload_vcsr_mc_device(V); });
            measure(name, [&] { float ms = 0; run_vcsr_mc_spmm_gpu(V, dB, O, tileK, dC, st, ms); return ms; },
                    convert + upload, convert, upload, "auto");
            destroy_vcsr_mc_device(st);
        } else {
            vcsrmc_csr* hc = nullptr;
            vcsrmc_format* hf = nullptr;
            vcsrmc_device_format* hd = nullptr;
            abi_ok(vcsrmc_csr_from_arrays(csr.M, csr.N, csr.nnz, csr.row_ptr.data(), csr.col.data(), csr.val.data(), &hc));
            abi_ok(vcsrmc_build_host(hc, fp32 ? 1 : 0, segw, 0, &hf));
            // the BAND plan runs on the tensor cores (FP16 format); the FP32 format takes ROWS
            const int my_plan = (plan_id == VCSRMC_PLAN_BAND && fp32) ? VCSRMC_PLAN_ROWS : plan_id;
            const int mask = my_plan == VCSRMC_PLAN_BAND ? (1 << VCSRMC_PLAN_BAND) : 0;
            const char* my_plan_name = my_plan == plan_id ? plan.c_str() : "rows";
            const float upload = wall_ms([&] { abi_ok(vcsrmc_upload_ex(hf, device_id, mask, st, &hd)); });
            measure(name,
                    [&] {
                        cudaEvent_t a, b;
                        cudaEventCreate(&a);
                        cudaEventCreate(&b);
                        cudaEventRecord(a, st);
                        abi_ok(vcsrmc_spmm_ex(hd, use_b16 ? static_cast<const void*>(dB16) : dB,
                                              use_b16 ? VCSRMC_F16 : VCSRMC_F32, O, O, tileK, dC, O, 1, my_plan, st));
                        cudaEventRecord(b, st);
                        cudaEventSynchronize(b);
                        float ms = 0;
                        cudaEventElapsedTime(&ms, a, b);
                        cudaEventDestroy(a);
                        cudaEventDestroy(b);
                        return ms;
                    },
                    convert + upload, convert, upload, my_plan_name);
            vcsrmc_device_free(hd);
            vcsrmc_format_free(hf);
            vcsrmc_csr_free(hc);
        }
    }
    if (selected("cusparse") || selected("cusparse_fp16")) {
        cuda_ok(cudaMalloc(&d_rowptr, sizeof(int) * (size_t(csr.M) + 1)), "cudaMalloc");
        cuda_ok(cudaMalloc(&d_col, sizeof(int) * std::max(csr.nnz, 1)), "cudaMalloc");
        cuda_ok(cudaMalloc(&d_val, sizeof(float) * std::max(csr.nnz, 1)), "cudaMalloc");
        cuda_ok(cudaMemcpy(d_rowptr, csr.row_ptr.data(), sizeof(int) * (size_t(csr.M) + 1), cudaMemcpyHostToDevice), "h2d");
        if (csr.nnz) {
            cuda_ok(cudaMemcpy(d_col, csr.col.data(), sizeof(int) * csr.nnz, cudaMemcpyHostToDevice), "h2d");
            cuda_ok(cudaMemcpy(d_val, csr.val.data(), sizeof(float) * csr.nnz, cudaMemcpyHostToDevice), "h2d");
        }
    }
    if (selected("cusparse")) {
        measure("cusparse", [&] {
            float ms = 0;
            if (vcsrmc_cusparse_spmm(csr.M, csr.N, csr.nnz, d_rowptr, d_col, d_val, 0, dB, 0, O, dC, 1.f, 0, 1, st, &ms))
                throw std::runtime_error(std::string("cuSPARSE: ") + vcsrmc_cusparse_last_error());
            return ms;
        }, 0.f, 0.f, 0.f, "-");
    }
    if (selected("cusparse_fp16")) {
        const float scale = half_scale(csr), inv = 1.f / scale;
        std::vector<__half> v16(std::max(csr.nnz, 1)), b16h(elementsB);
        for (int i = 0; i < csr.nnz; ++i) v16[i] = __float2half_rn(csr.val[i] * inv);
        for (size_t i = 0; i < elementsB; ++i) b16h[i] = __float2half_rn(hB[i]);
        cuda_ok(cudaMalloc(&d_val16, sizeof(__half) * v16.size()), "cudaMalloc");
        if (!dB16) cuda_ok(cudaMalloc(&dB16, sizeof(__half) * elementsB), "cudaMalloc");
        cuda_ok(cudaMemcpy(d_val16, v16.data(), sizeof(__half) * v16.size(), cudaMemcpyHostToDevice), "h2d");
        cuda_ok(cudaMemcpy(dB16, b16h.data(), sizeof(__half) * elementsB, cudaMemcpyHostToDevice), "h2d");
        measure("cusparse_fp16", [&] {
            float ms = 0;
            if (vcsrmc_cusparse_spmm(csr.M, csr.N, csr.nnz, d_rowptr, d_col, d_val16, 1, dB16, 1, O, dC, scale, 0, 1, st,
                                     &ms))
                throw std::runtime_error(std::string("cuSPARSE: ") + vcsrmc_cusparse_last_error());
            return ms;
        }, 0.f, 0.f, 0.f, "-");
    }
    cudaStreamDestroy(st);
    cudaFree(dB); cudaFree(dC); cudaFree(dB16); cudaFree(d_val16);
    cudaFree(d_rowptr); cudaFree(d_col); cudaFree(d_val);
    return 0;
}

int main(int argc, char** argv) {
    try {
        return benchmark_main(argc, argv);
    } catch (const std::exception& e) {
        std::fprintf(stderr, "Error: %s\n", e.what());
        return 2;
    }
}
