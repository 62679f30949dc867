// spmm_vcsr: the benchmark driver, with the reference's command-line surface (src/main.cpp:33-372):
//   --mtx FILE | --gen c1|c2|c3|rmat[:scale]  --O 128 --segw 16 --tileK 64 --repeat 10 --warmup 3
//   --stat mean|median --reorder none|rcm --algo vcsr_mc,vcsr_mc_fp32,cusparse,cusparse_fp16|all
//   --check cpu|none --csv --bdist pattern|normal|uniform|wide --lenient
// plus: --gen (seeded synthetic configurations, no download needed), --seed, --plan auto|rows|segment|band|hybrid,
// --b16 (the FP16 path reads fp16 B instead of converting fp32 B), --flush-l2 (write a buffer twice
// the L2 size before every launch, outside the timed events), --peak-gbs G (the HBM peak that
// roofline_frac is taken against). Two columns follow the reference's CSV columns and `plan`:
// gbps_alg (algorithmic bytes per second: A's column index and value, row_ptr, the B rows A
// touches, C written once) and roofline_frac (gbps_alg / peak, empty without --peak-gbs).
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
        "Usage: spmm_vcsr (--mtx file.mtx | --gen c1|c2|c3|c3links|rmat[:scale]) --O 128 [options]\n"
        "Algorithms: vcsr_mc (FP16 A/B, FP32 accumulate), vcsr_mc_fp32, cusparse (FP32),\n"
        "            cusparse_fp16 (FP16 A and B, FP32 compute and C), all\n"
        "Options: --segw 16 --tileK 64 --repeat 10 --warmup 3 --stat mean|median\n"
        "         --reorder none|rcm --check cpu|none --csv --bdist pattern|normal|uniform|wide\n"
        "         --lenient --seed 0 --plan auto|rows|segment|band|hybrid --b16 --flush-l2 --peak-gbs G\n"
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
    if (spec == "c3links") return gen_stencil27_links(100, 3, seed);
    if (spec.rfind("rmat", 0) == 0) {
        const int scale = spec.size() > 5 ? int_at_least(spec.c_str() + 5, 1) : 24;
        return gen_rmat(scale, int64_t(1) << (scale + 4), 0.57, 0.19, 0.19, seed);
    }
    throw std::runtime_error("Unknown --gen: " + spec + " (c1|c2|c3|c3links|rmat[:scale])");
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

// ---- checking, statistics and output --------------------------------------------------------
// The interface kept from the reference's driver (src/main.cpp:257-304): the CSV columns and their
// order, the acceptance bounds and the error messages. The code below is this driver's own.

// Norms of a kernel's C against the fp64 CPU result, summed per thread block of rows.
struct Fp64Comparison {
    bool finite = true;  // every element of C is finite
    double err_norm = 0, ref_norm = 0;
    double rel_l2() const {
        if (!finite) return INFINITY;
        return ref_norm > 0 ? err_norm / ref_norm : err_norm;
    }
};

Fp64Comparison compare_with_fp64(const std::vector<float>& got, const std::vector<double>& ref) {
    Fp64Comparison c;
    c.finite = std::all_of(got.begin(), got.end(), [](float x) { return std::isfinite(x); });
    if (!c.finite) return c;
    const int T = int(std::max(1u, std::min(16u, std::thread::hardware_concurrency())));
    std::vector<double> e2(T, 0.0), r2(T, 0.0);
    std::vector<std::thread> th;
    for (int t = 0; t < T; ++t)
        th.emplace_back([&, t] {
            const size_t lo = got.size() * size_t(t) / size_t(T), hi = got.size() * size_t(t + 1) / size_t(T);
            for (size_t i = lo; i < hi; ++i) {
                const double d = double(got[i]) - ref[i];
                e2[t] += d * d;
                r2[t] += ref[i] * ref[i];
            }
        });
    for (auto& x : th) x.join();
    c.err_norm = std::sqrt(std::accumulate(e2.begin(), e2.end(), 0.0));
    c.ref_norm = std::sqrt(std::accumulate(r2.begin(), r2.end(), 0.0));
    return c;
}

// Acceptance of a result: ||C - ref|| <= norm_factor * ||ref|| + 1e-5 * sqrt(numel), and the
// relative error at most rel_cap (the second bound keeps an all-zero C from passing on a reference
// whose norm is tiny). FP16-input kernels get the looser pair.
struct Acceptance {
    double norm_factor, rel_cap;
};
Acceptance acceptance_for(const std::string& kernel) {
    const bool fp16_inputs = kernel == "vcsr_mc" || kernel == "cusparse_fp16";
    return fp16_inputs ? Acceptance{3e-3, 1e-1} : Acceptance{1e-4, 1e-2};
}
bool accepted(const Fp64Comparison& c, const Acceptance& a, size_t numel) {
    if (!c.finite) return false;
    const double bound = a.norm_factor * c.ref_norm + 1e-5 * std::sqrt(double(numel));
    return c.err_norm <= bound && c.rel_l2() <= a.rel_cap;
}

// Mean and median of the timed launches.
struct TimingSummary {
    double mean = 0, median = 0;
};
TimingSummary summarize(std::vector<double> ms) {
    TimingSummary s;
    if (ms.empty()) return s;
    s.mean = std::accumulate(ms.begin(), ms.end(), 0.0) / double(ms.size());
    const size_t n = ms.size(), hi = n / 2;
    std::nth_element(ms.begin(), ms.begin() + hi, ms.end());
    s.median = ms[hi];
    if (n % 2 == 0) s.median = 0.5 * (s.median + *std::max_element(ms.begin(), ms.begin() + hi));
    return s;
}

// One line of output per kernel.
struct ResultRow {
    std::string algo, validation, plan;
    double ms = 0, gflops = 0, rel_l2 = 0, ms_mean = 0, ms_median = 0;
    double setup_ms = 0, convert_ms = 0, upload_ms = 0;
    double gbps_alg = 0, roofline_frac = -1;  // frac < 0: no peak given
};
// Fixed columns of every row of a run.
struct RunColumns {
    std::string gpu, source;
    int sm = 0, O = 0, segw = 0, bundle = 0, tileK = 0, repeat = 0;
};
constexpr const char* kCsvHeader =
    "gpu,sm,mtx,O,segw,bundle,tileK,repeat,algo,ms,gflops,validation,rel_l2,setup_ms,ms_mean,ms_median,"
    "convert_ms,upload_ms,plan,gbps_alg,roofline_frac";

void print_result(const ResultRow& r, const RunColumns& run, bool csv) {
    if (csv) {
        char frac[32] = "";
        if (r.roofline_frac >= 0) std::snprintf(frac, sizeof frac, "%.6g", r.roofline_frac);
        std::printf("%s,%d,%s,%d,%d,%d,%d,%d,%s,%.9g,%.9g,%s,%.9g,%.6g,%.9g,%.9g,%.6g,%.6g,%s,%.6g,%s\n",
                    csv_quote(run.gpu).c_str(), run.sm, csv_quote(run.source).c_str(), run.O, run.segw, run.bundle,
                    run.tileK, run.repeat, r.algo.c_str(), r.ms, r.gflops, r.validation.c_str(), r.rel_l2,
                    r.setup_ms, r.ms_mean, r.ms_median, r.convert_ms, r.upload_ms, r.plan.c_str(), r.gbps_alg, frac);
    } else {
        std::printf("%-20s %10.6f %12.2f   %s (rel_l2=%.3g, setup %.3f ms, plan %s)\n", r.algo.c_str(), r.ms,
                    r.gflops, r.validation.c_str(), r.rel_l2, r.setup_ms, r.plan.c_str());
    }
    std::fflush(stdout);
}

// Compulsory bytes of one SpMM: per entry its column index and value (a_bytes), row_ptr, the
// `distinct` rows of B that A touches (O values of b_bytes each), and C (fp32) written once.
double algorithmic_bytes(const CSR& csr, int64_t distinct, int O, int a_bytes, int b_bytes) {
    return double(csr.nnz) * (4 + a_bytes) + (double(csr.M) + 1) * 4 + double(distinct) * O * b_bytes +
           double(csr.M) * O * 4;
}

// Host wall time of one call, in milliseconds.
template <class F>
float host_ms(F&& f) {
    using clock = std::chrono::steady_clock;
    const clock::time_point start = clock::now();
    f();
    const std::chrono::duration<double, std::milli> spent = clock::now() - start;
    return float(spent.count());
}

}  // namespace

static int benchmark_main(int argc, char** argv) {
    std::string mtx, gen, algo = "all", check = "cpu", reorder = "none", bdist = "pattern", stat = "mean",
                         plan = "auto";
    int O = 128, segw = 16, tileK = 64, repeat = 10, warmup = 3;
    uint64_t seed = 0;
    bool csv = false, lenient = false, b16 = false, flush_l2 = false;
    double peak_gbs = 0;
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
        {"flush-l2", no_argument, nullptr, 'F'},     {"peak-gbs", required_argument, nullptr, 'P'},
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
            case 'F': flush_l2 = true; break;
            case 'P': peak_gbs = std::strtod(optarg, nullptr); break;
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
    if (plan != "auto" && plan != "rows" && plan != "segment" && plan != "band" && plan != "hybrid")
        throw std::runtime_error("Unknown --plan: " + plan);
    const int plan_id = plan == "rows"      ? VCSRMC_PLAN_ROWS
                        : plan == "segment" ? VCSRMC_PLAN_SEGMENT
                        : plan == "band"    ? VCSRMC_PLAN_BAND
                        : plan == "hybrid"  ? VCSRMC_PLAN_HYBRID
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
    int64_t distinct = 0;
    {
        std::vector<char> used(size_t(std::max(csr.N, 1)), 0);
        for (int p = 0; p < csr.nnz; ++p) used[size_t(csr.col[p])] = 1;
        for (char u : used) distinct += u;
    }
    void* flush_buf = nullptr;
    size_t flush_bytes = 0;
    if (flush_l2) {
        flush_bytes = 2 * size_t(std::max(device.l2CacheSize, 1 << 20));
        cuda_ok(cudaMalloc(&flush_buf, flush_bytes), "cudaMalloc");
    }
    int flushes = 0;
    RunColumns run_cols;
    run_cols.gpu = device.name;
    run_cols.sm = device.major * 10 + device.minor;
    run_cols.source = source;
    run_cols.O = O;
    run_cols.segw = segw;
    run_cols.bundle = bundle;
    run_cols.tileK = tileK;
    run_cols.repeat = repeat;
    if (csv) {
        std::printf("%s\n", kCsvHeader);
    } else {
        std::printf("Matrix: %d x %d, nnz=%d; O=%d segw=%d bundle=%d tileK=%d repeat=%d warmup=%d reorder=%s; "
                    "reference=%s\n",
                    csr.M, csr.N, csr.nnz, O, segw, bundle, tileK, repeat, warmup, reorder.c_str(), check.c_str());
        std::printf("Kernel                Time (ms)      GFLOP/s   Validation\n");
    }
    // One launch on a zeroed C (C += A*B), its event time in ms.
    auto launch_once = [&](const std::function<float()>& run) {
        cuda_ok(cudaMemsetAsync(dC, 0, elementsC * sizeof(float), st), "cudaMemsetAsync");
        if (flush_buf) cuda_ok(cudaMemsetAsync(flush_buf, ++flushes & 0xff, flush_bytes, st), "cudaMemsetAsync");
        cuda_ok(cudaStreamSynchronize(st), "cudaStreamSynchronize");
        const float ms = csr.nnz ? run() : 0.f;
        cuda_ok(cudaStreamSynchronize(st), "cudaStreamSynchronize");
        if (!std::isfinite(ms) || ms < 0) throw std::runtime_error("Invalid kernel timing");
        return double(ms);
    };
    // Warm-up launches (discarded), `repeat` timed launches, then the last C against the fp64 result.
    auto measure = [&](const char* name, const std::function<float()>& run, float setup_ms, float convert_ms,
                       float upload_ms, const char* plan_used) {
        for (int it = 0; it < warmup; ++it) launch_once(run);
        std::vector<double> times;
        times.reserve(size_t(repeat));
        for (int it = 0; it < repeat; ++it) times.push_back(launch_once(run));
        ResultRow row;
        row.algo = name;
        row.plan = plan_used;
        row.validation = "unchecked";
        if (check != "none") {
            std::vector<float> result(elementsC);
            cuda_ok(cudaMemcpy(result.data(), dC, elementsC * sizeof(float), cudaMemcpyDeviceToHost), "cudaMemcpy");
            const Fp64Comparison cmp = compare_with_fp64(result, reference);
            if (!cmp.finite && !lenient) throw std::runtime_error(std::string(name) + ": non-finite output");
            row.rel_l2 = cmp.rel_l2();
            const bool ok = accepted(cmp, acceptance_for(name), elementsC);
            if (!ok && cmp.finite && !lenient)
                throw std::runtime_error(std::string(name) + ": correctness check failed, rel_l2=" +
                                         std::to_string(row.rel_l2));
            row.validation = ok ? "pass" : "FAIL";
        }
        const TimingSummary t = summarize(times);
        row.ms_mean = t.mean;
        row.ms_median = t.median;
        row.ms = stat == "median" ? t.median : t.mean;
        row.gflops = row.ms > 0 ? (2.0 * csr.nnz * O) / (row.ms * 1e6) : 0;
        {
            const std::string k(name);
            const bool fp16_a = k == "vcsr_mc" || k == "cusparse_fp16";
            const bool fp16_b = k == "cusparse_fp16" || (k == "vcsr_mc" && b16);
            const double bytes = algorithmic_bytes(csr, distinct, O, fp16_a ? 2 : 4, fp16_b ? 2 : 4);
            row.gbps_alg = row.ms > 0 ? bytes / (row.ms * 1e6) : 0;
            if (peak_gbs > 0) row.roofline_frac = row.gbps_alg / peak_gbs;
        }
        row.setup_ms = setup_ms;
        row.convert_ms = convert_ms;
        row.upload_ms = upload_ms;
        print_result(row, run_cols, csv);
    };

    for (const bool fp32 : {false, true}) {
        const char* name = fp32 ? "vcsr_mc_fp32" : "vcsr_mc";
        if (!selected(name)) continue;
        VCSRMC V;
        const float convert = host_ms([&] { V = csr_to_vcsr_mc(csr, fp32, segw); });
        const bool use_b16 = b16 && !fp32;
        if (use_b16 && !dB16) {
            std::vector<__half> h(elementsB);
            for (size_t i = 0; i < elementsB; ++i) h[i] = __float2half_rn(hB[i]);
            cuda_ok(cudaMalloc(&dB16, elementsB * sizeof(__half)), "cudaMalloc");
            cuda_ok(cudaMemcpy(dB16, h.data(), elementsB * sizeof(__half), cudaMemcpyHostToDevice), "cudaMemcpy");
        }
        if (plan_id == VCSRMC_PLAN_AUTO && !use_b16) {
            // the reference's own call sequence (src/main.cpp:356-361)
            const float upload = host_ms([&] { upload_vcsr_mc_device(V); });
            measure(name, [&] { float ms = 0; run_vcsr_mc_spmm_gpu(V, dB, O, tileK, dC, st, ms); return ms; },
                    convert + upload, convert, upload, "auto");
            destroy_vcsr_mc_device(st);
        } else {
            vcsrmc_csr* hc = nullptr;
            vcsrmc_format* hf = nullptr;
            vcsrmc_device_format* hd = nullptr;
            abi_ok(vcsrmc_csr_from_arrays(csr.M, csr.N, csr.nnz, csr.row_ptr.data(), csr.col.data(), csr.val.data(), &hc));
            abi_ok(vcsrmc_build_host(hc, fp32 ? 1 : 0, segw, 0, &hf));
            // the BAND and HYBRID plans run on the tensor cores (FP16 format); the FP32 format takes ROWS
            const bool tensor_plan = plan_id == VCSRMC_PLAN_BAND || plan_id == VCSRMC_PLAN_HYBRID;
            const int my_plan = (tensor_plan && fp32) ? VCSRMC_PLAN_ROWS : plan_id;
            const int mask = (my_plan == VCSRMC_PLAN_BAND || my_plan == VCSRMC_PLAN_HYBRID) ? (1 << my_plan) : 0;
            const char* my_plan_name = my_plan == plan_id ? plan.c_str() : "rows";
            const float upload = host_ms([&] { abi_ok(vcsrmc_upload_ex(hf, device_id, mask, st, &hd)); });
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
    cudaFree(flush_buf);
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
