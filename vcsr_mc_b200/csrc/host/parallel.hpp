// Minimal host thread helpers for the builders and generators (std::thread only).
#pragma once
#include <algorithm>
#include <atomic>
#include <cstdint>
#include <cstdlib>
#include <exception>
#include <mutex>
#include <thread>
#include <vector>

namespace vcsrmc {

// <= 0 means "all hardware threads" (VCSRMC_THREADS in the environment overrides that).
inline int resolve_threads(int n) {
    if (n > 0) return n;
    if (const char* env = std::getenv("VCSRMC_THREADS")) {
        const int v = std::atoi(env);
        if (v > 0) return v;
    }
    const unsigned hc = std::thread::hardware_concurrency();
    return hc ? int(std::min(hc, 256u)) : 1;
}

namespace detail {
template <class Body>
void run_threads(int nthreads, Body&& body) {
    if (nthreads <= 1) { body(0); return; }
    std::vector<std::thread> th;
    std::exception_ptr err;
    std::mutex mu;
    th.reserve(nthreads);
    for (int t = 0; t < nthreads; ++t)
        th.emplace_back([&, t] {
            try { body(t); } catch (...) {
                std::lock_guard<std::mutex> lk(mu);
                if (!err) err = std::current_exception();
            }
        });
    for (auto& x : th) x.join();
    if (err) std::rethrow_exception(err);
}
}  // namespace detail

// Static split of [begin, end) into one contiguous block per thread; fn(lo, hi).
template <class Fn>
void parallel_for(int64_t begin, int64_t end, int nthreads, Fn&& fn) {
    const int64_t n = end - begin;
    if (n <= 0) return;
    const int t = int(std::max<int64_t>(1, std::min<int64_t>(nthreads, n)));
    detail::run_threads(t, [&](int k) {
        const int64_t lo = begin + n * k / t, hi = begin + n * (k + 1) / t;
        if (lo < hi) fn(lo, hi);
    });
}

// Dynamic split: threads take chunks of `grain` indices from a shared counter; fn(lo, hi).
template <class Fn>
void parallel_for_dynamic(int64_t begin, int64_t end, int nthreads, int64_t grain, Fn&& fn) {
    const int64_t n = end - begin;
    if (n <= 0) return;
    grain = std::max<int64_t>(1, grain);
    const int t = int(std::max<int64_t>(1, std::min<int64_t>(nthreads, (n + grain - 1) / grain)));
    std::atomic<int64_t> next{begin};
    detail::run_threads(t, [&](int) {
        for (;;) {
            const int64_t lo = next.fetch_add(grain);
            if (lo >= end) break;
            fn(lo, std::min(end, lo + grain));
        }
    });
}

}  // namespace vcsrmc
