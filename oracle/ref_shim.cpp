// C-ABI shim over the reference's own host contract -- TEST INFRASTRUCTURE ONLY.
//
// Compiled by oracle/Makefile against include/contract.hpp of shubhxho/cuda-kernel
// where it lies (the header is not copied into this repository); output goes
// to oracle/_ref/. It serves two purposes:
//   * pins the plain-C oracle (swiglu_oracle.c) bit-for-bit against the
//     reference's own decode::matvec / decode::silu / decode::compare;
//   * is the "reference" CPU baseline that bench.py times on the host cores.
// The composition below follows src/benchmark.cu:89-94 (random_half),
// :116-121 (draw order) and :131-141 (FFN reference) of the reference.
#include "contract.hpp"

#include <cuda_fp16.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <random>
#include <thread>
#include <vector>

namespace {

float h2f(uint16_t bits) {
    __half_raw raw;
    raw.x = bits;
    return __half2float(__half(raw));
}

uint16_t f2h(float v) {
    __half_raw raw = __half_raw(__float2half_rn(v));
    return raw.x;
}

std::vector<float> to_float(const uint16_t* p, size_t n) {
    std::vector<float> out(n);
    for (size_t i = 0; i < n; ++i) out[i] = h2f(p[i]);
    return out;
}

// benchmark.cu:89-94
void random_half(std::mt19937& rng, size_t n, float scale, uint16_t* out) {
    std::uniform_real_distribution<float> dist(-scale, scale);
    for (size_t i = 0; i < n; ++i) out[i] = f2h(dist(rng));
}

// decode::matvec over rows [r0, r1) of a row-major fp16 matrix. The reference
// converts the whole fp16 matrix to fp32 before its matvec (to_float,
// src/benchmark.cu:84-87); here each block of rows (at most 1 MiB of fp32) is
// converted and multiplied in turn, so the conversion cost stays in the timing but
// no thread allocates or re-reads a matrix-sized fp32 copy. Every row is still
// reduced by decode::matvec in column order: the results are the same bits.
void matvec_rows(const uint16_t* w, const std::vector<float>& x, int r0, int r1, float* y) {
    const size_t cols = x.size();
    if (r1 <= r0 || cols == 0) return;
    const int block = int(std::max<size_t>(1, (size_t(1) << 18) / cols));
    for (int b0 = r0; b0 < r1; b0 += block) {
        const int b1 = std::min(r1, b0 + block);
        std::vector<float> slice = to_float(w + size_t(b0) * cols, size_t(b1 - b0) * cols);
        std::vector<float> out = decode::matvec(slice, x, b1 - b0);
        std::copy(out.begin(), out.end(), y + b0);
    }
}

void matvec_threads(const uint16_t* w, const std::vector<float>& x, int rows, float* y, int threads) {
    if (threads <= 1) {
        matvec_rows(w, x, 0, rows, y);
        return;
    }
    std::vector<std::thread> pool;
    for (int t = 0; t < threads; ++t) {
        const int r0 = int(int64_t(rows) * t / threads), r1 = int(int64_t(rows) * (t + 1) / threads);
        pool.emplace_back(matvec_rows, w, std::cref(x), r0, r1, y);
    }
    for (auto& th : pool) th.join();
}

}  // namespace

extern "C" {

int ref_workload(unsigned seed, int hidden, int inter, uint16_t* wg, uint16_t* wu, uint16_t* wd,
                 uint16_t* x, uint16_t* bg, uint16_t* bu, uint16_t* bd) {
    if (hidden <= 0 || inter <= 0) return -1;
    std::mt19937 rng(seed);
    const size_t n = size_t(hidden) * size_t(inter);
    random_half(rng, n, 1 / std::sqrt(float(hidden)), wg);
    random_half(rng, n, 1 / std::sqrt(float(hidden)), wu);
    random_half(rng, n, 1 / std::sqrt(float(inter)), wd);
    random_half(rng, size_t(hidden), 1, x);
    random_half(rng, size_t(inter), .1f, bg);
    random_half(rng, size_t(inter), .1f, bu);
    random_half(rng, size_t(hidden), .1f, bd);
    return 0;
}

// benchmark.cu:131-141. threads > 1 splits the rows of each matvec across host
// threads; every row is still reduced by decode::matvec in column order.
int ref_ffn(const uint16_t* wg, const uint16_t* wu, const uint16_t* wd, const uint16_t* x,
            const uint16_t* bg, const uint16_t* bu, const uint16_t* bd, int hidden, int inter,
            float* proj, uint16_t* act, float* y, int threads) {
    try {
        if (hidden <= 0 || inter <= 0 || !y) return -1;
        auto fx = to_float(x, size_t(hidden));
        std::vector<float> g(inter), u(inter), a(inter);
        matvec_threads(wg, fx, inter, g.data(), threads);
        matvec_threads(wu, fx, inter, u.data(), threads);
        for (int i = 0; i < inter; ++i) {
            double v = decode::silu(double(g[i]) + h2f(bg[i])) * (double(u[i]) + h2f(bu[i]));
            a[i] = h2f(f2h(float(v)));
            if (act) act[i] = f2h(float(v));
        }
        matvec_threads(wd, a, hidden, y, threads);
        for (int i = 0; i < hidden; ++i) y[i] += fx[i] + h2f(bd[i]);
        if (proj) std::copy(g.begin(), g.end(), proj);
        return 0;
    } catch (...) {
        return -1;
    }
}

int ref_matvec(const float* w, const float* x, int rows, int cols, float* y) {
    try {
        std::vector<float> wv(w, w + size_t(rows) * size_t(cols)), xv(x, x + cols);
        auto out = decode::matvec(wv, xv, rows);
        std::copy(out.begin(), out.end(), y);
        return 0;
    } catch (const std::invalid_argument&) {
        return -1;
    }
}

double ref_silu(double v) { return decode::silu(v); }

int ref_compare(const float* a, const float* e, size_t n, double atol, double rtol, double* max_abs,
                double* max_scaled, int* passed) {
    try {
        auto err = decode::compare(std::vector<float>(a, a + n), std::vector<float>(e, e + n), atol, rtol);
        *max_abs = err.max_abs;
        *max_scaled = err.max_scaled;
        *passed = err.passed ? 1 : 0;
        return 0;
    } catch (const std::invalid_argument&) {
        return -1;
    }
}

int ref_median(const double* xs, size_t n, double* out) {
    try {
        *out = decode::median(std::vector<double>(xs, xs + n));
        return 0;
    } catch (const std::invalid_argument&) {
        return -1;
    }
}

int ref_hardware_threads(void) { return int(std::thread::hardware_concurrency()); }

}  // extern "C"
