// backbone_fixture.hpp -- random Q4_K backbone weights on the device for the
// C++ programs under tests/cpp (scheduler_test.cpp, scheduler_timing.cpp).
#pragma once

#include <cstdint>
#include <stdexcept>
#include <vector>

#include <cuda_runtime.h>

#include "hkv.h"

namespace fixture {

inline uint64_t g_rng = 0x9E3779B97F4A7C15ull;
// Sum of four uniforms scaled to unit variance (test data only).
inline float next_normal() {
    float s = 0.f;
    for (int i = 0; i < 4; ++i) {
        g_rng = g_rng * 6364136223846793005ull + 1442695040888963407ull;
        s += static_cast<float>((g_rng >> 40) & 0xFFFFFF) / 16777216.0f - 0.5f;
    }
    return s * 1.7320508f;
}

inline std::vector<void *> g_allocs;
inline void *dmalloc(size_t bytes) {
    void *p = nullptr;
    if (cudaMalloc(&p, bytes) != cudaSuccess) throw std::runtime_error("cudaMalloc");
    g_allocs.push_back(p);
    return p;
}
inline void free_all() {
    for (void *p : g_allocs) cudaFree(p);
    g_allocs.clear();
}

// F32 [rows][cols] of N(0, 0.02) values on the device.
inline float *normal_f32(int64_t rows, int64_t cols) {
    std::vector<float> h(static_cast<size_t>(rows * cols));
    for (float &x : h) x = 0.02f * next_normal();
    float *f = static_cast<float *>(dmalloc(h.size() * 4));
    cudaMemcpy(f, h.data(), h.size() * 4, cudaMemcpyHostToDevice);
    return f;
}

// A new Q4_K matrix quantised from the device F32 matrix `f`.
inline const void *q4k_from(const float *f, int64_t rows, int64_t cols) {
    void *b = dmalloc(static_cast<size_t>(rows * cols / 256 * 144));
    char msg[256];
    if (hkv_q4k_quantize(f, rows, cols, b, nullptr, msg, sizeof msg) != HKV_OK) throw std::runtime_error(msg);
    return b;
}

inline const void *q4k(int64_t rows, int64_t cols) { return q4k_from(normal_f32(rows, cols), rows, cols); }

// [n] RMSNorm weights around 1.
inline const float *norm(int64_t n) {
    std::vector<float> h(static_cast<size_t>(n));
    for (float &x : h) x = 1.0f + 0.1f * next_normal();
    float *d = static_cast<float *>(dmalloc(h.size() * 4));
    cudaMemcpy(d, h.data(), h.size() * 4, cudaMemcpyHostToDevice);
    return d;
}

}  // namespace fixture
