// Helpers shared by the C++ API tests (built by tests/cpp_build.py, run by
// tests/test_cpp_api_gpu.py).  Every program prints one PASS/FAIL line per case and
// exits non-zero if any case failed.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <vector>

static int g_failures = 0;

#define CK(x)                                                                          \
    do {                                                                               \
        cudaError_t e_ = (x);                                                          \
        if (e_ != cudaSuccess) {                                                       \
            fprintf(stderr, "CUDA error %s at %s:%d\n", cudaGetErrorString(e_), __FILE__, __LINE__); \
            exit(2);                                                                   \
        }                                                                              \
    } while (0)

static inline void report(const char* name, bool ok, const char* detail = "") {
    printf("%s %s %s\n", ok ? "PASS" : "FAIL", name, detail);
    fflush(stdout);
    if (!ok) ++g_failures;
}

// splitmix64-based byte pattern that differs per (seed, offset)
static inline void fill_pattern(void* p, size_t n, uint64_t seed) {
    uint8_t* b = static_cast<uint8_t*>(p);
    uint64_t x = seed * 0x9E3779B97F4A7C15ull + 1;
    for (size_t i = 0; i < n; i += 8) {
        uint64_t z = (x += 0x9E3779B97F4A7C15ull);
        z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
        z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
        z ^= z >> 31;
        const size_t k = n - i < 8 ? n - i : 8;
        memcpy(b + i, &z, k);
    }
}

static inline bool device_equals(const void* d, const void* h, size_t n) {
    std::vector<uint8_t> tmp(n);
    CK(cudaMemcpy(tmp.data(), d, n, cudaMemcpyDeviceToHost));
    return memcmp(tmp.data(), h, n) == 0;
}
