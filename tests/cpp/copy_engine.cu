// gfd::CopyEngineManager through its C++ API (reference src/copy_engine.cpp:13-218):
// scattered entries from a pinned pool land byte for byte, entries that continue each
// other and evenly strided runs (merged into one copy / one 2D copy) land the same as
// separate copies, and the three completion routes -- wait_completion,
// record_event_on_last_stream, make_stream_wait_on_all -- order later work after the
// copies.
#include <gfd/copy_engine.h>

#include <random>

#include "common.h"

namespace {

constexpr size_t kPool = 64ull << 20;
constexpr size_t kOut = 16ull << 20;

struct Case {
    std::vector<gfd::SGEntry> entries;
    std::vector<uint8_t> expect;  // the output buffer after the copies
    uint64_t bytes = 0;
};

void add(Case& c, const uint8_t* pool, char* out, size_t src_off, size_t dst_off, size_t n) {
    c.entries.push_back(gfd::SGEntry{reinterpret_cast<CUdeviceptr>(out + dst_off), pool + src_off, n});
    if (n) memcpy(c.expect.data() + dst_off, pool + src_off, n);
    c.bytes += n;
}

Case random_case(const uint8_t* pool, char* out, uint64_t seed, int count, size_t limit = kOut) {
    Case c;
    c.expect.assign(kOut, 0);
    std::mt19937_64 rng(seed);
    size_t dst = 0;
    for (int i = 0; i < count; ++i) {
        const size_t n = 1 + rng() % 20000;
        const size_t src = rng() % (kPool - n);
        dst += rng() % 64;  // ragged gaps, any alignment
        if (dst + n > limit) break;
        add(c, pool, out, src, dst, n);
        dst += n;
    }
    return c;
}

// 2x-stride sources into 3x-stride destinations, then runs that continue each other
// (merged), a zero-size entry and a lone odd-sized entry.
Case strided_case(const uint8_t* pool, char* out) {
    Case c;
    c.expect.assign(kOut, 0);
    for (int i = 0; i < 256; ++i) add(c, pool, out, 1024 + size_t(i) * 8192, size_t(i) * 12288, 4096);
    size_t dst = 256 * 12288;
    for (int i = 0; i < 40; ++i) add(c, pool, out, (5u << 20) + size_t(i) * 1000, dst + size_t(i) * 1000, 1000);
    dst += 40 * 1000;
    add(c, pool, out, 7u << 20, dst, 0);
    add(c, pool, out, (9u << 20) + 3, dst + 5, 123457);
    return c;
}

bool out_equals(const char* out, const Case& c) { return device_equals(out, c.expect.data(), kOut); }

}  // namespace

int main() {
    CK(cudaSetDevice(0));
    uint8_t* pool = nullptr;
    CK(cudaHostAlloc(reinterpret_cast<void**>(&pool), kPool, cudaHostAllocMapped));
    fill_pattern(pool, kPool, 0xCE);
    char* out = nullptr;
    CK(cudaMalloc(&out, kOut));

    gfd::CopyEngineManager ce;
    report("ce_init", ce.init(nullptr) == CUDA_SUCCESS && ce.is_initialized());

    {  // scattered entries, one call, blocking
        CK(cudaMemset(out, 0, kOut));
        const Case c = random_case(pool, out, 1, 700);
        const CUresult r = ce.submit_and_wait(c.entries.data(), static_cast<int>(c.entries.size()));
        char d[96];
        snprintf(d, sizeof d, "entries=%zu bytes=%llu", c.entries.size(), (unsigned long long)c.bytes);
        report("ce_random_submit_and_wait", r == CUDA_SUCCESS && out_equals(out, c), d);
        report("ce_stats", ce.get_total_submissions() == 1 && ce.get_total_entries() == c.entries.size() &&
                               ce.get_total_bytes() == static_cast<double>(c.bytes));
    }
    {  // fewer entries than channels: one copy per stream
        CK(cudaMemset(out, 0, kOut));
        const Case c = random_case(pool, out, 2, 2);
        const CUresult r = ce.submit_and_wait(c.entries.data(), static_cast<int>(c.entries.size()));
        report("ce_two_entries", r == CUDA_SUCCESS && out_equals(out, c));
    }
    {  // strided and continuing runs, ordered through make_stream_wait_on_all
        CK(cudaMemset(out, 0, kOut));
        const Case c = strided_case(pool, out);
        cudaStream_t user;
        CK(cudaStreamCreateWithFlags(&user, cudaStreamNonBlocking));
        std::vector<uint8_t> back(kOut);
        CUresult r = ce.submit_scatter_gather(c.entries.data(), static_cast<int>(c.entries.size()));
        if (r == CUDA_SUCCESS) r = ce.make_stream_wait_on_all(user);
        CK(cudaMemcpyAsync(back.data(), out, kOut, cudaMemcpyDeviceToHost, user));
        CK(cudaStreamSynchronize(user));
        const bool ok = r == CUDA_SUCCESS && memcmp(back.data(), c.expect.data(), kOut) == 0;
        report("ce_strided_stream_wait", ok && ce.wait_completion() == CUDA_SUCCESS);
        CK(cudaStreamDestroy(user));
    }
    {  // several submissions, then an event on the last stream and a final wait
        CK(cudaMemset(out, 0, kOut));
        Case all;
        all.expect.assign(kOut, 0);
        bool ok = true;
        for (int k = 0; k < 4; ++k) {
            // each submission fills its own quarter of the output
            const size_t base = size_t(k) * (kOut / 4);
            const Case c = random_case(pool, out + base, 10 + k, 150, kOut / 4);
            memcpy(all.expect.data() + base, c.expect.data(), kOut / 4);
            ok = ok && ce.submit_scatter_gather(c.entries.data(), static_cast<int>(c.entries.size())) == CUDA_SUCCESS;
        }
        cudaEvent_t ev;
        CK(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
        ok = ok && ce.record_event_on_last_stream(ev) == CUDA_SUCCESS;
        CK(cudaEventSynchronize(ev));
        ok = ok && ce.wait_completion() == CUDA_SUCCESS;
        report("ce_multi_submit", ok && out_equals(out, all));
        CK(cudaEventDestroy(ev));
    }
    {  // an empty call is a no-op
        report("ce_empty", ce.submit_and_wait(nullptr, 0) == CUDA_SUCCESS);
    }
    ce.shutdown();
    report("ce_shutdown", !ce.is_initialized());

    CK(cudaFree(out));
    CK(cudaFreeHost(pool));
    printf("%s\n", g_failures ? "FAILED" : "ALL PASSED");
    return g_failures ? 1 : 0;
}
