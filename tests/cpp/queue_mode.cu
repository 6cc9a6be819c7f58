// GPU-queued submit through the reference device API (write_and_commit /
// fence_and_commit / wait_for_completion) consumed by CpuPollingThread::start()
// (GPU drain kernels).  Mirrors the methodology of the reference
// examples/04_benchmark.cu (submit kernel + wait kernel, base_slot advancing across
// launches) and examples/01_basic_transfer.cu (submit, compute, wait in one kernel).
#include <gfd/device.cuh>
#include <gfd/gfd.h>

#include "common.h"

__global__ void submit_kernel(gfd::DescriptorQueue* q, const gfd::TokenInfo* tokens, void* gpu_buffer, int n,
                              uint32_t token_size, uint64_t base_slot) {
    const int tid = blockIdx.x * blockDim.x + threadIdx.x;
    const bool active = tid < n;
    gfd::device::write_and_commit(q, base_slot, tid, active, active ? tokens[tid].cpu_addr : 0, gpu_buffer,
                                  token_size, n);
}

__global__ void wait_kernel(gfd::DescriptorQueue* q, uint64_t expected, int* ok) {
    *ok = gfd::device::wait_for_completion_until(q, expected, 5000000000ull) ? 1 : 0;
}

// submit, unrelated compute, wait, then read the landed token (example 01 pattern)
__global__ void fused_kernel(gfd::DescriptorQueue* q, const gfd::TokenInfo* tokens, float* gpu_buffer, int n,
                             uint32_t token_size, uint64_t base_slot, float* sums) {
    const int tid = blockIdx.x * blockDim.x + threadIdx.x;
    const bool active = tid < n;
    if (active)
        gfd::device::write_descriptor(q, base_slot, tid, tokens[tid].cpu_addr, gpu_buffer, token_size, n);
    gfd::device::fence_and_commit(q, base_slot, tid, active);
    float acc = 0.f;
    for (int i = 0; i < 1000; ++i) acc += __sinf(acc + tid);
    if (threadIdx.x == 0) gfd::device::wait_for_completion(q, base_slot + n);
    __syncthreads();
    if (active) {
        const float* tok = reinterpret_cast<const float*>(reinterpret_cast<const char*>(gpu_buffer) +
                                                           static_cast<size_t>(tid) * token_size);
        float s = 0.f;
        for (uint32_t d = 0; d < token_size / 4; ++d) s += tok[d];
        sums[tid] = s + 0.f * acc;
    }
}

static void run(bool managed) {
    const int N = 2048;
    const uint32_t T = 4096;
    const size_t stride = 2 * T;
    char* cpu;
    CK(cudaMallocHost(&cpu, N * stride));
    fill_pattern(cpu, N * stride, managed ? 5 : 6);
    char* gpu;
    CK(cudaMalloc(&gpu, (size_t)N * T));
    gfd::DescriptorQueue* q;
    if (managed) CK(cudaMallocManaged(&q, sizeof(gfd::DescriptorQueue)));
    else CK(cudaHostAlloc(&q, sizeof(gfd::DescriptorQueue), cudaHostAllocMapped));
    memset(q, 0, sizeof(*q));
    std::vector<gfd::TokenInfo> h(N);
    for (int i = 0; i < N; ++i) h[i] = gfd::TokenInfo{(uint64_t)(cpu + (size_t)i * stride), (uint32_t)i, 0};
    gfd::TokenInfo* d_tokens;
    CK(cudaMalloc(&d_tokens, N * sizeof(gfd::TokenInfo)));
    CK(cudaMemcpy(d_tokens, h.data(), N * sizeof(gfd::TokenInfo), cudaMemcpyHostToDevice));
    int* d_ok;
    CK(cudaMalloc(&d_ok, sizeof(int)));

    gfd::CpuPollingThread poller(q, gpu, cpu, N * stride, true, 0, 0, 0, 0, 32);
    if (!poller.init_copy_engine()) {
        report(managed ? "queue_managed_init" : "queue_mapped_init", false);
        return;
    }
    poller.start();
    uint64_t base = 0;
    bool all = true;
    // 12 rounds x 2048 descriptors = 24576 slots: the 16384-slot ring wraps
    for (int round = 0; round < 12; ++round) {
        CK(cudaMemset(gpu, 0, (size_t)N * T));
        CK(cudaDeviceSynchronize());
        submit_kernel<<<(N + 255) / 256, 256>>>(q, d_tokens, gpu, N, T, base);
        base += N;
        wait_kernel<<<1, 1>>>(q, base, d_ok);
        CK(cudaDeviceSynchronize());
        int ok = 0;
        CK(cudaMemcpy(&ok, d_ok, sizeof(int), cudaMemcpyDeviceToHost));
        std::vector<char> got((size_t)N * T);
        CK(cudaMemcpy(got.data(), gpu, got.size(), cudaMemcpyDeviceToHost));
        int bad = 0, first_bad = -1;
        for (int i = 0; i < N; ++i)
            if (memcmp(got.data() + (size_t)i * T, cpu + (size_t)i * stride, T) != 0) {
                if (first_bad < 0) first_bad = i;
                ++bad;
            }
        if (ok != 1 || bad)
            printf("  round %d: wait_ok=%d bad_tokens=%d first_bad=%d done_idx=%llu timeouts=%u\n", round, ok, bad,
                   first_bad, (unsigned long long)q->done_idx, (unsigned)q->wait_timeouts);
        all = all && ok == 1 && bad == 0;
    }
    char detail[128];
    snprintf(detail, sizeof(detail), "done_idx=%llu read_idx=%llu processed=%llu", (unsigned long long)q->done_idx,
             (unsigned long long)q->read_idx, (unsigned long long)poller.get_descriptors_processed());
    report(managed ? "queue_managed_submit_wait_wrap" : "queue_mapped_submit_wait_wrap",
           all && q->done_idx == base && poller.get_descriptors_processed() == base, detail);

    // fused submit + compute + wait in one kernel (8 CTAs leave room for the drains)
    float* sums;
    CK(cudaMalloc(&sums, N * sizeof(float)));
    const int n2 = 2048;
    for (int i = 0; i < n2; ++i) {
        float* tok = reinterpret_cast<float*>(cpu + (size_t)i * stride);
        for (uint32_t d = 0; d < T / 4; ++d) tok[d] = (float)(i % 97) + 0.5f;
    }
    fused_kernel<<<(n2 + 255) / 256, 256>>>(q, d_tokens, reinterpret_cast<float*>(gpu), n2, T, base, sums);
    base += n2;
    CK(cudaDeviceSynchronize());
    std::vector<float> hs(n2);
    CK(cudaMemcpy(hs.data(), sums, n2 * sizeof(float), cudaMemcpyDeviceToHost));
    bool fused_ok = q->wait_timeouts == 0;
    int fbad = 0, ffirst = -1;
    for (int i = 0; i < n2; ++i)
        if (hs[i] != ((float)(i % 97) + 0.5f) * (T / 4)) {
            if (ffirst < 0) ffirst = i;
            ++fbad;
        }
    if (fbad) printf("  fused: bad=%d first=%d got=%f want=%f timeouts=%u\n", fbad, ffirst, hs[ffirst],
                     ((float)(ffirst % 97) + 0.5f) * (T / 4), (unsigned)q->wait_timeouts);
    fused_ok = fused_ok && fbad == 0;
    report(managed ? "queue_managed_fused_kernel" : "queue_mapped_fused_kernel", fused_ok);
    poller.stop();
    CK(cudaFree(sums));
    CK(cudaFree(d_ok));
    CK(cudaFree(d_tokens));
    if (managed) CK(cudaFree(q));
    else CK(cudaFreeHost(q));
    CK(cudaFree(gpu));
    CK(cudaFreeHost(cpu));
}

// submit_direct reads any host memory, as the reference's CPU gather does.  The poller's
// pageable cpu_base window is pinned while the poller lives (SM pull) and released with
// it; a second pageable buffer outside the window goes to the copy engine; a pinned pool
// takes the SM pull.  Entries from all three in one call, with continuing entries (one
// merged run) and odd sizes, land byte for byte.
static bool registered(const void* p) {
    cudaPointerAttributes a;
    const bool r = cudaPointerGetAttributes(&a, p) == cudaSuccess && a.type == cudaMemoryTypeHost;
    cudaGetLastError();
    return r;
}

static void direct_pageable() {
    const size_t kSrc = 8u << 20, kOut = 4u << 20;
    std::vector<char> window(kSrc), other(kSrc);
    fill_pattern(window.data(), kSrc, 11);
    fill_pattern(other.data(), kSrc, 13);
    char* pinned;
    CK(cudaMallocHost(&pinned, kSrc));
    fill_pattern(pinned, kSrc, 12);
    char* gpu;
    CK(cudaMalloc(&gpu, kOut));
    CK(cudaMemset(gpu, 0, kOut));
    std::vector<char> expect(kOut, 0);
    std::vector<gfd::SGEntry> e;
    size_t dst = 0;
    uint64_t x = 7;
    for (int i = 0; i < 300 && dst < kOut - 70000; ++i) {
        x = x * 6364136223846793005ull + 1442695040888963407ull;
        const size_t n = 1 + (x >> 33) % 12000;
        const char* base = i % 3 == 0 ? pinned : i % 3 == 1 ? window.data() : other.data();
        const size_t src = (x >> 13) % (kSrc - 2 * n);
        e.push_back(gfd::SGEntry{reinterpret_cast<CUdeviceptr>(gpu + dst), base + src, n});
        memcpy(expect.data() + dst, base + src, n);
        dst += n;
        if (i % 5 == 1) {  // a continuing entry: one merged run
            e.push_back(gfd::SGEntry{reinterpret_cast<CUdeviceptr>(gpu + dst), base + src + n, n});
            memcpy(expect.data() + dst, base + src + n, n);
            dst += n;
        }
        dst += (x >> 40) % 8;
    }
    bool pinned_while_alive = false;
    double us = -1.0;
    bool zero_count = false;
    {
        gfd::CpuPollingThread poller(nullptr, gpu, window.data(), kSrc, true, 0, 0, 0, 0, 0);
        const bool init = poller.init_direct_ce();
        pinned_while_alive = init && registered(window.data()) && !registered(other.data());
        us = init ? poller.submit_direct(e.data(), static_cast<int>(e.size())) : -1.0;
        zero_count = poller.submit_direct(e.data(), 0) == -1.0;  // count 0 -> -1.0, as the reference
    }
    const bool released = !registered(window.data());
    const bool ok = pinned_while_alive && released && us >= 0.0 && zero_count && device_equals(gpu, expect.data(), kOut);
    char detail[160];
    snprintf(detail, sizeof(detail), "entries=%zu bytes=%zu us=%.1f window_pinned=%d released=%d", e.size(), dst, us,
             (int)pinned_while_alive, (int)released);
    report("direct_submit_pageable_and_pinned_sources", ok, detail);
    CK(cudaFree(gpu));
    CK(cudaFreeHost(pinned));
}

int main() {
    direct_pageable();
    run(false);
    run(true);
    return g_failures ? 1 : 0;
}
