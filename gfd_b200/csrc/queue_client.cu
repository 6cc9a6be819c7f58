// GPU-queued submit client, timed the way the reference times its queue mode
// (examples/04_benchmark.cu:31-54 and 162-190): a submit kernel writes one descriptor
// per token with gfd::device::write_and_commit, a one-thread kernel waits for
// done_idx, and the host measures both launches plus cudaDeviceSynchronize.
//
// Only names the reference's public headers also declare are used (DescriptorQueue,
// TokenInfo, CpuPollingThread, StagingPool, write_and_commit), so the same file builds
// against either include tree:
//   - include/ + libgfd_b200.so   -> gfd_b200/libgfd_queue_client.so (this library's
//     ring consumer: the device-resident ring agent);
//   - the reference's include/ + its src/*.cpp objects -> oracle/_ref/
//     libgfd_ref_queue.so (the reference's CPU poller + batch processor + copy engine),
//     built by oracle/Makefile for the benchmark's reference columns.
// The completion wait is this file's own and bounded (10 s, %globaltimer): a consumer
// that stops making progress ends the wait with a status instead of a spinning GPU.

#include <cuda_runtime.h>

#include <chrono>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <vector>

#include "gfd/cpu_polling.h"
#include "gfd/descriptor_queue.h"
#include "gfd/device.cuh"
#include "gfd/staging_pool.h"

namespace {

constexpr unsigned long long kWaitLimitNs = 10ull * 1000 * 1000 * 1000;

__global__ void qc_submit(gfd::DescriptorQueue* q, const gfd::TokenInfo* tok, void* gpu, int n, uint32_t ts,
                          uint64_t base) {
    const int tid = blockIdx.x * blockDim.x + threadIdx.x;
    const bool active = tid < n;
    gfd::device::write_and_commit(q, base, tid, active, active ? tok[tid].cpu_addr : 0, gpu, ts, n);
}

__device__ __forceinline__ unsigned long long qc_now() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

__global__ void qc_wait(gfd::DescriptorQueue* q, uint64_t expected, volatile int* status) {
    const unsigned long long t0 = qc_now();
    for (;;) {
        const uint64_t done = *reinterpret_cast<volatile uint64_t*>(&q->done_idx);
        if (done >= expected) {
            *status = 0;
            return;
        }
        if (qc_now() - t0 > kWaitLimitNs) {
            *status = 1;
            return;
        }
        __nanosleep(200);
    }
}

struct QueueClient {
    gfd::DescriptorQueue* q = nullptr;
    gfd::CpuPollingThread* poller = nullptr;
    gfd::TokenInfo* d_tok = nullptr;
    int cap = 0;
    int* status = nullptr;  // pinned, device-mapped
    void* gpu = nullptr;
    uint64_t base = 0;
};

}  // namespace

extern "C" {

// gpu_buf / cpu_buf / total: the poller's registered regions (cpu_buf pinned).
// exclusive_core_count: cores handed to the poller (the reference's benchmark uses 32).
void* qc_create(int device, void* gpu_buf, void* cpu_buf, size_t total, int exclusive_core_count) {
    if (cudaSetDevice(device) != cudaSuccess) return nullptr;
    auto* c = new QueueClient;
    c->gpu = gpu_buf;
    // managed ring, as the reference's benchmark allocates it (examples/04_benchmark.cu:355-357)
    if (cudaMallocManaged(&c->q, sizeof(gfd::DescriptorQueue)) != cudaSuccess ||
        cudaHostAlloc(&c->status, sizeof(int), cudaHostAllocMapped) != cudaSuccess) {
        delete c;
        return nullptr;
    }
    std::memset(c->q, 0, sizeof(gfd::DescriptorQueue));
    gfd::StagingPool::instance().init(1, total);
    c->poller = new gfd::CpuPollingThread(c->q, gpu_buf, cpu_buf, total, true, 0, 0, 0, 0, exclusive_core_count);
    if (!c->poller->init_copy_engine()) {
        std::fprintf(stderr, "qc_create: init_copy_engine failed\n");
        delete c->poller;
        cudaFree(c->q);
        cudaFreeHost(c->status);
        delete c;
        return nullptr;
    }
    c->poller->init_direct_ce();
    c->poller->start();
    return c;
}

// Runs warmup + iters submit/wait rounds of n tokens of token_size bytes read from
// cpu_addrs[i] and landing at gpu_buf + i * token_size.  us_out[iters] receives each
// timed round (host wall clock, microseconds).  Returns 0, 1 on a bad argument, 2 when a
// wait ran out (the consumer stopped), 3 on a CUDA error.
int qc_run(void* h, const uint64_t* cpu_addrs, int n, uint32_t token_size, int warmup, int iters,
           double* us_out) {
    auto* c = static_cast<QueueClient*>(h);
    if (c == nullptr || n <= 0 || n > gfd::QUEUE_SIZE || token_size == 0) return 1;
    if (n > c->cap) {
        if (c->d_tok) cudaFree(c->d_tok);
        if (cudaMalloc(&c->d_tok, n * sizeof(gfd::TokenInfo)) != cudaSuccess) return 3;
        c->cap = n;
    }
    std::vector<gfd::TokenInfo> tok(n);
    for (int i = 0; i < n; ++i) tok[i] = gfd::TokenInfo{cpu_addrs[i], static_cast<uint32_t>(i), 0u};
    if (cudaMemcpy(c->d_tok, tok.data(), n * sizeof(gfd::TokenInfo), cudaMemcpyHostToDevice) != cudaSuccess)
        return 3;
    int* d_status = nullptr;
    cudaHostGetDevicePointer(reinterpret_cast<void**>(&d_status), c->status, 0);
    const int threads = 256, blocks = (n + threads - 1) / threads;
    for (int i = 0; i < warmup + iters; ++i) {
        *c->status = -1;
        const auto t0 = std::chrono::high_resolution_clock::now();
        qc_submit<<<blocks, threads>>>(c->q, c->d_tok, c->gpu, n, token_size, c->base);
        c->base += static_cast<uint64_t>(n);
        qc_wait<<<1, 1>>>(c->q, c->base, d_status);
        if (cudaDeviceSynchronize() != cudaSuccess) return 3;
        const auto t1 = std::chrono::high_resolution_clock::now();
        if (*c->status != 0) return 2;
        if (i >= warmup && us_out) us_out[i - warmup] = std::chrono::duration<double, std::micro>(t1 - t0).count();
    }
    return 0;
}

void qc_destroy(void* h) {
    auto* c = static_cast<QueueClient*>(h);
    if (c == nullptr) return;
    c->poller->stop();
    delete c->poller;
    if (c->d_tok) cudaFree(c->d_tok);
    cudaFree(c->q);
    cudaFreeHost(c->status);
    delete c;
}

}  // extern "C"
