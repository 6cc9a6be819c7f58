// TEST INFRASTRUCTURE ONLY -- extern "C" harness around the reference's own gather
// code, compiled together with the reference sources (oracle/Makefile, output in
// oracle/_ref/).  It never becomes part of libgfd_b200.
//
//  ref_parallel_gather  runs CpuPollingThread::parallel_gather (reference
//                       src/parallel_gather.cpp:74-116) with `workers` spin workers
//                       (gather_worker_loop, :44-72) on the host -- no GPU needed.
//  ref_direct_*         drive CpuPollingThread::submit_direct (src/direct_submit.cpp:
//                       28-164) exactly as examples/04_benchmark.cu:372-381 sets it
//                       up: StagingPool::init, use_ce=true, init_copy_engine,
//                       init_direct_ce.  Needs a GPU.
//  ref_memcpy_n         the reference benchmark's Memcpy(N) method
//                       (examples/04_benchmark.cu:92-115): one cudaMemcpyAsync per token
//                       on one stream, then a stream synchronize.
//  ref_host_alloc / ref_dev_alloc / ref_l2_flush / ref_verify
//                       what the benchmark's reference arm needs besides the reference
//                       itself, so that arm loads no library of this repository: the
//                       source pool from cudaMallocHost and the destination from
//                       cudaMalloc, as examples/04_benchmark.cu:346-356 allocates them;
//                       an L2 flush between calls; a byte compare of the gathered
//                       destination with the entries' sources.  The seeded input
//                       generators (gfd_b200/csrc/workload.c, gfdw_*) are linked in too.

// The harness reaches the private gather workers of CpuPollingThread directly.
#define private public
#include "gfd/cpu_polling.h"
#undef private
#include "gfd/staging_pool.h"

#include <cuda_runtime.h>
#include <chrono>
#include <cstring>
#include <thread>
#include <vector>

extern "C" {

int ref_parallel_gather(const void* entries, int n, void* staging, uint64_t min_dst, int workers) {
    if (workers < 0 || workers > gfd::MAX_GATHER_WORKERS) return -1;
    gfd::CpuPollingThread t(nullptr, nullptr, nullptr, 0, /*use_ce=*/false);
    t.active_gather_workers_ = workers;
    t.gather_workers_running_.store(true, std::memory_order_release);
    for (int i = 0; i < workers; ++i) {
        t.gather_tasks_[i].has_work.store(false);
        t.gather_tasks_[i].done.store(false);
        t.gather_threads_[i] = std::thread(&gfd::CpuPollingThread::gather_worker_loop, &t, i);
    }
    t.parallel_gather(static_cast<const gfd::SGEntry*>(entries), n, static_cast<char*>(staging),
                      static_cast<CUdeviceptr>(min_dst));
    t.gather_workers_running_.store(false, std::memory_order_release);
    for (int i = 0; i < workers; ++i) t.gather_threads_[i].join();
    return 0;
}

#ifndef GFD_REF_CPU_ONLY
struct RefDirect {
    gfd::DescriptorQueue* queue = nullptr;
    gfd::CpuPollingThread* poller = nullptr;
};

void* ref_direct_create(int device, void* gpu_buf, void* cpu_buf, size_t total, int excl_base,
                        int excl_count) {
    if (cudaSetDevice(device) != cudaSuccess) return nullptr;
    cudaFree(nullptr);  // make the primary context current on this thread
    RefDirect* h = new RefDirect();
    if (cudaMallocManaged(&h->queue, sizeof(gfd::DescriptorQueue)) != cudaSuccess) {
        delete h;
        return nullptr;
    }
    memset(h->queue, 0, sizeof(gfd::DescriptorQueue));
    gfd::StagingPool::instance().init(1, total);
    h->poller = new gfd::CpuPollingThread(h->queue, gpu_buf, cpu_buf, total, /*use_ce=*/true,
                                          /*numa_node=*/0, /*core_offset=*/0,
                                          /*num_ce_channels=*/0, excl_base, excl_count);
    if (!h->poller->init_copy_engine() || !h->poller->init_direct_ce()) {
        delete h->poller;
        cudaFree(h->queue);
        delete h;
        return nullptr;
    }
    return h;
}

int ref_direct_workers(void* hp) {
    return hp ? static_cast<RefDirect*>(hp)->poller->active_gather_workers_ : -1;
}

double ref_direct_submit(void* hp, const void* entries, int n) {
    RefDirect* h = static_cast<RefDirect*>(hp);
    return h->poller->submit_direct(static_cast<const gfd::SGEntry*>(entries), n);
}

void ref_direct_destroy(void* hp) {
    RefDirect* h = static_cast<RefDirect*>(hp);
    if (!h) return;
    delete h->poller;
    gfd::StagingPool::instance().shutdown();
    cudaFree(h->queue);
    delete h;
}

int ref_set_device(int device) { return cudaSetDevice(device) == cudaSuccess ? 0 : -1; }

void* ref_host_alloc(size_t bytes) {
    void* p = nullptr;
    if (cudaMallocHost(&p, bytes) != cudaSuccess) return nullptr;
    return p;
}

void ref_host_free(void* p) { cudaFreeHost(p); }

void* ref_dev_alloc(size_t bytes) {
    void* p = nullptr;
    if (cudaMalloc(&p, bytes) != cudaSuccess) return nullptr;
    return p;
}

void ref_dev_free(void* p) { cudaFree(p); }

// Overwrites a device buffer larger than L2 and waits, so the next call starts cold.
int ref_l2_flush(void* buf, size_t bytes) {
    if (cudaMemset(buf, 0, bytes) != cudaSuccess) return -1;
    return cudaDeviceSynchronize() == cudaSuccess ? 0 : -1;
}

// Copies the destination window back and compares every entry's bytes with its source:
// -1 when all match, the first mismatching entry's index, or -2 on a CUDA error / an
// entry outside the window.
long long ref_verify(const void* entries, int n, const void* dst_base, size_t dst_bytes) {
    const gfd::SGEntry* e = static_cast<const gfd::SGEntry*>(entries);
    std::vector<unsigned char> host(dst_bytes);
    if (cudaMemcpy(host.data(), dst_base, dst_bytes, cudaMemcpyDeviceToHost) != cudaSuccess) return -2;
    const uint64_t base = reinterpret_cast<uint64_t>(dst_base);
    for (int i = 0; i < n; ++i) {
        const uint64_t off = static_cast<uint64_t>(e[i].dst) - base;
        if (static_cast<uint64_t>(e[i].dst) < base || off > dst_bytes || e[i].size > dst_bytes - off) return -2;
        if (memcmp(host.data() + off, e[i].src, e[i].size) != 0) return i;
    }
    return -1;
}

double ref_memcpy_n(const void* entries, int n, void* stream) {
    const gfd::SGEntry* e = static_cast<const gfd::SGEntry*>(entries);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    auto t0 = std::chrono::high_resolution_clock::now();
    for (int i = 0; i < n; ++i)
        cudaMemcpyAsync(reinterpret_cast<void*>(e[i].dst), e[i].src, e[i].size,
                        cudaMemcpyHostToDevice, st);
    if (cudaStreamSynchronize(st) != cudaSuccess) return -1.0;
    auto t1 = std::chrono::high_resolution_clock::now();
    return std::chrono::duration<double, std::micro>(t1 - t0).count();
}
#endif

}  // extern "C"
