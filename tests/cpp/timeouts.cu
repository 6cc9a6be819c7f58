// Failure detection without a GPU fault: every device-side wait of the library has a
// time limit, after which it returns an error status the host reads, and the context
// stays usable.  Each case makes one wait run out on purpose -- a counter or marker
// that nothing ever advances -- with a short limit, then checks the status, the
// give-up counters and that the next CUDA work still runs.  (The reference's waits spin
// forever: include/gfd/device.cuh:110-118, device_primitives.cuh:117-150,
// sg_warp_spec.cuh:109-127, 221-249.)
#include <gfd/gfd.h>
#include <gfd/device.cuh>
#include <gfd/device_primitives.cuh>
#include <gfd/sg_warp_spec.cuh>

#include <chrono>

#include "common.h"

using clk = std::chrono::steady_clock;
static double ms_since(clk::time_point t0) {
    return std::chrono::duration<double, std::milli>(clk::now() - t0).count();
}

constexpr uint64_t kLimitNs = 100ull * 1000 * 1000;  // 100 ms

__global__ void wait_done_kernel(gfd::DescriptorQueue* q, uint64_t expected, uint64_t limit, int* status) {
    *status = gfd::device::wait_for_completion_until(q, expected, limit) ? 0 : 1;
}

__global__ void wait_tile_kernel(gfd::TiledQueue* tq, uint32_t tile, uint64_t expected, uint64_t limit, int* status) {
    *status = gfd::device::wait_chunk_done_until(tq, tile, expected, limit) ? 0 : 1;
}

__global__ void sg_wait_done_kernel(gfd::SGTaskQueue* sq, uint64_t lists) {
    gfd::sg::sg_wait_list_done(sq, lists);  // lane 0 waits, bounded by sq->wait_limit_ns
}

__global__ void sg_submit_into_full_pool(gfd::SGTaskQueue* sq, int* status) {
    const gfd::sg::SGSubmitter sub(sq);
    const bool ok = sub.wait_entry_space(gfd::MAX_SG_POOL_ENTRIES);  // nobody consumes
    if ((threadIdx.x & 31) == 0) *status = ok ? 0 : 1;
}

struct Nop {
    __device__ void operator()(gfd::sg_warp_spec::SGListView) const {}
};
GFD_SG_WARP_SPEC_KERNEL(sg_idle_kernel, Nop);

__global__ void add_one(int* p) { *p += 1; }

static bool context_usable() {
    int* d = nullptr;
    if (cudaMalloc(&d, sizeof(int)) != cudaSuccess) return false;
    int h = 41;
    bool ok = cudaMemcpy(d, &h, sizeof(int), cudaMemcpyHostToDevice) == cudaSuccess;
    add_one<<<1, 1>>>(d);
    ok = ok && cudaDeviceSynchronize() == cudaSuccess;
    ok = ok && cudaMemcpy(&h, d, sizeof(int), cudaMemcpyDeviceToHost) == cudaSuccess && h == 42;
    cudaFree(d);
    return ok;
}

static void queue_wait_gives_up() {
    gfd::DescriptorQueue* q = nullptr;
    int* status = nullptr;
    CK(cudaHostAlloc(&q, sizeof(*q), cudaHostAllocMapped));
    CK(cudaHostAlloc(&status, sizeof(int), cudaHostAllocMapped));
    memset(q, 0, sizeof(*q));
    *status = -1;
    const auto t0 = clk::now();
    wait_done_kernel<<<1, 1>>>(q, 1, kLimitNs, status);  // no consumer: done_idx stays 0
    const cudaError_t e = cudaDeviceSynchronize();
    const double ms = ms_since(t0);
    char detail[160];
    snprintf(detail, sizeof(detail), "status=%d wait_timeouts=%u after %.0f ms", *status, q->wait_timeouts, ms);
    report("timeout_done_idx_wait", e == cudaSuccess && *status == 1 && q->wait_timeouts == 1 && ms >= 90 && ms < 5000,
           detail);
    report("timeout_done_idx_context_usable", context_usable());
    cudaFreeHost(q);
    cudaFreeHost(status);
}

static void tile_wait_gives_up() {
    gfd::TiledQueue* tq = nullptr;
    int* status = nullptr;
    CK(cudaHostAlloc(&tq, sizeof(*tq), cudaHostAllocMapped));
    CK(cudaHostAlloc(&status, sizeof(int), cudaHostAllocMapped));
    memset(tq, 0, sizeof(*tq));
    tq->tile_chunk_done[7] = 3;  // three tokens of tile 7 landed, the fourth never does
    *status = -1;
    const auto t0 = clk::now();
    wait_tile_kernel<<<1, 1>>>(tq, 7, 4, kLimitNs, status);
    const cudaError_t e = cudaDeviceSynchronize();
    const double ms = ms_since(t0);
    char detail[160];
    snprintf(detail, sizeof(detail), "status=%d wait_timeouts=%u after %.0f ms", *status, tq->base.wait_timeouts, ms);
    report("timeout_tile_chunk_wait", e == cudaSuccess && *status == 1 && tq->base.wait_timeouts == 1 && ms >= 90,
           detail);
    *status = -1;
    wait_tile_kernel<<<1, 1>>>(tq, 7, 3, kLimitNs, status);  // already satisfied: no wait
    report("tile_chunk_wait_satisfied", cudaDeviceSynchronize() == cudaSuccess && *status == 0);
    cudaFreeHost(tq);
    cudaFreeHost(status);
}

// SG consumers waiting for a list that is never submitted: they give up after the
// session's limit, record where (timeout_site), and the kernel ends on its own.
static void sg_consumers_give_up() {
    gfd::SGWarpSpecConfig cfg;
    cfg.num_compute_warps = 1;
    cfg.num_blocks = 4;
    cfg.wait_timeout_ms = 100;
    gfd::SGWarpSpecSession session(cfg);
    if (!session.ok()) {
        report("timeout_sg_consumers", false, "session init failed");
        return;
    }
    const auto t0 = clk::now();
    session.launch(sg_idle_kernel, Nop{});
    const cudaError_t e = cudaDeviceSynchronize();  // ends when the waits give up
    const double ms = ms_since(t0);
    gfd::SGTaskQueue* sq = session.get_sg_queue();
    char detail[200];
    snprintf(detail, sizeof(detail), "wait_timeouts=%u timeout_site=%u after %.0f ms", sq->wait_timeouts,
             sq->timeout_site, ms);
    // the producers' wait for the list's commit and the compute warps' wait for a list
    // both run out; timeout_site keeps the last one recorded
    const bool site_ok = sq->timeout_site == 2 /* list commit */ || sq->timeout_site == 4 /* compute slot */;
    const bool ok = e == cudaSuccess && sq->wait_timeouts >= 1 && site_ok && ms >= 90 && ms < 5000;
    session.synchronize();
    report("timeout_sg_consumers", ok && session.timeouts() >= 1, detail);
    report("timeout_sg_context_usable", context_usable());
}

// A device-side SG submitter whose pool never drains, and a wait for lists that never
// complete: both return once the limit passes.
static void sg_submitter_gives_up() {
    gfd::SGWarpSpecConfig cfg;
    cfg.wait_timeout_ms = 100;
    gfd::SGWarpSpecSession session(cfg);
    if (!session.ok()) {
        report("timeout_sg_submitter", false, "session init failed");
        return;
    }
    auto p = session.get_launch_params();  // prepares the queue (limits, mirror)
    gfd::SGTaskQueue* sq = p.sq;
    int* status = nullptr;
    CK(cudaHostAlloc(&status, sizeof(int), cudaHostAllocMapped));
    *status = -1;
    // occupy the pool: 16,000 entries allocated, none consumed
    sq->entry_alloc_idx = 16000;
    const auto t0 = clk::now();
    sg_submit_into_full_pool<<<1, 32>>>(sq, status);
    cudaError_t e = cudaDeviceSynchronize();
    double ms = ms_since(t0);
    char detail[160];
    snprintf(detail, sizeof(detail), "status=%d wait_timeouts=%u after %.0f ms", *status, sq->wait_timeouts, ms);
    report("timeout_sg_entry_space", e == cudaSuccess && *status == 1 && sq->wait_timeouts == 1 && ms >= 90, detail);
    const auto t1 = clk::now();
    sg_wait_done_kernel<<<1, 32>>>(sq, 5);
    e = cudaDeviceSynchronize();
    ms = ms_since(t1);
    snprintf(detail, sizeof(detail), "wait_timeouts=%u after %.0f ms", sq->wait_timeouts, ms);
    report("timeout_sg_list_done", e == cudaSuccess && sq->wait_timeouts == 2 && ms >= 90, detail);
    session.reset();
    cudaFreeHost(status);
}

int main() {
    CK(cudaSetDevice(0));
    queue_wait_gives_up();
    tile_wait_gives_up();
    sg_consumers_give_up();
    sg_submitter_gives_up();
    return g_failures ? 1 : 0;
}
