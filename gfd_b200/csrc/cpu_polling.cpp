// gfd::CpuPollingThread (include/gfd/cpu_polling.h) on top of the C ABI.
//
//  submit_direct -> gfd_gather_sync (SM-pull gather, host latency in microseconds;
//                   runs from pageable sources go to the copy engine);
//  start / stop  -> gfd_ring_start / gfd_ring_stop: the ring agent, a device-resident
//                   consumer of the descriptor queue.
// Statistics mirror the reference getters (src/cpu_polling.h:61-85): descriptors and
// bytes count both paths, "batches" counts direct calls plus ring drains.

#include <cuda_runtime.h>
#include <pthread.h>
#include <sched.h>

#include "gfd/cpu_polling.h"
#include "gfd/log.h"
#include "gfd/sg_task_queue.h"
#include "gfd_b200.h"

namespace gfd {

CpuPollingThread::CpuPollingThread(DescriptorQueue* queue, void* gpu_base, void* cpu_base,
                                   size_t total_cpu_size, bool use_ce, int numa_node, int core_offset,
                                   int num_ce_channels, int exclusive_core_base, int exclusive_core_count)
    : queue_(queue),
      gpu_base_(gpu_base),
      cpu_base_(cpu_base),
      total_cpu_size_(total_cpu_size),
      use_ce_(use_ce),
      numa_node_(numa_node),
      core_offset_(core_offset),
      num_ce_channels_(num_ce_channels),
      exclusive_core_base_(exclusive_core_base),
      exclusive_core_count_(exclusive_core_count) {}

CpuPollingThread::~CpuPollingThread() {
    stop();
    if (ring_) gfd_ring_destroy(ring_);
    ring_ = nullptr;
    ce_manager_.shutdown();
    if (ctx_ && pinned_window_) gfd_pool_unregister(ctx_, cpu_base_);
    if (ctx_) gfd_ctx_destroy(ctx_);
    ctx_ = nullptr;
}

bool CpuPollingThread::ensure_context() {
    if (ctx_) return true;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        GFD_LOG_ERROR("CpuPollingThread: no current CUDA device\n");
        return false;
    }
    if (gfd_ctx_create(dev, &ctx_) != GFD_OK) {
        GFD_LOG_ERROR("CpuPollingThread: gfd_ctx_create(%d) failed\n", dev);
        ctx_ = nullptr;
        return false;
    }
    // A pageable cpu_base window is pinned and mapped for the poller's lifetime, so tokens
    // in it take the SM pull like a cudaMallocHost pool.  The reference's CPU gather reads
    // any host memory; a kernel can read only pinned, mapped memory.  If pinning fails,
    // pageable entries still work, through the copy engine (GFD_GATHER_PAGEABLE).
    if (cpu_base_ != nullptr && total_cpu_size_ > 0) {
        cudaPointerAttributes a;
        if (cudaPointerGetAttributes(&a, cpu_base_) == cudaSuccess && a.type == cudaMemoryTypeUnregistered) {
            if (gfd_pool_register(ctx_, cpu_base_, total_cpu_size_) == GFD_OK) {
                pinned_window_ = true;
                GFD_LOG_INFO("CpuPollingThread: pinned the pageable cpu_base window (%zu bytes)\n",
                             total_cpu_size_);
            } else {
                GFD_LOG_INFO("CpuPollingThread: cpu_base window left pageable (%s); its tokens go to the "
                             "copy engine\n", gfd_last_error(ctx_));
            }
        }
        cudaGetLastError();
    }
    return true;
}

bool CpuPollingThread::init_copy_engine() {
    if (!ensure_context()) return false;
    if (ce_manager_.init(nullptr, num_ce_channels_) != CUDA_SUCCESS) return false;
    // create the ring consumer now (outside any later kernel launch); start() re-creates
    // it if set_tiled_queue / set_sg_task_queue change the attached queues afterwards
    if (queue_ != nullptr && ring_ == nullptr) {
        if (gfd_ring_create(ctx_, queue_, tiled_queue_, sg_queue_, &ring_) != GFD_OK) {
            GFD_LOG_ERROR("CpuPollingThread: %s\n", gfd_last_error(ctx_));
            ring_ = nullptr;
            return false;
        }
        ring_tq_ = tiled_queue_;
        ring_sq_ = sg_queue_;
    }
    return true;
}

bool CpuPollingThread::init_direct_ce() { return ensure_context(); }

double CpuPollingThread::submit_direct(const SGEntry* entries, int count) {
    if (count <= 0 || entries == nullptr || !ensure_context()) return -1.0;
    double us = 0.0;
    // pageable sources are accepted (copy engine), as the reference's CPU gather reads any
    // host memory; pinned ones take the SM pull
    const int rc = gfd_gather_sync(ctx_, reinterpret_cast<const gfd_sg_entry*>(entries), count,
                                   GFD_GATHER_PAGEABLE, &us);
    if (rc != GFD_OK) {
        GFD_LOG_ERROR("submit_direct: %s\n", gfd_last_error(ctx_));
        return -1.0;
    }
    uint64_t bytes = 0;
    for (int i = 0; i < count; ++i) bytes += entries[i].size;
    direct_descriptors_ += static_cast<uint64_t>(count);
    direct_batches_ += 1;
    direct_bytes_ += bytes;
    return us;
}

void CpuPollingThread::start() {
    if (running_ || queue_ == nullptr || !ensure_context()) return;
    if (ring_ != nullptr && (ring_tq_ != tiled_queue_ || ring_sq_ != sg_queue_)) {
        gfd_ring_destroy(ring_);
        ring_ = nullptr;
    }
    if (ring_ == nullptr) {
        ring_tq_ = tiled_queue_;
        ring_sq_ = sg_queue_;
        if (gfd_ring_create(ctx_, queue_, tiled_queue_, sg_queue_, &ring_) != GFD_OK) {
            GFD_LOG_ERROR("CpuPollingThread::start: %s\n", gfd_last_error(ctx_));
            ring_ = nullptr;
            return;
        }
    }
    // the windows the constructor names are trusted without a query (the agent still asks
    // the host once about any other range a descriptor uses)
    if (gpu_base_ != nullptr) gfd_ring_allow(ring_, gpu_base_, 0);
    if (cpu_base_ != nullptr) gfd_ring_allow(ring_, cpu_base_, 0);
    if (gfd_ring_start(ring_) != GFD_OK) {
        GFD_LOG_ERROR("CpuPollingThread::start: %s\n", gfd_last_error(ctx_));
        return;
    }
    running_ = true;
}

void CpuPollingThread::stop() {
    if (!running_ || ring_ == nullptr) return;
    if (gfd_ring_stop(ring_) != GFD_OK) GFD_LOG_ERROR("CpuPollingThread::stop: %s\n", gfd_last_error(ctx_));
    running_ = false;
}

uint64_t CpuPollingThread::get_descriptors_processed() const {
    uint64_t c = 0;
    if (ring_) gfd_ring_counters(ring_, &c, nullptr, nullptr);
    return direct_descriptors_.load() + c - ring_desc_base_;
}

uint64_t CpuPollingThread::get_batches_submitted() const {
    uint64_t d = 0;
    if (ring_) gfd_ring_counters(ring_, nullptr, &d, nullptr);
    return direct_batches_.load() + d - ring_drain_base_;
}

double CpuPollingThread::get_total_bytes_copied() const {
    uint64_t b = 0;
    if (ring_) gfd_ring_counters(ring_, nullptr, nullptr, &b);
    return static_cast<double>(direct_bytes_.load() + b - ring_bytes_base_);
}

void CpuPollingThread::reset_stats() {
    direct_descriptors_ = 0;
    direct_batches_ = 0;
    direct_bytes_ = 0;
    coalesced_entries_ = 0;
    dma_wait_us_ = 0;
    ring_desc_base_ = ring_drain_base_ = ring_bytes_base_ = 0;
    if (ring_) gfd_ring_counters(ring_, &ring_desc_base_, &ring_drain_base_, &ring_bytes_base_);
}

}  // namespace gfd
