#pragma once
// CpuPollingThread: the reference's host entry object for direct submit and for
// consuming the GPU-written descriptor ring.
//
// Same public interface as the reference include/gfd/cpu_polling.h:21-85 (constructor
// arguments, init_copy_engine, init_direct_ce, submit_direct, set_tiled_queue,
// set_sg_task_queue, start/stop, statistics getters, reset_stats).  What runs
// underneath is different:
//   submit_direct   validates the entries and launches the sm_100a SM-pull gather
//                   (gfd_gather_sync); no host core touches payload bytes, no staging
//                   copy, no gather workers.  Returns host latency in microseconds or
//                   -1.0 on error (count == 0 is an error, as in the reference).
//                   Sources may be pageable, as in the reference: a pageable cpu_base
//                   window is pinned for the poller's lifetime (cudaHostRegister, first
//                   use), so its tokens take the SM pull; other pageable sources go to
//                   the copy engine through the driver's staging (GFD_GATHER_PAGEABLE).
//   start / stop    run the ring agent, a device-resident kernel that polls the ring's
//                   commit markers, pulls the bytes, clears the markers, advances
//                   read_idx and publishes done_idx / tile counters / list completion;
//                   a host service thread only launches it and answers range queries.
//                   stop() drains every committed slot first (reference
//                   src/cpu_polling.cpp:438-489).
// Constructor arguments that select host cores (core_offset, exclusive_core_base,
// exclusive_core_count) only place the service thread; num_ce_channels sizes the
// copy-engine manager; use_ce is accepted for compatibility (the GPU consumer can
// write both device and managed memory, so both settings take the same path).

#include <atomic>
#include <cstdint>
#include <cstring>
#include <thread>

#include "gfd/copy_engine.h"
#include "gfd/tiled_queue.h"

struct gfd_ctx;
struct gfd_ring;

namespace gfd {

struct SGTaskQueue;

constexpr int MAX_GATHER_WORKERS = 15;
constexpr int NUM_GATHER_WORKERS = 7;

class CpuPollingThread {
public:
    CpuPollingThread(DescriptorQueue* queue, void* gpu_base, void* cpu_base, size_t total_cpu_size,
                     bool use_ce = true, int numa_node = 0, int core_offset = 0,
                     int num_ce_channels = 0, int exclusive_core_base = -1,
                     int exclusive_core_count = 0);
    ~CpuPollingThread();
    CpuPollingThread(const CpuPollingThread&) = delete;
    CpuPollingThread& operator=(const CpuPollingThread&) = delete;

    bool init_copy_engine();
    double submit_direct(const SGEntry* entries, int count);
    bool init_direct_ce();

    void set_tiled_queue(TiledQueue* tq) { tiled_queue_ = tq; }
    void set_sg_task_queue(SGTaskQueue* sq) { sg_queue_ = sq; }

    void start();
    void stop();

    uint64_t get_descriptors_processed() const;
    uint64_t get_batches_submitted() const;
    uint64_t get_coalesced_entries() const { return coalesced_entries_.load(std::memory_order_relaxed); }
    uint64_t get_staging_batches() const { return 0; }  // no staging copies exist
    double get_total_bytes_copied() const;
    const CopyEngineManager& get_ce_manager() const { return ce_manager_; }
    bool is_ce_mode() const { return use_ce_; }
    uint64_t get_gather_us() const { return 0; }  // no host gather
    uint64_t get_dma_wait_us() const { return dma_wait_us_.load(std::memory_order_relaxed); }
    uint64_t get_dma_submit_us() const { return 0; }
    uint64_t get_queue_read_us() const { return 0; }

    void reset_stats();

    // ---- library additions ----
    gfd_ctx* context() const { return ctx_; }
    gfd_ring* ring() const { return ring_; }

private:
    bool ensure_context();

    DescriptorQueue* queue_;
    TiledQueue* tiled_queue_ = nullptr;
    SGTaskQueue* sg_queue_ = nullptr;
    void* gpu_base_;
    void* cpu_base_;
    size_t total_cpu_size_;
    bool use_ce_;
    int numa_node_;
    int core_offset_;
    int num_ce_channels_;
    int exclusive_core_base_;
    int exclusive_core_count_;

    gfd_ctx* ctx_ = nullptr;
    gfd_ring* ring_ = nullptr;
    TiledQueue* ring_tq_ = nullptr;   // queues the ring was created with
    SGTaskQueue* ring_sq_ = nullptr;
    bool running_ = false;
    bool pinned_window_ = false;  // this poller pinned a pageable cpu_base window
    CopyEngineManager ce_manager_;

    // direct-submit counters (ring counters are added on read)
    std::atomic<uint64_t> direct_descriptors_{0};
    std::atomic<uint64_t> direct_batches_{0};
    std::atomic<uint64_t> direct_bytes_{0};
    std::atomic<uint64_t> coalesced_entries_{0};
    std::atomic<uint64_t> dma_wait_us_{0};
    // ring counters at the last reset_stats()
    uint64_t ring_desc_base_ = 0, ring_drain_base_ = 0, ring_bytes_base_ = 0;
};

}  // namespace gfd
