// WarpSpecSession / SGWarpSpecSession (include/gfd/warp_spec_session.h): lifecycle
// of the warp-specialised kernels.  Mirrors the reference src/warp_spec_session.cpp
// and src/sg_warp_spec_session.cpp (allocation of the host-mapped queues and the
// device completion arrays, poller ownership, synchronize / reset / get_stats), with
// three additions: the source and destination ranges are validated before any
// launch (a kernel never sees an address outside pinned host memory or device
// memory), host waits are bounded, and host list submission applies backpressure
// while a kernel is consuming.

#include <cuda_runtime.h>
#include <time.h>

#include <atomic>
#include <chrono>
#include <cstring>
#include <thread>
#include <vector>

#include "gfd/log.h"
#include "gfd/warp_spec_session.h"
#include "internal.h"

namespace gfd {
namespace {

uint64_t limit_ns(uint64_t ms) { return (ms ? ms : DEFAULT_WAIT_TIMEOUT_MS) * 1000000ull; }

bool range_ok(gfd_ctx* ctx, const void* p, uint64_t n, bool host) {
    if (ctx == nullptr || p == nullptr) return false;
    if (n == 0) return true;
    std::lock_guard<std::mutex> lk(ctx->mu);
    return host ? gfdb::check_host(ctx, reinterpret_cast<uint64_t>(p), n)
                : gfdb::check_dev(ctx, reinterpret_cast<uint64_t>(p), n);
}

// Bytes of pinned, device-mapped host memory from p to the end of its allocation.
uint64_t host_extent(gfd_ctx* ctx, const void* p) {
    if (ctx == nullptr || p == nullptr) return 0;
    std::lock_guard<std::mutex> lk(ctx->mu);
    const uint64_t a = reinterpret_cast<uint64_t>(p);
    if (!gfdb::check_host(ctx, a, 1)) return 0;
    const gfdb::Range* r = ctx->host_ranges.find(a, 1);
    return r ? r->hi - a : 0;
}

}  // namespace

// ===========================================================================
// WarpSpecSession
// ===========================================================================
WarpSpecSession::WarpSpecSession(const WarpSpecConfig& config) : config_(config) {
    if (config_.total_tokens == 0 || config_.token_size == 0) {
        GFD_LOG_ERROR("WarpSpecSession: total_tokens and token_size must be > 0\n");
        return;
    }
    const uint32_t C = config_.effective_tokens_per_chunk();
    if (config_.tokens_per_tile == 0 || C == 0) {
        GFD_LOG_ERROR("WarpSpecSession: tokens_per_tile and tokens_per_chunk must be > 0\n");
        return;
    }
    if (config_.tokens_per_tile % C != 0) {
        GFD_LOG_ERROR("WarpSpecSession: tokens_per_tile must be divisible by tokens_per_chunk\n");
        return;
    }
    if (config_.block_size() > 1024) {
        GFD_LOG_ERROR("WarpSpecSession: %d threads per block (too many chunks per tile)\n", config_.block_size());
        return;
    }
    if (config_.num_blocks > 0) {
        num_blocks_ = config_.num_blocks;
    } else {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&num_blocks_, cudaDevAttrMultiProcessorCount, dev);
    }
    if (cudaHostAlloc(reinterpret_cast<void**>(&tq_), sizeof(TiledQueue), cudaHostAllocMapped) != cudaSuccess) {
        tq_ = nullptr;
        GFD_LOG_ERROR("WarpSpecSession: cannot allocate the tiled queue\n");
        return;
    }
    memset(tq_, 0, sizeof(TiledQueue));
    tq_->scheduler.total_tiles = config_.total_tiles();
    tq_->scheduler.tokens_per_tile = config_.tokens_per_tile;
    tq_->scheduler.tokens_per_chunk = C;
    tq_->scheduler.chunks_per_tile = config_.chunks_per_tile();
    tq_->scheduler.token_size = config_.token_size;
    uint64_t* d_signal = nullptr;
    if (cudaMalloc(&d_signal, MAX_TILES * sizeof(uint64_t)) == cudaSuccess) {
        cudaMemset(d_signal, 0, MAX_TILES * sizeof(uint64_t));
        tq_->d_tile_chunk_done = d_signal;
    }
    if (cudaMalloc(&stats_, sizeof(TransferStats)) != cudaSuccess) stats_ = nullptr;
    if (stats_) cudaMemset(stats_, 0, sizeof(TransferStats));

    const size_t total = static_cast<size_t>(config_.total_tokens) * config_.token_size;
    StagingPool::instance().init(1, total);
    poller_ = new CpuPollingThread(&tq_->base, config_.gpu_dst, config_.cpu_src, total, config_.use_copy_engine,
                                   config_.numa_node);
    poller_->set_tiled_queue(tq_);
    if (!poller_->init_copy_engine()) {
        GFD_LOG_ERROR("WarpSpecSession: failed to initialise the GPU context\n");
        return;
    }
    // The framework reads cpu_src and writes gpu_dst for every token of every full tile.
    const uint64_t used = static_cast<uint64_t>(config_.total_tiles()) * config_.tokens_per_tile * config_.token_size;
    uint64_t src_span = used;
    if (config_.block_table != nullptr) {
        // page-table mode: the kernels check every id against the pool's block count on
        // each launch; the pool is the pinned allocation that starts at cpu_src
        const uint64_t ntok = static_cast<uint64_t>(config_.total_tiles()) * config_.tokens_per_tile;
        if (!range_ok(poller_->context(), config_.block_table, ntok * sizeof(uint32_t), false)) {
            GFD_LOG_ERROR("WarpSpecSession: block_table is not device memory covering %llu ids\n",
                          (unsigned long long)ntok);
            return;
        }
        const uint64_t pool = config_.src_pool_bytes ? config_.src_pool_bytes
                                                      : host_extent(poller_->context(), config_.cpu_src);
        const uint64_t blocks = pool / config_.token_size;
        if (blocks == 0) {
            GFD_LOG_ERROR("WarpSpecSession: the block pool at cpu_src holds no block of %u bytes\n",
                          config_.token_size);
            return;
        }
        tq_->scheduler.table_blocks = static_cast<uint32_t>(blocks > 0xffffffffull ? 0xffffffffull : blocks);
        src_span = blocks * config_.token_size;
    }
    if (!range_ok(poller_->context(), config_.cpu_src, src_span, true)) {
        GFD_LOG_ERROR("WarpSpecSession: cpu_src is not pinned, device-mapped host memory covering %llu bytes\n",
                      (unsigned long long)src_span);
        return;
    }
    if (!range_ok(poller_->context(), config_.gpu_dst, used, false)) {
        GFD_LOG_ERROR("WarpSpecSession: gpu_dst is not device memory covering %llu bytes\n", (unsigned long long)used);
        return;
    }
    if (config_.total_tokens % config_.tokens_per_tile != 0)
        GFD_LOG_INFO("WarpSpecSession: %u tail tokens beyond the last full tile are not transferred\n",
                     config_.total_tokens % config_.tokens_per_tile);
    ok_ = true;
}

WarpSpecSession::~WarpSpecSession() {
    if (poller_) {
        poller_->stop();
        delete poller_;
    }
    if (tq_) {
        if (tq_->d_tile_chunk_done) cudaFree(tq_->d_tile_chunk_done);
        cudaFreeHost(tq_);
    }
    if (stats_) cudaFree(stats_);
    StagingPool::instance().shutdown();
}

void WarpSpecSession::prepare_launch() {
    tq_->scheduler.producer_warps = static_cast<uint32_t>(config_.producer_warp_count());
    tq_->scheduler.compute_sets = config_.double_buffer ? 2u : 1u;
    tq_->scheduler.wait_limit_ns = limit_ns(config_.wait_timeout_ms);
    tq_->scheduler.stats = stats_;
    tq_->scheduler.block_table = config_.block_table;
    tq_->base.wait_timeouts = 0;
    std::atomic_thread_fence(std::memory_order_seq_cst);
}

WarpSpecSession::LaunchParams WarpSpecSession::get_launch_params() const {
    if (tq_) const_cast<WarpSpecSession*>(this)->prepare_launch();
    LaunchParams p;
    p.tq = tq_;
    p.gpu_buffer = config_.gpu_dst;
    p.cpu_base = config_.cpu_src;
    p.grid = dim3(num_blocks_);
    p.block = dim3(config_.block_size());
    return p;
}

void WarpSpecSession::synchronize() {
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) GFD_LOG_ERROR("WarpSpecSession::synchronize: %s\n", cudaGetErrorString(e));
    if (poller_started_) {
        poller_->stop();
        poller_started_ = false;
    }
    if (stats_) cudaMemcpy(&last_, stats_, sizeof(last_), cudaMemcpyDeviceToHost);
    if (tq_ && tq_->base.wait_timeouts)
        GFD_LOG_ERROR("WarpSpecSession: %u in-kernel wait(s) gave up after the time limit\n",
                      (unsigned)tq_->base.wait_timeouts);
    if (last_.rejected)
        GFD_LOG_ERROR("WarpSpecSession: %llu token(s) skipped: block_table id beyond the source pool\n",
                      (unsigned long long)last_.rejected);
}

void WarpSpecSession::reset() {
    if (poller_started_) {
        poller_->stop();
        poller_started_ = false;
    }
    if (!tq_) return;
    if (tq_->d_tile_chunk_done) cudaMemset(tq_->d_tile_chunk_done, 0, MAX_TILES * sizeof(uint64_t));
    memset(const_cast<uint64_t*>(tq_->tile_chunk_done), 0, sizeof(tq_->tile_chunk_done));
    tq_->scheduler.next_tile = 0;
    if (stats_) cudaMemset(stats_, 0, sizeof(TransferStats));
    last_ = TransferStats{};
    if (poller_) poller_->reset_stats();
}

uint64_t WarpSpecSession::timeouts() const {
    return last_.timeouts + (tq_ ? tq_->base.wait_timeouts : 0);
}

WarpSpecSession::Stats WarpSpecSession::get_stats() const {
    const double ms = std::chrono::duration<double, std::milli>(std::chrono::high_resolution_clock::now() -
                                                                launch_time_).count();
    const double total = static_cast<double>(config_.total_tokens) * config_.token_size;
    Stats s;
    s.descriptors_processed = last_.tokens + (poller_ ? poller_->get_descriptors_processed() : 0);
    s.bytes_transferred = last_.bytes + (poller_ ? static_cast<uint64_t>(poller_->get_total_bytes_copied()) : 0);
    s.elapsed_ms = ms;
    s.bandwidth_gbps = ms > 0 ? total / (ms * 1e6) : 0.0;
    return s;
}

// ===========================================================================
// SGWarpSpecSession
// ===========================================================================
SGWarpSpecSession::SGWarpSpecSession(const SGWarpSpecConfig& config) : config_(config) {
    if (config_.num_blocks > 0) {
        num_blocks_ = config_.num_blocks;
    } else {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&num_blocks_, cudaDevAttrMultiProcessorCount, dev);
    }
    if (cudaHostAlloc(reinterpret_cast<void**>(&sq_), sizeof(SGTaskQueue), cudaHostAllocMapped) != cudaSuccess ||
        cudaHostAlloc(reinterpret_cast<void**>(&dq_), sizeof(DescriptorQueue), cudaHostAllocMapped) != cudaSuccess) {
        GFD_LOG_ERROR("SGWarpSpecSession: cannot allocate the task queues\n");
        return;
    }
    memset(sq_, 0, sizeof(SGTaskQueue));
    memset(dq_, 0, sizeof(DescriptorQueue));
    uint64_t* d_list_done = nullptr;
    if (cudaMalloc(&d_list_done, MAX_SG_LISTS * sizeof(uint64_t)) == cudaSuccess) {
        cudaMemset(d_list_done, 0, MAX_SG_LISTS * sizeof(uint64_t));
        sq_->d_list_done = d_list_done;
    } else {
        GFD_LOG_ERROR("SGWarpSpecSession: failed to allocate d_list_done\n");
    }
    if (cudaMalloc(&stats_, sizeof(TransferStats)) != cudaSuccess) stats_ = nullptr;
    if (stats_) cudaMemset(stats_, 0, sizeof(TransferStats));
    // consumers waiting for lists poll this device-memory mirror, not host memory
    SGPollMirror* mirror = nullptr;
    if (cudaMalloc(&mirror, sizeof(SGPollMirror)) == cudaSuccess) {
        cudaMemset(mirror, 0, sizeof(SGPollMirror));
        sq_->poll_mirror = mirror;
    } else {
        cudaGetLastError();
    }
    const size_t staging = static_cast<size_t>(MAX_SG_POOL_ENTRIES) * 4096;
    StagingPool::instance().init(1, staging);
    poller_ = new CpuPollingThread(dq_, nullptr, nullptr, staging, config_.use_copy_engine, config_.numa_node);
    poller_->set_sg_task_queue(sq_);
    if (!poller_->init_copy_engine()) {
        GFD_LOG_ERROR("SGWarpSpecSession: failed to initialise the GPU context\n");
        return;
    }
    ok_ = true;
}

SGWarpSpecSession::~SGWarpSpecSession() {
    if (poller_) {
        poller_->stop();
        delete poller_;
    }
    if (sq_) {
        if (sq_->d_list_done) cudaFree(sq_->d_list_done);
        if (sq_->poll_mirror) cudaFree(sq_->poll_mirror);
        cudaFreeHost(sq_);
    }
    if (dq_) cudaFreeHost(dq_);
    if (stats_) cudaFree(stats_);
}

uint64_t SGWarpSpecSession::submit_sg_list(const DeviceSGEntry* entries, uint32_t count, uint32_t list_id,
                                           uint32_t flags) {
    if (!ok_ || sq_ == nullptr) return UINT64_MAX;
    if (count > static_cast<uint32_t>(MAX_SG_POOL_ENTRIES) || (count > 0 && entries == nullptr)) {
        GFD_LOG_ERROR("submit_sg_list: %u entries (the pool holds %d)\n", count, MAX_SG_POOL_ENTRIES);
        return UINT64_MAX;
    }
    for (uint32_t i = 0; i < count; ++i) {
        if (!range_ok(poller_->context(), reinterpret_cast<const void*>(entries[i].src_addr), entries[i].size, true) ||
            !range_ok(poller_->context(), reinterpret_cast<const void*>(entries[i].dst_addr), entries[i].size, false)) {
            GFD_LOG_ERROR("submit_sg_list: entry %u has a source outside pinned host memory or a destination "
                          "outside device memory\n", i);
            return UINT64_MAX;
        }
    }
    // room in the pool and in the list ring (only wait while a kernel is consuming)
    const uint64_t t0 = gfdb::now_ns();
    for (;;) {
        const uint64_t alloc = sq_->entry_alloc_idx;
        const uint64_t consumed = __atomic_load_n(&sq_->entry_consumed_idx, __ATOMIC_ACQUIRE);
        const uint64_t lalloc = sq_->list_alloc_idx;
        const uint64_t lread = __atomic_load_n(&sq_->list_read_idx, __ATOMIC_ACQUIRE);
        // consumers may claim list indices before they are submitted (lread > lalloc)
        const uint64_t pending = lalloc > lread ? lalloc - lread : 0;
        const bool room = alloc + count - consumed <= static_cast<uint64_t>(MAX_SG_POOL_ENTRIES) &&
                          pending < static_cast<uint64_t>(MAX_SG_LISTS - 1) &&
                          __atomic_load_n(&sq_->lists[lalloc % MAX_SG_LISTS].sequence, __ATOMIC_ACQUIRE) == 0;
        if (room) break;
        if (!launched_ || gfdb::now_ns() - t0 > limit_ns(config_.wait_timeout_ms)) {
            GFD_LOG_ERROR("submit_sg_list: no room for %u entries (pool %llu/%d used, %llu lists pending)\n",
                          count, (unsigned long long)(alloc - consumed), MAX_SG_POOL_ENTRIES,
                          (unsigned long long)pending);
            return UINT64_MAX;
        }
        std::this_thread::sleep_for(std::chrono::microseconds(20));
    }
    const uint64_t pool_offset = sq_->entry_alloc_idx;
    sq_->entry_alloc_idx = pool_offset + count;
    for (uint32_t i = 0; i < count; ++i) sq_->entries[(pool_offset + i) % MAX_SG_POOL_ENTRIES] = entries[i];
    const uint64_t slot = sq_->list_alloc_idx;
    sq_->list_alloc_idx = slot + 1;
    SGList& l = sq_->lists[slot % MAX_SG_LISTS];
    l.pool_offset = static_cast<uint32_t>(pool_offset % MAX_SG_POOL_ENTRIES);
    l.count = count;
    l.list_id = list_id;
    l.flags = flags;
    __atomic_thread_fence(__ATOMIC_RELEASE);
    __atomic_store_n(&l.sequence, slot + 1, __ATOMIC_RELEASE);
    __atomic_thread_fence(__ATOMIC_SEQ_CST);
    return slot;
}

void SGWarpSpecSession::prepare_launch() {
    if (poller_started_) {
        poller_->stop();
        poller_started_ = false;
    }
    sq_->terminate = 0;
    sq_->lists_completed = 0;
    sq_->wait_timeouts = 0;
    sq_->timeout_site = 0;
    sq_->producer_warps = static_cast<uint32_t>(config_.producer_warp_count());
    sq_->wait_limit_ns = limit_ns(config_.wait_timeout_ms);
    sq_->stats = stats_;
    if (sq_->d_list_done) cudaMemset(sq_->d_list_done, 0, MAX_SG_LISTS * sizeof(uint64_t));
    if (sq_->poll_mirror) cudaMemset(sq_->poll_mirror, 0, sizeof(SGPollMirror));
    if (stats_) cudaMemset(stats_, 0, sizeof(TransferStats));
    last_ = TransferStats{};
    dq_->write_idx = 0;
    dq_->read_idx = 0;
    dq_->done_idx = 0;
    if (dq_->mirror) cudaMemset(dq_->mirror, 0, sizeof(QueueMirror));  // copies follow the host indices
    poller_->reset_stats();
    std::atomic_thread_fence(std::memory_order_seq_cst);
}

SGWarpSpecSession::LaunchParams SGWarpSpecSession::get_launch_params() {
    LaunchParams p{dq_, sq_, dim3(num_blocks_), dim3(config_.block_size())};
    if (ok_) {
        prepare_launch();
        launched_ = true;
    }
    return p;
}

void SGWarpSpecSession::synchronize() {
    const uint64_t limit = limit_ns(config_.wait_timeout_ms);
    const uint64_t t0 = gfdb::now_ns();
    for (;;) {
        const uint64_t expected = __atomic_load_n(&sq_->list_alloc_idx, __ATOMIC_ACQUIRE);
        if (__atomic_load_n(&sq_->lists_completed, __ATOMIC_ACQUIRE) >= expected) break;
        if (gfdb::now_ns() - t0 > limit) {
            GFD_LOG_ERROR("SGWarpSpecSession::synchronize: %llu of %llu lists completed before the time limit\n",
                          (unsigned long long)sq_->lists_completed, (unsigned long long)expected);
            break;
        }
        struct timespec ts = {0, 100000};
        nanosleep(&ts, nullptr);
    }
    __atomic_store_n(&sq_->terminate, 1u, __ATOMIC_RELEASE);
    __atomic_thread_fence(__ATOMIC_SEQ_CST);
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) GFD_LOG_ERROR("SGWarpSpecSession::synchronize: %s\n", cudaGetErrorString(e));
    launched_ = false;
    if (poller_started_) {
        poller_->stop();
        poller_started_ = false;
    }
    if (stats_) cudaMemcpy(&last_, stats_, sizeof(last_), cudaMemcpyDeviceToHost);
    if (sq_->wait_timeouts)
        GFD_LOG_ERROR("SGWarpSpecSession: %u in-kernel wait(s) gave up after the time limit\n",
                      (unsigned)sq_->wait_timeouts);
}

void SGWarpSpecSession::reset() {
    if (poller_started_) {
        poller_->stop();
        poller_started_ = false;
    }
    sq_->list_alloc_idx = 0;
    sq_->list_read_idx = 0;
    sq_->entry_alloc_idx = 0;
    sq_->entry_consumed_idx = 0;
    sq_->lists_completed = 0;
    sq_->terminate = 0;
    sq_->lists_released = 0;
    for (int i = 0; i < MAX_SG_LISTS; ++i) {
        sq_->lists[i].sequence = 0;
        sq_->lists[i].release_end = 0;
    }
    if (sq_->d_list_done) cudaMemset(sq_->d_list_done, 0, MAX_SG_LISTS * sizeof(uint64_t));
    dq_->write_idx = 0;
    dq_->read_idx = 0;
    dq_->done_idx = 0;
    if (dq_->mirror) cudaMemset(dq_->mirror, 0, sizeof(QueueMirror));  // copies follow the host indices
    if (stats_) cudaMemset(stats_, 0, sizeof(TransferStats));
    last_ = TransferStats{};
    poller_->reset_stats();
}

uint64_t SGWarpSpecSession::timeouts() const { return last_.timeouts + (sq_ ? sq_->wait_timeouts : 0); }

SGWarpSpecSession::Stats SGWarpSpecSession::get_stats() const {
    const double ms = std::chrono::duration<double, std::milli>(std::chrono::high_resolution_clock::now() -
                                                                launch_time_).count();
    Stats s;
    s.descriptors_processed = last_.tokens + (poller_ ? poller_->get_descriptors_processed() : 0);
    s.bytes_transferred = last_.bytes + (poller_ ? static_cast<uint64_t>(poller_->get_total_bytes_copied()) : 0);
    s.elapsed_ms = ms;
    s.bandwidth_gbps = (s.bytes_transferred > 0 && ms > 0) ? s.bytes_transferred / (ms * 1e6) : 0.0;
    return s;
}

}  // namespace gfd
