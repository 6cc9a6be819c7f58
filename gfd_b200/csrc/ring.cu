// GPU-queued submit: consumer of the descriptor ring written by GPU producers.
//
// Reference behaviour being replaced (src/cpu_polling.cpp:337-436,
// src/batch_processor.cpp:69-446): a pinned CPU thread spins on the commit markers,
// copies descriptors out, gathers the payload on CPU cores into staging buffers,
// DMAs it with the copy engine and publishes done_idx / per-tile counters / per-list
// completion.
//
// Here a light doorbell (a host thread, or gfd_ring_poll from any thread) watches the
// commit markers.  For every committed run of slots [s, s+n) it copies the descriptors
// out (the ring sits in host memory, so this costs the host a few ns per slot), frees
// the slots (markers back to 0), validates the entries, counts per-tile tokens and
// landed lists, and issues ONE pull kernel on the ring's own stream through the same
// staging path as direct submit; the pull's last CTA applies the tile / list counts and
// advances read_idx and done_idx (RingEpilogue).  No drain kernel waits on anything:
// each starts only after its slots are committed, so no two launches ever wait on one
// another.  Producer kernels that spin on done_idx / tile counters / list flags must
// leave SM room for the drains (the device API bounds those spins; see device.cuh).

#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cstdio>
#include <thread>
#include <vector>

#if defined(__x86_64__)
#include <immintrin.h>
#endif

#include "gfd/descriptor_queue.h"
#include "gfd/sg_task_queue.h"
#include "gfd/tiled_queue.h"
#include "drain.h"
#include "internal.h"

namespace gfdb {

constexpr uint32_t kDrainMax = 8192;  // slots per drain (the reference's MAX_BATCH_SIZE)

static inline void cpu_relax() {
#if defined(__x86_64__)
    _mm_pause();
#endif
}

}  // namespace gfdb

struct gfd_ring {
    gfd_ctx* ctx = nullptr;
    gfd::DescriptorQueue* q = nullptr;
    gfd::TiledQueue* tq = nullptr;
    gfd::SGTaskQueue* sq = nullptr;
    cudaStream_t stream = nullptr;
    uint64_t next = 0;  // first slot not yet handed to a drain

    unsigned long long* d_counters = nullptr;  // [0] bytes moved
    gfd::QueueMirror* d_mirror = nullptr;      // device copy of read_idx / done_idx

    // drain scratch (doorbell side, under mu)
    std::vector<gfd_sg_entry> ents;
    gfdb::RingDrain drain;
    gfdb::RingTables tables;
    uint32_t tile_tokens[gfd::MAX_TILES] = {};

    std::mutex mu;
    std::thread thread;
    std::atomic<bool> running{false};
    std::atomic<uint64_t> consumed{0}, drains{0}, host_rejected{0};
    gfdb::BatchGate gate;
};

namespace {

using namespace gfdb;

// One doorbell pass; the caller holds ring->mu.  force: launch whatever is committed.
int poll_locked(gfd_ring* r, bool force, int* launched) {
    *launched = 0;
    for (;;) {
        const uint64_t s = r->next;
        bool urgent = false;
        const uint32_t n = committed_run(r->q, s, kDrainMax, &urgent);
        // batch like the reference poller: go when a batch boundary is flagged, when the
        // run is large, or when the producers have stopped extending it
        if (!r->gate.ready(n, urgent, force, now_ns())) return GFD_OK;

        // Copy the drain out of the ring: validated entries for the pull, per-tile token
        // counts and landed lists for the completion; then the slots are free again.
        RingDrain& drain = r->drain;
        RingTables& tab = r->tables;
        drain.read_idx = &r->q->read_idx;
        drain.done_idx = &r->q->done_idx;
        drain.mirror_read = r->d_mirror != nullptr ? &r->d_mirror->read_idx : nullptr;
        drain.mirror_done = r->d_mirror != nullptr ? &r->d_mirror->done_idx : nullptr;
        drain.tile_done = nullptr;
        if (r->tq != nullptr)
            drain.tile_done = r->tq->d_tile_chunk_done != nullptr ? r->tq->d_tile_chunk_done
                                                                : const_cast<uint64_t*>(r->tq->tile_chunk_done);
        drain.list_done = r->sq != nullptr ? r->sq->d_list_done : nullptr;
        drain.lists_completed = r->sq != nullptr ? &r->sq->lists_completed : nullptr;
        drain.tables = nullptr;
        drain.end = s + n;
        DrainAccounting acct(r->tq != nullptr, r->sq != nullptr, r->tile_tokens, tab.tile_id, tab.tile_count,
                             tab.list_id, static_cast<uint32_t>(kEpiLists));
        r->ents.clear();
        uint32_t bad = 0;
        int rc;
        {
            std::lock_guard<std::mutex> lk(r->ctx->mu);
            // most descriptors of a run share one pool and one destination buffer: test
            // the ranges of the previous descriptor before searching the registry
            uint64_t slo = 1, shi = 1, dlo = 1, dhi = 1;
            for (uint32_t i = 0; i < n; ++i) {
                gfd::Descriptor* d = &r->q->entries[(s + i) % gfd::QUEUE_SIZE];
                const uint64_t src = d->src_addr, dst = d->dst_addr, size = d->size;
                acct.add(d->flags, d->user_data);
                __atomic_store_n(&d->sequence, 0ull, __ATOMIC_RELEASE);  // slot free for producers
                if (size == 0) continue;
                const bool src_hit = src >= slo && size <= shi - slo && src - slo <= shi - slo - size;
                const bool dst_hit = dst >= dlo && size <= dhi - dlo && dst - dlo <= dhi - dlo - size;
                if (!(src_hit && dst_hit)) {
                    if (!check_host(r->ctx, src, size) || !check_dev(r->ctx, dst, size)) {
                        ++bad;
                        continue;
                    }
                    if (const Range* hs = r->ctx->host_ranges.find(src, size)) {
                        slo = hs->lo;
                        shi = hs->hi;
                    }
                    if (const Range* ds = r->ctx->dev_ranges.find(dst, size)) {
                        dlo = ds->lo;
                        dhi = ds->hi;
                    }
                }
                r->ents.push_back(gfd_sg_entry{dst, reinterpret_cast<const void*>(src), size});
            }
            acct.finish();
            drain.n_tiles = acct.n_tiles();
            drain.n_lists = acct.n_lists();
            drain.lists_landed = acct.lists_landed();
            std::atomic_thread_fence(std::memory_order_seq_cst);  // markers out before the launch
            if (bad) {
                set_error(r->ctx, GFD_ERR_INVALID,
                          "ring: %u descriptor(s) in slots [%llu, %llu) rejected (source not in pinned "
                          "host memory or destination not in device memory)",
                          bad, (unsigned long long)s, (unsigned long long)(s + n));
                r->host_rejected += bad;
            }
            rc = gather_drain(r->ctx, r->ents.data(), static_cast<int64_t>(r->ents.size()), r->stream, drain, tab,
                              r->d_counters);
        }
        // A failed launch leaves next (and so done_idx) behind these slots for good: waiters
        // time out with the error in gfd_last_error rather than see done_idx cover bytes
        // that never landed.
        if (rc != GFD_OK) return rc;
        r->next = s + n;
        r->consumed += n;
        r->drains++;
        ++*launched;
    }
}

void doorbell_loop(gfd_ring* r) {
    driver().ctx_set_current(r->ctx->cu_ctx);  // the context the ring's stream lives in
    uint32_t idle = 0;
    while (r->running.load(std::memory_order_acquire)) {
        int launched = 0;
        {
            std::lock_guard<std::mutex> lk(r->mu);
            poll_locked(r, false, &launched);
        }
        if (launched) {
            idle = 0;
            continue;
        }
        ++idle;
        if (idle < 20000) {
            cpu_relax();
        } else {
            // producers idle for a while: back off to 50 us naps
            std::this_thread::sleep_for(std::chrono::microseconds(50));
        }
    }
}

}  // namespace

extern "C" {

int gfd_ring_create(gfd_ctx* ctx, void* queue, void* tiled, void* sg, gfd_ring** out) {
    if (!ctx || !queue || !out) return GFD_ERR_INVALID;
    *out = nullptr;
    auto* tq = static_cast<gfd::TiledQueue*>(tiled);
    if (tq != nullptr && static_cast<void*>(&tq->base) != queue)
        return set_error(ctx, GFD_ERR_INVALID, "ring: tiled queue's base is not the given queue");
    CtxScope scope(ctx->cu_ctx);
    gfd_ring* r = new gfd_ring();
    r->ctx = ctx;
    r->q = static_cast<gfd::DescriptorQueue*>(queue);
    r->tq = tq;
    r->sq = static_cast<gfd::SGTaskQueue*>(sg);
    r->next = __atomic_load_n(&r->q->read_idx, __ATOMIC_ACQUIRE);
    int lo = 0, hi = 0;
    cudaDeviceGetStreamPriorityRange(&lo, &hi);
    cudaError_t e = cudaStreamCreateWithPriority(&r->stream, cudaStreamNonBlocking, hi);
    if (e == cudaSuccess) e = cudaMalloc(&r->d_counters, sizeof(unsigned long long));
    // The mirror is published in the queue only while the ring runs (start .. stop) and
    // is never freed: a kernel that is still waiting when the ring goes away keeps
    // reading valid device memory until its bounded wait gives up.
    if (e == cudaSuccess) e = cudaMalloc(&r->d_mirror, sizeof(gfd::QueueMirror));
    if (e == cudaSuccess) e = cudaMemsetAsync(r->d_counters, 0, sizeof(unsigned long long), r->stream);
    // only this ring's stream: the caller may have kernels running that wait on the ring
    if (e == cudaSuccess) e = cudaStreamSynchronize(r->stream);
    // load the drain kernels now, not at the first drain (lazy loading would queue that
    // launch behind a producer kernel that is waiting for it)
    if (e == cudaSuccess) e = preload_gather_kernels();
    if (e == cudaSuccess) {
        std::lock_guard<std::mutex> lk(ctx->mu);
        if (reserve_drain_slots(ctx, kDrainMax) != GFD_OK) e = cudaErrorMemoryAllocation;
    }
    // A managed-memory ring stays resident in host memory and is mapped by the GPU,
    // so the doorbell's reads do not migrate pages back and forth.
    cudaPointerAttributes pa;
    if (e == cudaSuccess && cudaPointerGetAttributes(&pa, queue) == cudaSuccess && pa.type == cudaMemoryTypeManaged) {
        cudaMemAdvise(queue, sizeof(gfd::DescriptorQueue), cudaMemAdviseSetPreferredLocation, cudaCpuDeviceId);
        cudaMemAdvise(queue, sizeof(gfd::DescriptorQueue), cudaMemAdviseSetAccessedBy, ctx->device);
    }
    cudaGetLastError();
    if (e != cudaSuccess) {
        gfd_ring_destroy(r);
        return cuda_error(ctx, e, "ring create");
    }
    *out = r;
    return GFD_OK;
}

int gfd_ring_destroy(gfd_ring* r) {
    if (!r) return GFD_OK;
    gfd_ring_stop(r);
    CtxScope scope(r->ctx->cu_ctx);
    if (r->stream) {
        cudaStreamSynchronize(r->stream);
        cudaStreamDestroy(r->stream);
    }
    cudaFree(r->d_counters);  // d_mirror is kept (see gfd_ring_create)
    cudaGetLastError();
    delete r;
    return GFD_OK;
}

int gfd_ring_start(gfd_ring* r) {
    if (!r) return GFD_ERR_INVALID;
    CtxScope scope(r->ctx->cu_ctx);
    if (r->running.exchange(true)) return GFD_OK;
    {
        std::lock_guard<std::mutex> lk(r->mu);
        // slots consumed while stopped (or reset by the owner) restart from read_idx
        cudaStreamSynchronize(r->stream);
        const uint64_t ri = __atomic_load_n(&r->q->read_idx, __ATOMIC_ACQUIRE);
        r->next = ri;
        r->gate.reset();
        // device-side waits poll the mirror while the ring runs
        const gfd::QueueMirror init{ri, __atomic_load_n(&r->q->done_idx, __ATOMIC_ACQUIRE)};
        if (r->d_mirror != nullptr &&
            cudaMemcpyAsync(r->d_mirror, &init, sizeof(init), cudaMemcpyHostToDevice, r->stream) == cudaSuccess &&
            cudaStreamSynchronize(r->stream) == cudaSuccess) {
            r->q->mirror = r->d_mirror;
            std::atomic_thread_fence(std::memory_order_seq_cst);
        }
        cudaGetLastError();
    }
    r->thread = std::thread(doorbell_loop, r);
    return GFD_OK;
}

int gfd_ring_stop(gfd_ring* r) {
    if (!r) return GFD_ERR_INVALID;
    CtxScope scope(r->ctx->cu_ctx);
    int rc = GFD_OK;
    if (r->running.exchange(false)) {
        if (r->thread.joinable()) r->thread.join();
        // drain every slot committed before the stop (the queue is still owned by the
        // caller here; after a stop the ring never touches it again)
        int launched = 0;
        std::lock_guard<std::mutex> lk(r->mu);
        rc = poll_locked(r, true, &launched);
        cudaError_t e = cudaStreamSynchronize(r->stream);
        // waits started from now on poll the host fields again
        if (r->q->mirror == r->d_mirror) r->q->mirror = nullptr;
        std::atomic_thread_fence(std::memory_order_seq_cst);
        if (e != cudaSuccess) return cuda_error(r->ctx, e, "ring stop");
        return rc;
    }
    cudaError_t e = cudaStreamSynchronize(r->stream);
    if (e != cudaSuccess) return cuda_error(r->ctx, e, "ring stop");
    return rc;
}

int gfd_ring_poll(gfd_ring* r, int* launched) {
    if (!r) return GFD_ERR_INVALID;
    int l = 0;
    CtxScope scope(r->ctx->cu_ctx);
    std::lock_guard<std::mutex> lk(r->mu);
    int rc = poll_locked(r, true, &l);
    if (launched) *launched = l;
    return rc;
}

int gfd_ring_wait(gfd_ring* r, uint64_t target) {
    if (!r) return GFD_ERR_INVALID;
    CtxScope scope(r->ctx->cu_ctx);
    const uint64_t t0 = now_ns();
    while (__atomic_load_n(&r->q->done_idx, __ATOMIC_ACQUIRE) < target) {
        if (now_ns() - t0 > r->ctx->timeout_ns)
            return set_error(r->ctx, GFD_ERR_TIMEOUT, "ring: done_idx %llu did not reach %llu in time",
                             (unsigned long long)r->q->done_idx, (unsigned long long)target);
        if (!r->running.load()) {
            int l = 0;
            std::lock_guard<std::mutex> lk(r->mu);
            int rc = poll_locked(r, true, &l);
            if (rc != GFD_OK) return rc;
        }
        cudaError_t q = cudaStreamQuery(r->stream);
        if (q != cudaSuccess && q != cudaErrorNotReady) return cuda_error(r->ctx, q, "ring drain");
        std::this_thread::sleep_for(std::chrono::microseconds(5));
    }
    return GFD_OK;
}

int gfd_ring_counters(const gfd_ring* r, uint64_t* consumed, uint64_t* drains, uint64_t* bytes) {
    if (!r) return GFD_ERR_INVALID;
    if (consumed) *consumed = r->consumed.load();
    if (drains) *drains = r->drains.load();
    if (bytes) {
        unsigned long long b = 0;
        CtxScope scope(r->ctx->cu_ctx);
        cudaStreamSynchronize(r->stream);
        cudaError_t e = cudaMemcpy(&b, r->d_counters, sizeof(b), cudaMemcpyDeviceToHost);
        if (e != cudaSuccess) return GFD_ERR_CUDA;
        *bytes = b;
    }
    return GFD_OK;
}

}  // extern "C"
