// GPU-queued submit: consumer of the descriptor ring written by GPU producers.
//
// Reference behaviour being replaced (src/cpu_polling.cpp:337-436,
// src/batch_processor.cpp:69-446): a pinned CPU thread spins on the commit markers,
// copies descriptors out, gathers the payload on CPU cores into staging buffers,
// DMAs it with the copy engine and publishes done_idx / per-tile counters / per-list
// completion.
//
// Here a light doorbell (a host thread, or gfd_ring_poll from any thread) only
// watches the commit markers.  For every committed run of slots [s, s+n) it
// launches three stream-ordered kernels on the ring's own stream:
//   plan_kernel     (kind 1: reads the 64-byte descriptors straight from the ring,
//                    validates them against the ranges the doorbell checked, merges
//                    contiguous runs with a warp ballot + block prefix scan),
//   pull_kernel     (moves the bytes host -> HBM, same kernel as direct submit),
//   finalize_kernel (clears the markers, adds per-tile token counts, raises
//                    d_list_done / lists_completed for lists whose last descriptor
//                    landed, then advances read_idx and done_idx).
// None of these kernels waits on anything: each drain starts only after its slots
// are committed, so no two launches ever wait on one another.  Producer kernels that
// spin on done_idx / tile counters / list flags must leave SM room for the drains
// (the device API bounds those spins; see device.cuh).

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
#include "internal.h"

namespace gfdb {

constexpr uint32_t kDrainMax = 8192;  // slots per drain (the reference's MAX_BATCH_SIZE)
constexpr uint32_t kUrgentFlags = gfd::FLAG_LAST_IN_BATCH | gfd::FLAG_URGENT |
                                  gfd::FLAG_LAST_IN_TILE | gfd::FLAG_LAST_CHUNK_IN_TILE;

struct FinalizeArgs {
    gfd::DescriptorQueue* q;
    gfd::TiledQueue* tq;   // per-tile accounting when non-null
    gfd::SGTaskQueue* sq;  // per-list accounting when non-null
    uint64_t begin;
    uint32_t n;
    const PlanHeader* hdr;
    unsigned long long* rejected;  // device counter of entries the plan refused
    const uint32_t* flags;         // descriptor flags / user_data, copied out of the ring
    const uint64_t* user;          // by the plan kernel (device memory)
    gfd::QueueMirror* mirror;      // device-memory copy of read_idx / done_idx (written last)
};

__global__ void __launch_bounds__(256) finalize_kernel(FinalizeArgs a) {
    __shared__ uint32_t tile_count[gfd::MAX_TILES];
    __shared__ uint32_t lists_done;
    for (int i = threadIdx.x; i < gfd::MAX_TILES; i += blockDim.x) tile_count[i] = 0;
    if (threadIdx.x == 0) lists_done = 0;
    __syncthreads();
    for (uint32_t i = threadIdx.x; i < a.n; i += blockDim.x) {
        gfd::Descriptor* d = &a.q->entries[(a.begin + i) % gfd::QUEUE_SIZE];
        const uint64_t user = a.user[i];
        const uint32_t flags = a.flags[i];
        const uint32_t id = static_cast<uint32_t>(user >> 32);
        if (a.tq != nullptr && id < static_cast<uint32_t>(gfd::MAX_TILES)) atomicAdd(&tile_count[id], 1u);
        if (a.sq != nullptr && (flags & gfd::FLAG_LAST_IN_TILE) && id < static_cast<uint32_t>(gfd::MAX_SG_LISTS)) {
            uint64_t* done = a.sq->d_list_done;
            if (done != nullptr) *reinterpret_cast<volatile uint64_t*>(&done[id]) = 1;
            atomicAdd(&lists_done, 1u);
        }
        d->sequence = 0;  // slot free for producers
    }
    __syncthreads();
    if (a.tq != nullptr) {
        uint64_t* dev = a.tq->d_tile_chunk_done;
        for (int t = threadIdx.x; t < gfd::MAX_TILES; t += blockDim.x) {
            const uint32_t c = tile_count[t];
            if (c == 0) continue;
            if (dev != nullptr) {
                volatile uint64_t* p = &dev[t];
                *p = *p + c;
            } else {
                volatile uint64_t* p = &a.tq->tile_chunk_done[t];
                *p = *p + c;
            }
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        if (a.rejected != nullptr && a.hdr->status != GFD_OK) atomicAdd(a.rejected, 1ull);
        __threadfence_system();
        if (a.sq != nullptr && lists_done != 0) {
            volatile uint64_t* lc = &a.sq->lists_completed;
            *lc = *lc + lists_done;
        }
        const uint64_t end = a.begin + a.n;
        a.q->read_idx = end;
        __threadfence_system();
        if (a.q->done_idx < end) a.q->done_idx = end;
        __threadfence_system();
        if (a.mirror != nullptr) {  // after the host fields: the mirror never runs ahead
            a.mirror->read_idx = end;
            if (a.mirror->done_idx < end) a.mirror->done_idx = end;
            __threadfence();
        }
    }
}

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

    gfdb::PullRow* d_rows = nullptr;
    gfdb::PullRow* d_misc = nullptr;
    uint32_t* d_cta_first = nullptr;
    gfdb::PlanHeader* d_hdr = nullptr;
    unsigned long long* d_counters = nullptr;  // [0] bytes, [1] rejected drains
    uint32_t* d_flags = nullptr;               // per drained slot: descriptor flags
    uint64_t* d_user = nullptr;                // per drained slot: descriptor user_data
    gfdb::TileTotals* d_tiles = nullptr;       // multi-CTA plan scratch
    gfd::QueueMirror* d_mirror = nullptr;      // device copy of read_idx / done_idx

    std::mutex mu;
    std::thread thread;
    std::atomic<bool> running{false};
    std::atomic<uint64_t> consumed{0}, drains{0}, host_rejected{0};
    uint32_t pending_n = 0;
    uint64_t pending_since = 0;
};

namespace {

using namespace gfdb;

// One doorbell pass; the caller holds ring->mu.  force: launch whatever is committed.
int poll_locked(gfd_ring* r, bool force, int* launched) {
    *launched = 0;
    for (;;) {
        const uint64_t s = r->next;
        uint32_t n = 0;
        bool urgent = false;
        while (n < kDrainMax) {
            gfd::Descriptor* d = &r->q->entries[(s + n) % gfd::QUEUE_SIZE];
            const uint64_t seq = __atomic_load_n(&d->sequence, __ATOMIC_ACQUIRE);
            if (seq != s + n + 1) break;
            if (d->flags & kUrgentFlags) urgent = true;
            ++n;
        }
        if (n == 0) {
            r->pending_n = 0;
            return GFD_OK;
        }
        // Batch like the reference poller: go when a batch boundary is flagged, when
        // the run is large, or when the producers have stopped extending it.
        if (!force && !urgent && n < static_cast<uint32_t>(gfd::BATCH_THRESHOLD_SMALL)) {
            const uint64_t now = now_ns();
            if (n != r->pending_n) {
                r->pending_n = n;
                r->pending_since = now;
                return GFD_OK;
            }
            if (now - r->pending_since < 20000) return GFD_OK;
        }
        r->pending_n = 0;

        // Host-side validation of every descriptor; collect the ranges they use.
        RangeTable src_t, dst_t;
        memset(&src_t, 0, sizeof(src_t));
        memset(&dst_t, 0, sizeof(dst_t));
        uint32_t bad = 0;
        {
            std::lock_guard<std::mutex> lk(r->ctx->mu);
            auto add = [](RangeTable& t, const Range* x) {
                if (x == nullptr) return;
                for (uint32_t k = 0; k < t.n; ++k)
                    if (t.lo[k] == x->lo) return;
                if (t.n < kMaxCheckRanges) {
                    t.lo[t.n] = x->lo;
                    t.hi[t.n] = x->hi;
                    t.n++;
                }
            };
            // most descriptors of a run share one pool and one destination buffer: test
            // the ranges of the previous descriptor before searching the registry
            uint64_t slo = 1, shi = 1, dlo = 1, dhi = 1;
            for (uint32_t i = 0; i < n; ++i) {
                const gfd::Descriptor* d = &r->q->entries[(s + i) % gfd::QUEUE_SIZE];
                const uint64_t src = d->src_addr, dst = d->dst_addr, size = d->size;
                if (size == 0) continue;
                const bool src_hit = src >= slo && size <= shi - slo && src - slo <= shi - slo - size;
                const bool dst_hit = dst >= dlo && size <= dhi - dlo && dst - dlo <= dhi - dlo - size;
                if (src_hit && dst_hit) continue;
                if (!check_host(r->ctx, src, size) || !check_dev(r->ctx, dst, size)) {
                    ++bad;
                    continue;
                }
                const Range* hs = r->ctx->host_ranges.find(src, size);
                const Range* ds = r->ctx->dev_ranges.find(dst, size);
                add(src_t, hs);
                add(dst_t, ds);
                if (hs) {
                    slo = hs->lo;
                    shi = hs->hi;
                }
                if (ds) {
                    dlo = ds->lo;
                    dhi = ds->hi;
                }
            }
            if (bad) {
                set_error(r->ctx, GFD_ERR_INVALID,
                          "ring: %u descriptor(s) in slots [%llu, %llu) rejected (source not in pinned "
                          "host memory or destination not in device memory)",
                          bad, (unsigned long long)s, (unsigned long long)(s + n));
                r->host_rejected += bad;
            }
        }

        const int grid = std::min(2 * r->ctx->num_sms, kMaxPullGrid);
        PlanArgs p;
        memset(&p, 0, sizeof(p));
        p.entries = r->q->entries;
        p.n = n;
        p.stride = sizeof(gfd::Descriptor);
        p.kind = 1;
        p.ring_begin = s;
        p.ring_size = gfd::QUEUE_SIZE;
        p.src_ok = src_t;
        p.dst_ok = dst_t;
        p.rows = r->d_rows;
        p.misc = r->d_misc;
        p.cta_first = r->d_cta_first;
        p.grid = static_cast<uint32_t>(grid);
        p.hdr = r->d_hdr;
        p.meta_flags = r->d_flags;
        p.meta_user = r->d_user;
        p.tiles = r->d_tiles;
        cudaError_t e = launch_plan(p, r->stream);
        PullArgs a;
        memset(&a, 0, sizeof(a));
        a.rows = r->d_rows;
        a.misc = r->d_misc;
        a.cta_first = r->d_cta_first;
        a.hdr = r->d_hdr;
        a.bytes_ctr = r->d_counters;
        if (e == cudaSuccess) e = launch_pull(a, grid, r->stream);
        FinalizeArgs f{r->q, r->tq, r->sq, s, n, r->d_hdr, r->d_counters + 1, r->d_flags, r->d_user, r->d_mirror};
        if (e == cudaSuccess) {
            finalize_kernel<<<1, 256, 0, r->stream>>>(f);
            e = cudaGetLastError();
        }
        if (e != cudaSuccess) return cuda_error(r->ctx, e, "ring drain launch");
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
    if (e == cudaSuccess) e = cudaMalloc(&r->d_rows, kDrainMax * sizeof(PullRow));
    if (e == cudaSuccess) e = cudaMalloc(&r->d_misc, kDrainMax * sizeof(PullRow));
    if (e == cudaSuccess) e = cudaMalloc(&r->d_cta_first, kMaxPullGrid * sizeof(uint32_t));
    if (e == cudaSuccess) e = cudaMalloc(&r->d_hdr, sizeof(PlanHeader));
    if (e == cudaSuccess) e = cudaMalloc(&r->d_counters, 2 * sizeof(unsigned long long));
    if (e == cudaSuccess) e = cudaMalloc(&r->d_flags, kDrainMax * sizeof(uint32_t));
    if (e == cudaSuccess) e = cudaMalloc(&r->d_user, kDrainMax * sizeof(uint64_t));
    if (e == cudaSuccess) e = cudaMalloc(&r->d_tiles, plan_tile_slots(kDrainMax) * sizeof(TileTotals));
    // The mirror is published in the queue only while the ring runs (start .. stop) and
    // is never freed: a kernel that is still waiting when the ring goes away keeps
    // reading valid device memory until its bounded wait gives up.
    if (e == cudaSuccess) e = cudaMalloc(&r->d_mirror, sizeof(gfd::QueueMirror));
    if (e == cudaSuccess) e = cudaMemsetAsync(r->d_counters, 0, 2 * sizeof(unsigned long long), r->stream);
    // only this ring's stream: the caller may have kernels running that wait on the ring
    if (e == cudaSuccess) e = cudaStreamSynchronize(r->stream);
    // load the drain kernels now, not at the first drain (lazy loading would queue that
    // launch behind a producer kernel that is waiting for it)
    cudaFuncAttributes fa;
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, finalize_kernel);
    if (e == cudaSuccess) e = preload_gather_kernels();
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
    cudaFree(r->d_rows);
    cudaFree(r->d_misc);
    cudaFree(r->d_cta_first);
    cudaFree(r->d_hdr);
    cudaFree(r->d_counters);
    cudaFree(r->d_flags);
    cudaFree(r->d_user);
    cudaFree(r->d_tiles);  // d_mirror is kept (see gfd_ring_create)
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
        r->pending_n = 0;
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
