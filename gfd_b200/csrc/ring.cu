// GPU-queued submit: consumer of the descriptor ring written by GPU producers.
//
// Reference behaviour being replaced (src/cpu_polling.cpp:337-436,
// src/batch_processor.cpp:69-446): a pinned CPU thread spins on the commit markers,
// copies descriptors out, gathers the payload on CPU cores into staging buffers,
// DMAs it with the copy engine and publishes done_idx / per-tile counters / per-list
// completion.
//
// Here, between gfd_ring_start and gfd_ring_stop, a device-resident kernel -- the ring
// agent (agent.cu) -- does all of that on the GPU: it polls the markers, copies the
// descriptors out, clears the markers, validates, merges runs, pulls the bytes and
// publishes read_idx, done_idx, tile counts and landed lists.  No host core reads a
// descriptor or a payload byte.  The host side is a service thread that only
//   * launches the agent (gfd_ring_start waits until all its CTAs run, so kernels the
//     application launches afterwards find it resident);
//   * answers the agent's range queries: a source or destination range the agent has
//     not seen is checked once against the driver's allocation records (pinned host
//     memory, device memory of this GPU) and the answer is cached on the device;
//   * relaunches the agent when it has exited after `linger_ns` with nothing committed
//     (it exits so that cudaDeviceSynchronize / cudaFree in the application, which wait
//     for every kernel of the context, return) and a new marker is committed.  While the
//     agent runs, this thread sleeps between mailbox checks; while it is parked it reads
//     one marker word.  In resident mode (gfd_ring_configure) the agent stays until
//     gfd_ring_stop, for producers that occupy every SM and synchronise with streams.
// Without gfd_ring_start, gfd_ring_poll drains what is committed from the calling thread
// instead: it copies each committed run out, validates it on the host and issues ONE pull
// kernel whose last CTA applies the completion (RingEpilogue).

#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cstdio>
#include <thread>
#include <vector>

#if defined(__x86_64__)
#include <immintrin.h>
#include <sys/prctl.h>
#endif

#include "gfd/descriptor_queue.h"
#include "gfd/sg_task_queue.h"
#include "gfd/tiled_queue.h"
#include "agent.h"
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
    uint64_t next = 0;  // first slot not yet consumed (host drains) / where the agent resumes

    unsigned long long* d_counters = nullptr;  // [0] bytes moved
    gfd::QueueMirror* d_mirror = nullptr;      // device copy of read_idx / done_idx

    // host drains (gfd_ring_poll without gfd_ring_start), under mu
    std::vector<gfd_sg_entry> ents;
    gfdb::RingDrain drain;
    gfdb::RingTables tables;
    uint32_t tile_tokens[gfd::MAX_TILES] = {};
    gfdb::BatchGate gate;

    // ring agent
    gfdb::AgentDev* d_agent = nullptr;        // device memory
    gfdb::AgentHost* h_agent = nullptr;       // pinned, device-mapped
    gfdb::AgentRanges* h_tables = nullptr;    // pinned staging of the [src, dst] tables for a launch
    cudaEvent_t agent_end = nullptr;          // recorded after each launch
    uint32_t movers = gfdb::kAgentDefaultMovers;
    uint64_t linger_ns = 20000;
    bool resident = false;
    uint32_t launches = 0;
    bool agent_live = false;                  // a launch is in flight (service thread)
    bool tables_current = false;              // d_agent's tables equal h_tables (tables_sum)
    uint64_t tables_sum = 0;
    struct Window {
        int kind;  // 0 pinned host source, 1 device destination
        uint64_t lo, hi;
    };
    std::vector<Window> windows;              // declared (gfd_ring_allow) and learnt ranges, under mu
    std::atomic<bool> stopping{false};
    std::atomic<uint64_t> agent_launches{0}, agent_queries{0};
    // host-side fault injection for the timeout tests (GFD_RING_TEST_DROP_QUERIES=1 at
    // create): the service thread never answers the agent's range queries, so the
    // agent's bounded mailbox wait runs out and the descriptor is rejected
    bool drop_queries = false;

    std::mutex mu;
    std::thread thread;
    std::atomic<bool> running{false};
    std::atomic<uint64_t> consumed{0}, drains{0}, host_rejected{0};
};

namespace {

using namespace gfdb;

// One host-driven drain pass (gfd_ring_poll); the caller holds ring->mu.  force: launch whatever is committed.
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

// Allocation of the given kind holding [p, p + n): 0 pinned host memory mapped at the same
// address, 1 device memory of the ring's GPU (or managed memory).  The caller holds ctx->mu.
bool allocation_of(gfd_ctx* ctx, int kind, uint64_t p, uint64_t n, uint64_t* lo, uint64_t* hi) {
    if (n == 0 || p + n < p) return false;
    if (kind == 0 ? !check_host(ctx, p, n) : !check_dev(ctx, p, n)) return false;
    const Range* r = (kind == 0 ? ctx->host_ranges : ctx->dev_ranges).find(p, n);
    if (r == nullptr) return false;
    *lo = r->lo;
    *hi = r->hi;
    return true;
}

void remember(gfd_ring* r, int kind, uint64_t lo, uint64_t hi) {
    for (const auto& w : r->windows)
        if (w.kind == kind && w.lo == lo && w.hi == hi) return;
    r->windows.push_back(gfd_ring::Window{kind, lo, hi});
}

// Answers a pending range query of the agent, if any.
bool answer_query(gfd_ring* r) {
    AgentHost* h = r->h_agent;
    const uint32_t q = h->q_seq;
    if (q == h->a_seq || r->drop_queries) return false;
    std::atomic_thread_fence(std::memory_order_acquire);
    const int kind = static_cast<int>(h->q_kind);
    const uint64_t addr = h->q_addr, size = h->q_size;
    uint64_t lo = 0, hi = 0;
    bool ok;
    {
        std::lock_guard<std::mutex> lk(r->ctx->mu);
        ok = allocation_of(r->ctx, kind, addr, size, &lo, &hi);
    }
    if (ok) {
        std::lock_guard<std::mutex> lk(r->mu);
        remember(r, kind, lo, hi);
    }
    h->a_ok = ok ? 1u : 0u;
    h->a_lo = lo;
    h->a_hi = hi;
    std::atomic_thread_fence(std::memory_order_seq_cst);
    h->a_seq = q;
    std::atomic_thread_fence(std::memory_order_seq_cst);
    r->agent_queries++;
    return true;
}

// Launches the agent at r->next.  Range tables: pools this library pinned, plus every
// declared or learnt window the driver still confirms (a window whose memory was freed
// is dropped, so the agent never trusts a stale range).  The caller holds r->mu.
int launch_agent_locked(gfd_ring* r) {
    AgentRanges* src = &r->h_tables[0];
    AgentRanges* dst = &r->h_tables[1];
    src->n = dst->n = 0;
    src->evict = dst->evict = 0;
    auto add = [](AgentRanges* t, uint64_t lo, uint64_t hi) {
        if (t->n < static_cast<uint32_t>(kAgentRanges)) {
            t->lo[t->n] = lo;
            t->hi[t->n] = hi;
            ++t->n;
        }
    };
    {
        std::lock_guard<std::mutex> lk(r->ctx->mu);
        for (const Range& h : r->ctx->host_ranges.snapshot())
            if (h.owned || h.registered) add(src, h.lo, h.hi);
        std::vector<gfd_ring::Window> keep;
        for (const auto& w : r->windows) {
            uint64_t lo = 0, hi = 0;
            if (allocation_of(r->ctx, w.kind, w.lo, w.hi - w.lo, &lo, &hi) && lo <= w.lo && w.hi <= hi) {
                keep.push_back(w);
                add(w.kind == 0 ? src : dst, w.lo, w.hi);
            }
        }
        r->windows.swap(keep);
    }
    AgentArgs a;
    memset(&a, 0, sizeof(a));
    a.q = r->q;
    a.mirror = r->d_mirror;
    if (r->tq != nullptr)
        a.tile_done = r->tq->d_tile_chunk_done != nullptr ? r->tq->d_tile_chunk_done
                                                         : const_cast<uint64_t*>(r->tq->tile_chunk_done);
    if (r->sq != nullptr) {
        a.list_done = r->sq->d_list_done;
        a.lists_completed = &r->sq->lists_completed;
    }
    a.dev = r->d_agent;
    a.host = r->h_agent;
    a.bytes_ctr = r->d_counters;
    a.start_slot = r->next;
    a.linger_ns = r->linger_ns;
    a.wait_limit_ns = r->ctx->timeout_ns;
    a.idle_limit_ns = r->ctx->timeout_ns;
    a.movers = r->movers;
    a.launch_id = ++r->launches;
    a.resident = r->resident ? 1u : 0u;
    // upload the tables only when they changed since the last launch (the agent appends
    // the ranges it learns to its own copy; those are among r->windows by then)
    uint64_t sum = 0xcbf29ce484222325ull;
    for (int k = 0; k < 2; ++k) {
        const AgentRanges& t = r->h_tables[k];
        for (uint32_t i = 0; i < t.n; ++i) sum = (sum ^ t.lo[i] ^ (t.hi[i] << 1)) * 0x100000001b3ull;
        sum = (sum ^ t.n) * 0x100000001b3ull;
    }
    cudaError_t e = cudaSuccess;
    if (!r->tables_current || sum != r->tables_sum) {
        e = cudaMemcpyAsync(&r->d_agent->src, r->h_tables, 2 * sizeof(AgentRanges), cudaMemcpyHostToDevice, r->stream);
        r->tables_sum = sum;
        r->tables_current = e == cudaSuccess;
    }
    // the launch counters (gen .. left) start at zero: the previous launch cleared them, or
    // the host does it here
    if (e == cudaSuccess && !(r->launches > 0 && r->h_agent->reset_ok))
        e = cudaMemsetAsync(&r->d_agent->gen, 0, 6 * sizeof(uint32_t), r->stream);
    if (e == cudaSuccess) e = launch_agent(a, r->stream);
    if (e == cudaSuccess) e = cudaEventRecord(r->agent_end, r->stream);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return cuda_error(r->ctx, e, "ring agent launch");
    }
    r->agent_live = true;
    r->agent_launches++;
    return GFD_OK;
}

// The agent of the last launch has finished: take over its position and status.  The
// caller holds r->mu.
int agent_finished_locked(gfd_ring* r) {
    r->agent_live = false;
    r->next = r->h_agent->next;
    if (r->h_agent->status == kAgentError)
        return set_error(r->ctx, GFD_ERR_TIMEOUT,
                         "ring agent: a bounded wait gave up (%llu so far); the ring stops consuming",
                         (unsigned long long)r->h_agent->timeouts);
    return GFD_OK;
}

bool marker_committed(const gfd_ring* r, uint64_t slot) {
    return __atomic_load_n(&r->q->entries[slot % gfd::QUEUE_SIZE].sequence, __ATOMIC_ACQUIRE) == slot + 1;
}

// Service thread: runs from gfd_ring_start to gfd_ring_stop.  It never touches
// descriptors or payload: while an agent launch runs it answers range queries (sleeping
// between checks); while none runs it watches the marker at r->next and relaunches.
void service_loop(gfd_ring* r) {
    driver().ctx_set_current(r->ctx->cu_ctx);  // the context the ring's stream lives in
    // This thread's naps are short waits for the agent; the default 50 us timer slack
    // would stretch every one of them (and the next relaunch behind it) past 70 us.
    prctl(PR_SET_TIMERSLACK, 1000UL, 0UL, 0UL, 0UL);
    uint32_t idle = 0;
    uint64_t stop_t0 = 0;
    for (;;) {
        bool live;
        {
            std::lock_guard<std::mutex> lk(r->mu);
            live = r->agent_live;
        }
        if (live) {
            const bool answered = answer_query(r);
            const cudaError_t q = cudaEventQuery(r->agent_end);
            if (q == cudaSuccess) {
                // a query left unanswered by a launch that ended is moot: the next launch
                // asks again with a new number
                std::lock_guard<std::mutex> lk(r->mu);
                if (agent_finished_locked(r) != GFD_OK || r->stopping.load()) return;
                idle = 0;
                continue;
            }
            if (q != cudaErrorNotReady) {
                std::lock_guard<std::mutex> lk(r->mu);
                r->agent_live = false;
                cuda_error(r->ctx, q, "ring agent");
                return;
            }
            if (answered) {
                idle = 0;
                continue;
            }
            if (r->stopping.load()) {
                // the agent drains what is committed and leaves; bound the wait for it
                if (stop_t0 == 0) stop_t0 = now_ns();
                if (now_ns() - stop_t0 > r->ctx->timeout_ns) {
                    set_error(r->ctx, GFD_ERR_TIMEOUT, "ring stop: the agent did not finish in time");
                    return;
                }
            }
            ++idle;
            if (idle < 200) cpu_relax();
            else std::this_thread::sleep_for(std::chrono::microseconds(5));
            continue;
        }
        if (r->stopping.load()) return;
        bool launched = false;
        {
            std::lock_guard<std::mutex> lk(r->mu);
            if (marker_committed(r, r->next)) {
                if (launch_agent_locked(r) != GFD_OK) return;
                launched = true;
            }
        }
        if (launched) {
            idle = 0;
            continue;
        }
        ++idle;
        if (idle < 20000) {
            cpu_relax();
        } else {
            // producers idle for a while: back off to 20 us naps
            std::this_thread::sleep_for(std::chrono::microseconds(20));
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
    if (const char* v = getenv("GFD_RING_RESIDENT")) r->resident = atoi(v) != 0;
    if (const char* v = getenv("GFD_RING_TEST_DROP_QUERIES")) r->drop_queries = atoi(v) != 0;
    if (const char* v = getenv("GFD_RING_LINGER_NS")) r->linger_ns = strtoull(v, nullptr, 10);
    if (const char* v = getenv("GFD_RING_MOVERS")) {
        const int m = atoi(v);
        if (m >= 1 && m <= kAgentMaxMovers) r->movers = static_cast<uint32_t>(m);
    }
    int lo = 0, hi = 0;
    cudaDeviceGetStreamPriorityRange(&lo, &hi);
    cudaError_t e = cudaStreamCreateWithPriority(&r->stream, cudaStreamNonBlocking, hi);
    if (e == cudaSuccess) e = cudaMalloc(&r->d_counters, sizeof(unsigned long long));
    // The mirror is published in the queue only while the ring runs (start .. stop) and
    // is never freed: a kernel that is still waiting when the ring goes away keeps
    // reading valid device memory until its bounded wait gives up.
    if (e == cudaSuccess) e = cudaMalloc(&r->d_mirror, sizeof(gfd::QueueMirror));
    if (e == cudaSuccess) e = cudaMalloc(&r->d_agent, sizeof(AgentDev));
    if (e == cudaSuccess) e = cudaMemsetAsync(r->d_agent, 0, sizeof(AgentDev), r->stream);
    if (e == cudaSuccess)
        e = cudaHostAlloc(reinterpret_cast<void**>(&r->h_agent), sizeof(AgentHost),
                          cudaHostAllocMapped | cudaHostAllocPortable);
    if (e == cudaSuccess) memset(const_cast<AgentHost*>(r->h_agent), 0, sizeof(AgentHost));
    if (e == cudaSuccess)
        e = cudaHostAlloc(reinterpret_cast<void**>(&r->h_tables), 2 * sizeof(AgentRanges), cudaHostAllocDefault);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&r->agent_end, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaMemsetAsync(r->d_counters, 0, sizeof(unsigned long long), r->stream);
    // only this ring's stream: the caller may have kernels running that wait on the ring
    if (e == cudaSuccess) e = cudaStreamSynchronize(r->stream);
    // load the kernels now, not at the first launch (lazy loading would queue that
    // launch behind a producer kernel that is waiting for it)
    if (e == cudaSuccess) e = preload_gather_kernels();
    if (e == cudaSuccess) e = preload_agent();
    if (e == cudaSuccess) {
        std::lock_guard<std::mutex> lk(ctx->mu);
        if (reserve_drain_slots(ctx, kDrainMax) != GFD_OK) e = cudaErrorMemoryAllocation;
    }
    // A managed-memory ring stays resident in host memory and is mapped by the GPU,
    // so neither the agent's reads nor the service thread's marker checks migrate pages.
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
    if (r->agent_end) cudaEventDestroy(r->agent_end);
    cudaFree(r->d_counters);  // d_mirror is kept (see gfd_ring_create)
    cudaFree(r->d_agent);
    if (r->h_agent) cudaFreeHost(const_cast<AgentHost*>(r->h_agent));
    if (r->h_tables) cudaFreeHost(r->h_tables);
    cudaGetLastError();
    delete r;
    return GFD_OK;
}

int gfd_ring_configure(gfd_ring* r, uint32_t movers, uint64_t linger_ns, int resident) {
    if (!r || movers > static_cast<uint32_t>(kAgentMaxMovers)) return GFD_ERR_INVALID;
    if (r->running.load()) return set_error(r->ctx, GFD_ERR_STATE, "gfd_ring_configure: the ring is running");
    std::lock_guard<std::mutex> lk(r->mu);
    r->movers = movers ? movers : static_cast<uint32_t>(kAgentDefaultMovers);
    r->linger_ns = linger_ns;
    r->resident = resident != 0;
    return GFD_OK;
}

int gfd_ring_allow(gfd_ring* r, const void* ptr, size_t bytes) {
    if (!r || !ptr) return GFD_ERR_INVALID;
    CtxScope scope(r->ctx->cu_ctx);
    const uint64_t p = reinterpret_cast<uint64_t>(ptr);
    uint64_t lo = 0, hi = 0;
    int kind = -1;
    {
        std::lock_guard<std::mutex> lk(r->ctx->mu);
        for (int k = 0; k < 2 && kind < 0; ++k)
            if (allocation_of(r->ctx, k, p, bytes ? bytes : 1, &lo, &hi)) kind = k;
    }
    if (kind < 0)
        return set_error(r->ctx, GFD_ERR_INVALID,
                         "gfd_ring_allow: %p is neither pinned, device-mapped host memory nor device memory of GPU %d",
                         ptr, r->ctx->device);
    if (bytes) {  // the declared window itself, not the whole allocation
        lo = p;
        hi = p + bytes;
    }
    std::lock_guard<std::mutex> lk(r->mu);
    remember(r, kind, lo, hi);
    return GFD_OK;
}

int gfd_ring_start(gfd_ring* r) {
    if (!r) return GFD_ERR_INVALID;
    CtxScope scope(r->ctx->cu_ctx);
    if (r->running.exchange(true)) return GFD_OK;
    int rc = GFD_OK;
    {
        std::lock_guard<std::mutex> lk(r->mu);
        // slots consumed while stopped (or reset by the owner) restart from read_idx
        cudaStreamSynchronize(r->stream);
        const uint64_t ri = __atomic_load_n(&r->q->read_idx, __ATOMIC_ACQUIRE);
        r->next = ri;
        r->gate.reset();
        r->stopping = false;
        r->h_agent->stop = 0;
        // device-side waits poll the mirror while the ring runs
        const gfd::QueueMirror init{ri, __atomic_load_n(&r->q->done_idx, __ATOMIC_ACQUIRE)};
        if (r->d_mirror != nullptr &&
            cudaMemcpyAsync(r->d_mirror, &init, sizeof(init), cudaMemcpyHostToDevice, r->stream) == cudaSuccess &&
            cudaStreamSynchronize(r->stream) == cudaSuccess) {
            r->q->mirror = r->d_mirror;
            std::atomic_thread_fence(std::memory_order_seq_cst);
        }
        cudaGetLastError();
        rc = launch_agent_locked(r);
        if (rc == GFD_OK && r->resident) {
            // resident mode: return once every CTA of the agent runs, so kernels launched
            // from now on find it on the GPU (bounded).  In the default mode the agent
            // leaves after linger_ns anyway and may start later (behind a kernel that
            // fills the GPU, e.g. a session's own), so there is nothing to wait for.
            const uint32_t id = r->launches;
            const uint64_t t0 = now_ns(), limit = std::min<uint64_t>(r->ctx->timeout_ns, 2000000000ull);
            while (r->h_agent->resident != id && r->h_agent->exited != id) {
                if (now_ns() - t0 > limit) {
                    rc = set_error(r->ctx, GFD_ERR_TIMEOUT,
                                   "ring start: the agent's %u CTAs did not become resident (SMs busy?)",
                                   r->movers + 1);
                    r->h_agent->stop = 1;  // if it starts later, it drains and leaves
                    break;
                }
                std::this_thread::sleep_for(std::chrono::microseconds(5));
            }
        }
    }
    r->thread = std::thread(service_loop, r);
    if (rc != GFD_OK) {
        gfd_ring_stop(r);
        return rc;
    }
    return GFD_OK;
}

int gfd_ring_stop(gfd_ring* r) {
    if (!r) return GFD_ERR_INVALID;
    CtxScope scope(r->ctx->cu_ctx);
    int rc = GFD_OK;
    if (r->running.exchange(false)) {
        // the agent drains what is committed and leaves; the service thread follows it
        r->h_agent->stop = 1;
        std::atomic_thread_fence(std::memory_order_seq_cst);
        r->stopping = true;
        if (r->thread.joinable()) r->thread.join();
        std::lock_guard<std::mutex> lk(r->mu);
        if (r->agent_live && cudaEventQuery(r->agent_end) != cudaSuccess) {
            // the agent has not finished within the bound (see service_loop): leave the
            // queue published to it rather than wait without a limit
            cudaGetLastError();
            return set_error(r->ctx, GFD_ERR_TIMEOUT, "ring stop: the agent did not finish in time");
        }
        cudaError_t e = cudaStreamSynchronize(r->stream);
        if (r->agent_live) rc = agent_finished_locked(r);
        // slots committed after the agent left: drain them from here (the queue is still
        // owned by the caller; after a stop the ring never touches it again)
        int launched = 0;
        if (rc == GFD_OK) rc = poll_locked(r, true, &launched);
        if (e == cudaSuccess) e = cudaStreamSynchronize(r->stream);
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
    if (launched) *launched = 0;
    if (r->running.load()) return GFD_OK;  // the agent consumes the ring
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
            cudaError_t q = cudaStreamQuery(r->stream);
            if (q != cudaSuccess && q != cudaErrorNotReady) return cuda_error(r->ctx, q, "ring drain");
        }
        std::this_thread::sleep_for(std::chrono::microseconds(5));
    }
    return GFD_OK;
}

int gfd_ring_counters(const gfd_ring* r, uint64_t* consumed, uint64_t* drains, uint64_t* bytes) {
    if (!r) return GFD_ERR_INVALID;
    // descriptors and batches completed by agent launches live in device memory; read them
    // with a copy that does not wait for the (possibly running) agent
    unsigned long long dev[3] = {0, 0, 0};
    {
        CtxScope scope(r->ctx->cu_ctx);
        if (!r->running.load()) cudaStreamSynchronize(r->stream);
        cudaError_t e = cudaMemcpy(&dev[0], &r->d_agent->consumed, 2 * sizeof(unsigned long long),
                                   cudaMemcpyDeviceToHost);
        if (e == cudaSuccess) e = cudaMemcpy(&dev[2], r->d_counters, sizeof(unsigned long long), cudaMemcpyDeviceToHost);
        if (e != cudaSuccess) {
            cudaGetLastError();
            return GFD_ERR_CUDA;
        }
    }
    if (consumed) *consumed = r->consumed.load() + dev[0];
    if (drains) *drains = r->drains.load() + dev[1];
    if (bytes) *bytes = dev[2];
    return GFD_OK;
}

int gfd_ring_agent_stats(const gfd_ring* r, gfd_ring_agent_stats_t* out) {
    if (!r || !out) return GFD_ERR_INVALID;
    out->launches = r->agent_launches.load();
    out->queries = r->h_agent->queries;
    out->rejected = r->h_agent->rejected;
    out->timeouts = r->h_agent->timeouts;
    out->idle_exits = r->h_agent->exits[kAgentIdle];
    out->stop_exits = r->h_agent->exits[kAgentStopped];
    out->error_exits = r->h_agent->exits[kAgentError];
    out->resident = r->resident ? 1 : 0;
    const AgentHost* h = r->h_agent;
    const uint64_t t0 = h->t_start;
    auto rel = [t0](uint64_t t) { return t > t0 ? t - t0 : 0ull; };
    out->last_first_batch_ns = h->t_first ? rel(h->t_first) : 0;
    out->last_done_ns = h->t_done ? rel(h->t_done) : 0;
    out->last_exit_ns = h->t_exit ? rel(h->t_exit) : 0;
    return GFD_OK;
}

}  // extern "C"
