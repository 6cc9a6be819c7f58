#pragma once
// Warp-specialised scatter-gather framework (dynamic (src, dst, size) lists).
//
// Same user contract as the reference interface include/gfd/sg_warp_spec.cuh:31-314:
// a functor with __device__ void operator()(gfd::sg_warp_spec::SGListView), the
// macro GFD_SG_WARP_SPEC_KERNEL, kernel signature (DescriptorQueue*, SGTaskQueue*,
// ComputeFn), lists claimed with atomicAdd on list_read_idx and accepted when their
// marker equals slot + 1 (or abandoned when `terminate` is set), d_list_done[list_id]
// raised and lists_completed incremented once the list's bytes are in GPU memory,
// the functor called once per list by one warp, the list's marker cleared once the
// list is released.
//
// B200 mechanism: the producer warps read the list's entries from the pool and pull
// the payload themselves (one warp per entry, 32 entries prefetched per warp with
// one coalesced load), instead of converting entries to descriptors for a CPU
// poller.  Lists a device submitter committed as device-entry lists
// (SG_FLAG_DEVICE_ENTRIES, sg_device_primitives.cuh) are read from the session's device
// mirror instead of the host pool.  Compute warps take successive lists round-robin from an 8-deep shared
// memory ring, so pulling list i+1 overlaps computing on list i.  A list is released
// (marker cleared, entry_consumed_idx raised to the end of its entries) after the
// functor has run -- SGListView reads the entries -- and strictly in list order.  Producer warp count comes from sq->producer_warps (set by
// SGWarpSpecSession); with 0 the reference layout is assumed (warp 0 pulls, the rest
// compute).  Every wait is bounded by sq->wait_limit_ns (0: GFD_DEVICE_WAIT_LIMIT_NS);
// a give-up increments sq->wait_timeouts and winds the CTA down.

#include <cstdint>

#include "gfd/descriptor_queue.h"
#include "gfd/pull.cuh"
#include "gfd/sg_device_primitives.cuh"
#include "gfd/wait.cuh"

namespace gfd {
namespace sg_warp_spec {

struct SGListView {
    uint32_t list_id;
    uint32_t count;
    uint32_t flags;
    int lane_id;
    uint32_t pool_offset;
    const SGTaskQueue* sq;
    const DeviceSGEntry* pool;  // library extension: the device pool of a device-entry list
                                // (SG_FLAG_DEVICE_ENTRIES), else null (sq->entries)

    // Volatile loads: pool slots are rewritten as the pool wraps, so an entry must not
    // come from a cache line an earlier list left in L1.
    __device__ __forceinline__ DeviceSGEntry get_entry(uint32_t idx) const {
        const DeviceSGEntry* e = (pool != nullptr ? pool : sq->entries) + (pool_offset + idx) % MAX_SG_POOL_ENTRIES;
        DeviceSGEntry r;
        r.src_addr = *reinterpret_cast<const volatile uint64_t*>(&e->src_addr);
        r.dst_addr = *reinterpret_cast<const volatile uint64_t*>(&e->dst_addr);
        r.size = *reinterpret_cast<const volatile uint32_t*>(&e->size);
        r.tag = *reinterpret_cast<const volatile uint32_t*>(&e->tag);
        return r;
    }
    template <typename T>
    __device__ __forceinline__ T* dst_ptr(uint32_t idx) const {
        return reinterpret_cast<T*>(get_entry(idx).dst_addr);
    }
    __device__ __forceinline__ uint32_t entry_size(uint32_t idx) const { return get_entry(idx).size; }
};

// Reference shared-state layout, kept for hand-written kernels that declare it.
struct _SGWarpSpecState {
    uint32_t list_id;
    uint32_t count;
    uint32_t pool_offset;
    uint32_t flags;
    volatile int list_ready;
    volatile int compute_done;
    volatile int terminated;
};

constexpr int kListSlots = 8;
constexpr uint32_t kSlotEmpty = 0xffffffffu;
constexpr uint32_t kListEnd = 0xffffffffu;

struct _ListSlot {
    volatile uint32_t seq;  // local list number held, kSlotEmpty when free
    uint32_t list_id;       // kListEnd: no more lists
    uint32_t count;
    uint32_t pool_offset;
    uint32_t flags;
    uint64_t release_to;    // absolute entry index one past this list
    uint64_t claim_idx;     // list index claimed from list_read_idx
    const DeviceSGEntry* pool;  // device pool of a device-entry list, else null
};

struct _ListPipe {
    _ListSlot slot[kListSlots];
    volatile uint32_t abort;
    volatile uint32_t b_state, b_list_id, b_count, b_pool_offset, b_flags, b_ring;
    volatile unsigned long long b_release, b_idx;
    const DeviceSGEntry* volatile b_pool;  // where the list's entries are
};

__device__ __forceinline__ void _sg_producer_bar(uint32_t threads) {
    asm volatile("bar.sync 1, %0;" ::"r"(threads) : "memory");
}

// Wait sites recorded in sq->timeout_site when a wait gives up.
enum : uint32_t { kSiteSlotFree = 1, kSiteListCommit = 2, kSiteEndSlot = 3, kSiteComputeSlot = 4 };

template <typename Pred>
__device__ __forceinline__ bool _sg_wait(volatile uint32_t* abort, Pred pred, uint64_t limit_ns, SGTaskQueue* sq,
                                         uint32_t site) {
    const uint64_t t0 = wait::now();
    uint32_t polls = 0;
    while (!pred()) {
        if (*abort) return false;
        if (wait::expired(t0, limit_ns)) {
            *abort = 1;
            sq->timeout_site = site;
            wait::note_timeout(&sq->wait_timeouts);
            if (sq->stats) atomicAdd(&sq->stats->timeouts, 1ull);
            return false;
        }
        wait::backoff(polls);
    }
    return true;
}

// One poll round by the token holder: reads the markers of lists [scan, scan + window)
// and the terminate word from host memory and publishes them in the device-memory
// mirror.  Non-blocking.  The loads are relaxed so that all of them are in flight
// together -- acquire loads would wait for one another, one PCIe round trip each, and
// under a saturated link a round trip queues behind the payload reads (measured: the
// start of a config 5 pass pulled at ~1/6 of the link rate for ~200 us while lists
// were discovered this way) -- and the system fence after them makes the round an
// acquire of everything the markers published.
__device__ __forceinline__ void _sg_mirror_round(SGTaskQueue* sq, SGPollMirror* m) {
    const uint64_t now = wait::now();
    if (now - m->last_poll_ns < kMirrorPollNs) return;
    m->last_poll_ns = now;
    const uint64_t scan = m->scan;
    uint64_t seq[kMirrorWindow];
#pragma unroll
    for (uint32_t k = 0; k < kMirrorWindow; ++k)
        seq[k] = wait::load_relaxed_sys(&sq->lists[(scan + k) % MAX_SG_LISTS].sequence);
    const uint32_t term = wait::load_relaxed_sys(&sq->terminate);
    // acquire of what the markers published (headers, pool entries), and release of it
    // to anyone who sees the mirror entries written below
    __threadfence_system();
    uint64_t adv = scan;
    bool prefix = true;
#pragma unroll
    for (uint32_t k = 0; k < kMirrorWindow; ++k) {
        if (seq[k] == scan + k + 1) {
            m->committed[(scan + k) % MAX_SG_LISTS] = scan + k + 1;
            if (prefix) adv = scan + k + 1;
        } else if (m->committed[(scan + k) % MAX_SG_LISTS] == scan + k + 1) {
            // a device-entry list: committed in device memory only (no host marker)
            if (prefix) adv = scan + k + 1;
        } else {
            prefix = false;
        }
    }
    m->scan = adv;
    if (term) m->terminate = 1u;
    __threadfence();
}

// Waits until list `idx` is committed (*committed = true) or the queue terminates.
// Returns false when the wait gave up (abort flag or time limit).
__device__ __forceinline__ bool _sg_wait_commit(SGTaskQueue* sq, uint64_t idx, volatile uint32_t* abort,
                                                uint64_t limit_ns, bool* committed) {
    SGList* l = &sq->lists[idx % MAX_SG_LISTS];
    SGPollMirror* m = sq->poll_mirror;
    *committed = false;
    const uint64_t t0 = wait::now();
    uint32_t polls = 0;
    for (;;) {
        if (m == nullptr) {
            if (wait::load_acquire_sys(&l->sequence) == idx + 1) {
                *committed = true;
                return true;
            }
            if (wait::load_acquire_sys(&sq->terminate) != 0u) return true;
        } else {
            if (m->committed[idx % MAX_SG_LISTS] == idx + 1) {
                __threadfence_system();  // acquire: pairs with the holder's fence
                *committed = true;
                return true;
            }
            if (m->terminate != 0u) return true;
            if (atomicCAS(&m->token, 0u, 1u) == 0u) {
                _sg_mirror_round(sq, m);
                atomicExch(&m->token, 0u);
            }
        }
        if (*abort) return false;
        if (wait::expired(t0, limit_ns)) {
            *abort = 1;
            sq->timeout_site = kSiteListCommit;
            wait::note_timeout(&sq->wait_timeouts);
            if (sq->stats) atomicAdd(&sq->stats->timeouts, 1ull);
            return false;
        }
        wait::backoff(polls);
    }
}

__device__ __forceinline__ uint64_t _ld_volatile_u64(const void* p) {
    return *static_cast<const volatile uint64_t*>(p);
}

// Marks the list claimed as `idx` (ring slot idx % MAX_SG_LISTS) as processed, then
// releases every processed list at the head of the ring in list order: clears its
// marker (the slot may be reused) and raises entry_consumed_idx to the end of its
// entries.  Releasing strictly in list order keeps a fast CTA from freeing pool
// entries of an older list that another CTA is still reading.
// Mirror mode of _release_list: cursor, marks and consumed count in device memory; the
// list markers (host) are cleared and entry_consumed_idx published once per release
// round.  A round releases every processed list at the head of the ring at once (up to
// kReleaseBatch): the marks and markers of all of them are cleared, then one system
// fence makes the marker clears land before the slots are handed back (slot_free) --
// instead of three system fences per list, each of which waits a PCIe round trip that
// queues behind the payload reads of a saturated link (measured ~70 us per release, so
// the in-order release chain fell behind the pulls and kept the pool full).
constexpr uint32_t kReleaseBatch = 64;

__device__ __forceinline__ void _release_list_mirror(SGTaskQueue* sq, SGPollMirror* m, uint64_t idx,
                                                     uint64_t entries_end) {
    m->release_end[idx % MAX_SG_LISTS] = entries_end + 1;  // +1: an empty first list ends at 0
    __threadfence();
    for (uint32_t guard = 0; guard < 4u * MAX_SG_LISTS; ++guard) {
        const unsigned long long r = *reinterpret_cast<volatile unsigned long long*>(&m->released);
        // a mark is cleared when its list is released and set only by the list's own
        // consumer (the slot's previous list was released before this one was committed)
        uint32_t k = 0;
        uint64_t end = 0;
        while (k < kReleaseBatch) {
            const uint64_t mark = m->release_end[(r + k) % MAX_SG_LISTS];
            if (mark == 0) break;  // not processed yet
            end = mark - 1;
            ++k;
        }
        if (k == 0) break;                                     // head not processed yet
        if (atomicCAS(&m->released, r, r + k) != r) continue;  // another CTA advanced it
        for (uint32_t j = 0; j < k; ++j) m->release_end[(r + j) % MAX_SG_LISTS] = 0;
        __threadfence();  // the marks are clear before any slot can be reused
        for (uint32_t j = 0; j < k; ++j) sq->lists[(r + j) % MAX_SG_LISTS].sequence = 0;  // slots free for submitters
        __threadfence_system();  // the clears land before a new marker can follow
        for (uint32_t j = 0; j < k; ++j) m->slot_free[(r + j) % MAX_SG_LISTS] = r + j + 1;
        atomicMax(&m->consumed, static_cast<unsigned long long>(end));
        wait::publish_max(&sq->entry_consumed_idx, end);
        __threadfence();
    }
}

__device__ __forceinline__ void _release_list(SGTaskQueue* sq, uint64_t idx, uint64_t entries_end) {
    if (sq->poll_mirror != nullptr) {
        _release_list_mirror(sq, sq->poll_mirror, idx, entries_end);
        return;
    }
    sq->lists[idx % MAX_SG_LISTS].release_end = entries_end;
    __threadfence_system();
    unsigned long long* cursor = reinterpret_cast<unsigned long long*>(const_cast<uint64_t*>(&sq->lists_released));
    unsigned long long* consumed =
        reinterpret_cast<unsigned long long*>(const_cast<uint64_t*>(&sq->entry_consumed_idx));
    for (uint32_t guard = 0; guard < 4u * MAX_SG_LISTS; ++guard) {
        const unsigned long long r = wait::load_acquire_sys(&sq->lists_released);
        SGList* l = &sq->lists[r % MAX_SG_LISTS];
        const uint64_t end = wait::load_acquire_sys(&l->release_end);
        if (end == 0 || wait::load_acquire_sys(&l->sequence) != r + 1) break;  // head not processed yet
        if (atomicCAS(cursor, r, r + 1) != r) continue;                          // another CTA advanced it
        l->release_end = 0;
        __threadfence_system();
        l->sequence = 0;
        unsigned long long cur = *reinterpret_cast<volatile unsigned long long*>(consumed);
        while (cur < end) {
            const unsigned long long prev = atomicCAS(consumed, cur, static_cast<unsigned long long>(end));
            if (prev == cur) break;
            cur = prev;
        }
        __threadfence_system();
    }
}

// Signals that list `idx` (list_id) has landed: d_list_done[list_id], lists_completed
// and, with the mirror, list_read_idx (published here rather than at the claim).  Lane 0 of
// the warp that runs the list's functor calls it before the functor, after it has seen
// the producers' hand-off of the list (their payload stores precede it), so the fences
// and host-memory round trips it costs stay off the producer warps' path.
__device__ __forceinline__ void _sg_list_landed(SGTaskQueue* sq, uint32_t list_id, uint64_t idx) {
    __threadfence();
    if (sq->d_list_done != nullptr && list_id < static_cast<uint32_t>(MAX_SG_LISTS))
        *reinterpret_cast<volatile uint64_t*>(&sq->d_list_done[list_id]) = 1;
    __threadfence_system();
    if (sq->poll_mirror != nullptr) {  // count in device memory, publish the host counters
        wait::publish_max(&sq->list_read_idx, idx + 1);
        const unsigned long long done = atomicAdd(&sq->poll_mirror->completed, 1ull) + 1ull;
        wait::publish_max(&sq->lists_completed, done);
    } else {
        atomicAdd(reinterpret_cast<unsigned long long*>(const_cast<uint64_t*>(&sq->lists_completed)), 1ull);
    }
    __threadfence_system();
}

// framework_warps: the first framework_warps warps of the block run the framework
// (0: all of them), so a kernel may add warps of its own, e.g. a GPU-side list
// submitter, after them.  Only the framework warps may call this function.
template <typename ComputeFn>
__device__ void _sg_transfer_warp_loop(DescriptorQueue* dq, SGTaskQueue* sq, ComputeFn compute_fn,
                                       uint32_t framework_warps = 0) {
    (void)dq;  // descriptors are not needed: producers pull the entries directly
    __shared__ _ListPipe pipe;
    const uint32_t warp = threadIdx.x >> 5;
    const uint32_t lane = threadIdx.x & 31;
    const uint32_t nwarps = framework_warps ? framework_warps : (blockDim.x >> 5);
    uint32_t P = sq->producer_warps ? sq->producer_warps : 1u;
    if (nwarps == 1) P = 1;
    else if (P > nwarps - 1) P = nwarps - 1;
    const uint32_t Kc = nwarps - P;  // 0 only when the block is a single warp
    const uint64_t limit = sq->wait_limit_ns;
    TransferStats* stats = sq->stats;

    if (threadIdx.x < kListSlots) pipe.slot[threadIdx.x].seq = kSlotEmpty;
    if (threadIdx.x == 0) pipe.abort = 0;
    asm volatile("bar.sync 2, %0;" ::"r"(nwarps * 32u) : "memory");  // framework warps only

    if (warp < P) {
        const uint32_t pt = threadIdx.x, np = P * 32u;
        for (uint32_t j = 0;; ++j) {
            _ListSlot& s = pipe.slot[j % kListSlots];
            if (pt == 0) {
                uint32_t state = 0;  // 0 list, 1 end
                if (!_sg_wait(&pipe.abort, [&] { return Kc == 0 || s.seq == kSlotEmpty; }, limit, sq, kSiteSlotFree)) {
                    state = 1;
                } else {
                    SGPollMirror* const mm = sq->poll_mirror;
                    unsigned long long idx;
                    if (mm != nullptr) {  // claim in device memory; list_read_idx follows when it lands
                        idx = atomicAdd(&mm->claim, 1ull);
                    } else {
                        idx = atomicAdd(reinterpret_cast<unsigned long long*>(const_cast<uint64_t*>(&sq->list_read_idx)),
                                        1ull);
                    }
                    const uint32_t ring = static_cast<uint32_t>(idx % MAX_SG_LISTS);
                    SGList* l = &sq->lists[ring];
                    bool committed = false;
                    const bool ok = _sg_wait_commit(sq, idx, &pipe.abort, limit, &committed);
                    if (!ok || !committed) {
                        state = 1;
                    } else {
                        // with the mirror, list_read_idx is published when the list has
                        // landed (_sg_list_landed): the claims of every CTA at launch do not
                        // queue on one host word, and the pull does not wait for it
                        pipe.b_ring = ring;
                        pipe.b_idx = idx;
                        const SGDeviceListHdr* dh = mm != nullptr ? &mm->hdr[ring] : nullptr;
                        if (dh != nullptr && dh->seq == idx + 1) {
                            // device-entry list: header, entries and first index in device memory
                            pipe.b_pool_offset = *reinterpret_cast<const volatile uint32_t*>(&dh->pool_offset);
                            pipe.b_count = *reinterpret_cast<const volatile uint32_t*>(&dh->count);
                            pipe.b_list_id = *reinterpret_cast<const volatile uint32_t*>(&dh->list_id);
                            pipe.b_flags = *reinterpret_cast<const volatile uint32_t*>(&dh->flags);
                            pipe.b_release = *reinterpret_cast<const volatile unsigned long long*>(&dh->first_entry);
                            pipe.b_pool = mm->pool;
                        } else {
                            const uint32_t off = *reinterpret_cast<volatile uint32_t*>(&l->pool_offset);
                            const uint32_t count = *reinterpret_cast<volatile uint32_t*>(&l->count);
                            pipe.b_list_id = *reinterpret_cast<volatile uint32_t*>(&l->list_id);
                            pipe.b_flags = *reinterpret_cast<volatile uint32_t*>(&l->flags);
                            pipe.b_pool_offset = off;
                            pipe.b_count = count;
                            pipe.b_pool = sq->entries;
                            // absolute index of the list's first entry: the largest value
                            // congruent to `off` not above entry_alloc_idx - count (any
                            // allocation count from this list's end up to one pool past it
                            // gives the same answer; device submitters count in the mirror
                            // first and publish entry_alloc_idx after the marker)
                            uint64_t a = wait::load_acquire_sys(&sq->entry_alloc_idx);
                            if (mm != nullptr && *reinterpret_cast<volatile unsigned int*>(&mm->alloc_state) == 2u) {
                                const uint64_t ad = sg::detail::ld_dev(&mm->entry_alloc);
                                if (ad > a) a = ad;
                            }
                            const uint64_t x = a - count - off;
                            pipe.b_release = a - count - (x % MAX_SG_POOL_ENTRIES);
                        }
                    }
                }
                pipe.b_state = state;
            }
            _sg_producer_bar(np);
            const uint32_t state = pipe.b_state;
            const uint32_t count = pipe.b_count, off = pipe.b_pool_offset;
            const DeviceSGEntry* const pool = pipe.b_pool;
            _sg_producer_bar(np);
            if (state != 0) {
                if (pt == 0 && !pipe.abort) {
                    for (uint32_t e = 0; e < Kc; ++e) {
                        _ListSlot& se = pipe.slot[(j + e) % kListSlots];
                        if (!_sg_wait(&pipe.abort, [&] { return se.seq == kSlotEmpty; }, limit, sq, kSiteEndSlot)) break;
                        se.list_id = kListEnd;
                        __threadfence_block();
                        se.seq = j + e;
                    }
                }
                break;
            }
            // pull: producer warp w takes entries w*32 .. in groups of 32 (one coalesced prefetch)
            uint64_t moved = 0;
            for (uint32_t base = warp * 32u; base < count; base += P * 32u) {
                const uint32_t i = base + lane;
                uint64_t src = 0, dst = 0, size = 0;
                if (i < count) {
                    const DeviceSGEntry* e = &pool[(off + i) % MAX_SG_POOL_ENTRIES];
                    src = _ld_volatile_u64(&e->src_addr);
                    dst = _ld_volatile_u64(&e->dst_addr);
                    size = *reinterpret_cast<const volatile uint32_t*>(&e->size);
                }
                const uint32_t n_here = count - base < 32u ? count - base : 32u;
                for (uint32_t q = 0; q < n_here; ++q) {
                    const uint64_t qs = __shfl_sync(0xffffffffu, src, q);
                    const uint64_t qd = __shfl_sync(0xffffffffu, dst, q);
                    const uint64_t qn = __shfl_sync(0xffffffffu, size, q);
                    pull::warp_copy(reinterpret_cast<void*>(qd), reinterpret_cast<const void*>(qs), qn);
                    moved += qn;
                }
            }
            _sg_producer_bar(np);
            if (lane == 0 && stats != nullptr && moved) atomicAdd(&stats->bytes, static_cast<unsigned long long>(moved));
            if (pt == 0) {
                const uint32_t list_id = pipe.b_list_id;
                // the compute warp that takes the list signals it (_sg_list_landed); a
                // single-warp block signals here
                if (Kc == 0) _sg_list_landed(sq, list_id, pipe.b_idx);
                else __threadfence();
                if (stats != nullptr) atomicAdd(&stats->tokens, static_cast<unsigned long long>(count));
                s.list_id = list_id;
                s.count = count;
                s.pool_offset = off;
                s.flags = pipe.b_flags;
                s.release_to = pipe.b_release + count;
                s.claim_idx = pipe.b_idx;
                s.pool = pool == sq->entries ? nullptr : pool;
                __threadfence_block();
                s.seq = j;
            }
            if (Kc == 0) {
                // single-warp block: the producer warp is also the compute warp
                __syncwarp();
                SGListView v{s.list_id, s.count, s.flags, static_cast<int>(lane), s.pool_offset, sq, s.pool};
                compute_fn(v);
                __syncwarp();
                if (lane == 0) {
                    _release_list(sq, s.claim_idx, s.release_to);
                    s.seq = kSlotEmpty;
                }
            }
            if (pipe.abort) break;
        }
    } else {
        const uint32_t c = warp - P;
        for (uint32_t j = c;; j += Kc) {
            _ListSlot& s = pipe.slot[j % kListSlots];
            int ok = 1;
            if (lane == 0) ok = _sg_wait(&pipe.abort, [&] { return s.seq == j; }, limit, sq, kSiteComputeSlot);
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) break;
            __threadfence_block();
            if (s.list_id == kListEnd) break;
            if (lane == 0) _sg_list_landed(sq, s.list_id, s.claim_idx);
            __syncwarp();
            SGListView v{s.list_id, s.count, s.flags, static_cast<int>(lane), s.pool_offset, sq, s.pool};
            compute_fn(v);
            __syncwarp();
            if (lane == 0) {
                _release_list(sq, s.claim_idx, s.release_to);
                __threadfence_block();
                s.seq = kSlotEmpty;
            }
        }
    }
}

}  // namespace sg_warp_spec
}  // namespace gfd

// Compiled for blocks of up to GFD_SG_WARP_SPEC_MAX_THREADS threads (define it before
// including this header to change it); the session refuses larger launch shapes.
#ifndef GFD_SG_WARP_SPEC_MAX_THREADS
#define GFD_SG_WARP_SPEC_MAX_THREADS 640
#endif

#define GFD_SG_WARP_SPEC_KERNEL(kernel_name, ComputeFnType)                                     \
    __global__ void __launch_bounds__(GFD_SG_WARP_SPEC_MAX_THREADS)                            \
        kernel_name(gfd::DescriptorQueue* dq, gfd::SGTaskQueue* sq, ComputeFnType compute_fn) { \
        gfd::sg_warp_spec::_sg_transfer_warp_loop(dq, sq, compute_fn);                         \
    }
