#pragma once
// Warp-collective device primitives for the scatter-gather task queue.
//
// Same functions and protocol as the reference interface
// include/gfd/sg_device_primitives.cuh:28-243: reserve pool entries and a list slot
// with atomics, write the entries, then commit (header, fence, marker sequence =
// slot + 1).  Waits are bounded by sq->wait_limit_ns
// (0: GFD_DEVICE_WAIT_LIMIT_NS); a give-up increments sq->wait_timeouts.
// sg_wait_list_space additionally waits until the ring slot it will use has been
// released by the consumer (its marker is 0).

#include <cstdint>

#include "gfd/sg_task_queue.h"
#include "gfd/wait.cuh"

namespace gfd {
namespace sg {

namespace detail {

__device__ __forceinline__ uint64_t ld_dev(const unsigned long long* p) {
    return *reinterpret_cast<const volatile unsigned long long*>(p);
}

}  // namespace detail

// Submitter-side view of a queue (library extension): the control fields the host sets
// before the launch (mirror pointer, wait limit) read once, so a warp that submits many
// lists does not cross PCIe for them on every call.  The sg_* functions below build one
// per call; kernels that submit in a loop may build one up front and use its members.
//
// With the session's device mirror, allocation and the pool / ring space checks run on
// device-memory counters (seeded once per launch from entry_alloc_idx / list_alloc_idx,
// so lists the host submitted first are counted), and the host-visible counters are
// raised after each list's marker; without it every step works on the host words as
// in the reference.
struct SGSubmitter {
    SGTaskQueue* sq;
    SGPollMirror* m;
    uint64_t limit_ns;

    __device__ __forceinline__ explicit SGSubmitter(SGTaskQueue* q) : sq(q) {
        uint64_t mv, lv;
        asm("ld.global.nc.u64 %0, [%1];" : "=l"(mv) : "l"(&q->poll_mirror));
        asm("ld.global.nc.u64 %0, [%1];" : "=l"(lv) : "l"(&q->wait_limit_ns));
        m = reinterpret_cast<SGPollMirror*>(mv);
        limit_ns = lv;
    }

    // Lane 0 only.  Seeds the device counters once per launch (the first device
    // submitter does it; others wait, bounded).  False when the wait gave up.
    __device__ __forceinline__ bool mirror_ready() const {
        volatile unsigned int* state = &m->alloc_state;
        if (*state == 2u) return true;
        if (atomicCAS(&m->alloc_state, 0u, 1u) == 0u) {
            const uint64_t e = wait::load_acquire_sys(&sq->entry_alloc_idx);
            const uint64_t l = wait::load_acquire_sys(&sq->list_alloc_idx);
            *reinterpret_cast<volatile unsigned long long*>(&m->entry_alloc) = e;
            *reinterpret_cast<volatile unsigned long long*>(&m->list_alloc) = l;
            __threadfence();
            atomicExch(&m->alloc_state, 2u);
            return true;
        }
        const uint64_t t0 = wait::now();
        uint32_t polls = 0;
        while (*state != 2u) {
            if (wait::expired(t0, limit_ns)) {
                wait::note_timeout(&sq->wait_timeouts);
                return false;
            }
            wait::backoff(polls);
        }
        __threadfence();
        return true;
    }

    __device__ __forceinline__ bool mirrored() const { return m != nullptr && mirror_ready(); }

    // Lane 0 waits until the pool has room for `needed` more entries.  Returns false
    // (warp-uniform) when the wait gave up.
    __device__ __forceinline__ bool wait_entry_space(uint32_t needed) const {
        int ok = 1;
        if ((threadIdx.x & 31) == 0) {
            const bool mir = m != nullptr;
            ok = !mir || mirror_ready();
            if (ok) {
                const uint64_t t0 = wait::now();
                uint32_t polls = 0;
                for (;;) {
                    uint64_t alloc, consumed;
                    if (mir) {
                        alloc = detail::ld_dev(&m->entry_alloc);
                        consumed = detail::ld_dev(&m->consumed);
                    } else {
                        alloc = sq->entry_alloc_idx;
                        consumed = wait::load_acquire_sys(&sq->entry_consumed_idx);
                    }
                    if (alloc - consumed <= static_cast<uint64_t>(MAX_SG_POOL_ENTRIES - needed)) break;
                    if (wait::expired(t0, limit_ns)) {
                        wait::note_timeout(&sq->wait_timeouts);
                        ok = 0;
                        break;
                    }
                    wait::backoff(polls);
                }
            }
        }
        return __shfl_sync(0xffffffffu, ok, 0) != 0;
    }

    // Lane 0 waits until the list ring has `n` free slots after the ones allocated: the
    // reference condition (with consumers that claimed ahead counted as no backlog), plus:
    // the last of those slots has been released by its previous list (slots are released
    // in list order, so the ones before it have been too; with the mirror this is the
    // per-slot release record, else the marker in host memory).  Returns false
    // (warp-uniform) when the wait gave up.
    __device__ __forceinline__ bool wait_list_space(uint32_t n = 1) const {
        int ok = 1;
        if ((threadIdx.x & 31) == 0) {
            const bool mir = m != nullptr;
            ok = !mir || mirror_ready();
            if (ok) {
                const uint64_t t0 = wait::now();
                uint32_t polls = 0;
                for (;;) {
                    bool room;
                    if (mir) {
                        const uint64_t alloc = detail::ld_dev(&m->list_alloc);
                        const uint64_t read = detail::ld_dev(&m->claim);
                        const uint64_t pending = alloc > read ? alloc - read : 0;
                        const uint64_t last = alloc + n - 1;
                        room = pending + n <= static_cast<uint64_t>(MAX_SG_LISTS - 1) &&
                               (last < static_cast<uint64_t>(MAX_SG_LISTS) ||
                                m->slot_free[last % MAX_SG_LISTS] >= last - MAX_SG_LISTS + 1);
                    } else {
                        const uint64_t alloc = sq->list_alloc_idx;
                        const uint64_t read = wait::load_acquire_sys(&sq->list_read_idx);
                        const uint64_t pending = alloc > read ? alloc - read : 0;
                        room = pending + n <= static_cast<uint64_t>(MAX_SG_LISTS - 1) &&
                               wait::load_acquire_sys(&sq->lists[(alloc + n - 1) % MAX_SG_LISTS].sequence) == 0;
                    }
                    if (room) break;
                    if (wait::expired(t0, limit_ns)) {
                        wait::note_timeout(&sq->wait_timeouts);
                        ok = 0;
                        break;
                    }
                    wait::backoff(polls);
                }
            }
        }
        return __shfl_sync(0xffffffffu, ok, 0) != 0;
    }

    // Reserves `count` pool entries (warp-uniform result).
    __device__ __forceinline__ uint64_t alloc_entries(uint32_t count) const {
        unsigned long long base = 0;
        if ((threadIdx.x & 31) == 0) {
            if (mirrored())
                base = atomicAdd(&m->entry_alloc, static_cast<unsigned long long>(count));
            else
                base = atomicAdd(reinterpret_cast<unsigned long long*>(const_cast<uint64_t*>(&sq->entry_alloc_idx)),
                                 static_cast<unsigned long long>(count));
        }
        return __shfl_sync(0xffffffffu, base, 0);
    }

    // Reserves `n` consecutive list slots; returns the first (warp-uniform result).
    __device__ __forceinline__ uint64_t alloc_list(uint32_t n = 1) const {
        unsigned long long slot = 0;
        if ((threadIdx.x & 31) == 0) {
            if (mirrored())
                slot = atomicAdd(&m->list_alloc, static_cast<unsigned long long>(n));
            else
                slot = atomicAdd(reinterpret_cast<unsigned long long*>(const_cast<uint64_t*>(&sq->list_alloc_idx)),
                                 static_cast<unsigned long long>(n));
        }
        return __shfl_sync(0xffffffffu, slot, 0);
    }

    // Writes a list's header (lane 0); the marker follows in publish().
    __device__ __forceinline__ void write_header(uint64_t slot, uint32_t pool_offset, uint32_t count,
                                                 uint32_t list_id, uint32_t flags) const {
        if ((threadIdx.x & 31) == 0) {
            SGList* l = &sq->lists[slot % MAX_SG_LISTS];
            l->pool_offset = pool_offset % MAX_SG_POOL_ENTRIES;
            l->count = count;
            l->list_id = list_id;
            l->flags = flags;
        }
    }

    // ---- device-entry lists (library extension; mirror mode only) ----
    // The entries go to device_pool()[(first entry) % MAX_SG_POOL_ENTRIES] and the headers
    // to the mirror (write_header_device); publish_device commits them with device-scope
    // fences only.  The lists carry SG_FLAG_DEVICE_ENTRIES; consumers of the same GPU
    // read them from device memory (SGListView included).  Null without the mirror: then
    // use the host pool, write_header and publish.
    __device__ __forceinline__ DeviceSGEntry* device_pool() const { return m != nullptr ? m->pool : nullptr; }

    // Lane 0 writes the mirror header of list `slot` whose `count` entries start at
    // absolute pool index `first_entry`.
    __device__ __forceinline__ void write_header_device(uint64_t slot, uint64_t first_entry, uint32_t count,
                                                        uint32_t list_id, uint32_t flags) const {
        if ((threadIdx.x & 31) == 0) {
            SGDeviceListHdr* h = &m->hdr[slot % MAX_SG_LISTS];
            h->pool_offset = static_cast<uint32_t>(first_entry % MAX_SG_POOL_ENTRIES);
            h->count = count;
            h->list_id = list_id;
            h->flags = flags | SG_FLAG_DEVICE_ENTRIES;
            h->first_entry = first_entry;
        }
    }

    // Commits device-entry lists [first_slot, first_slot + n): a device fence by every lane
    // (its pool and header writes), the headers' sequence words, a fence, the commit words
    // the consumers poll; then the host-visible allocation counters.
    __device__ __forceinline__ void publish_device(uint64_t first_slot, uint32_t n) const {
        const uint32_t lane = threadIdx.x & 31;
        __threadfence();
        __syncwarp();
        for (uint32_t i = lane; i < n; i += 32) m->hdr[(first_slot + i) % MAX_SG_LISTS].seq = first_slot + i + 1;
        __threadfence();
        __syncwarp();
        for (uint32_t i = lane; i < n; i += 32) m->committed[(first_slot + i) % MAX_SG_LISTS] = first_slot + i + 1;
        __threadfence();
        if (lane == 0) {
            wait::publish_max(&sq->list_alloc_idx, detail::ld_dev(&m->list_alloc));
            wait::publish_max(&sq->entry_alloc_idx, detail::ld_dev(&m->entry_alloc));
        }
        __syncwarp();
    }

    // Commits lists [first_slot, first_slot + n) whose entries and headers this warp has
    // written: one system-scope fence by every lane (each orders the entries it wrote;
    // consumers read entries and headers only after they see a marker, so one fence per
    // batch suffices -- it costs a few PCIe round trips), then the markers, then (with
    // the mirror) the host-visible allocation counters.
    __device__ __forceinline__ void publish(uint64_t first_slot, uint32_t n) const {
        __threadfence_system();
        __syncwarp();
        const uint32_t lane = threadIdx.x & 31;
        for (uint32_t i = lane; i < n; i += 32) sq->lists[(first_slot + i) % MAX_SG_LISTS].sequence = first_slot + i + 1;
        if (lane == 0 && m != nullptr) {
            wait::publish_max(&sq->list_alloc_idx, detail::ld_dev(&m->list_alloc));
            wait::publish_max(&sq->entry_alloc_idx, detail::ld_dev(&m->entry_alloc));
        }
        __syncwarp();
    }
};

// Lane 0 waits until the pool has room for `needed` more entries.
__device__ __forceinline__ void sg_wait_entry_space(SGTaskQueue* sq, uint32_t needed) {
    SGSubmitter(sq).wait_entry_space(needed);
}

// Lane 0 waits until the list ring has a free slot.
__device__ __forceinline__ void sg_wait_list_space(SGTaskQueue* sq) { SGSubmitter(sq).wait_list_space(); }

__device__ __forceinline__ uint64_t sg_alloc_entries(SGTaskQueue* sq, uint32_t count) {
    return SGSubmitter(sq).alloc_entries(count);
}

__device__ __forceinline__ void sg_write_entries(SGTaskQueue* sq, uint64_t pool_offset,
                                                 const DeviceSGEntry* src_entries, uint32_t count) {
    for (uint32_t i = threadIdx.x & 31u; i < count; i += 32)
        sq->entries[(pool_offset + i) % MAX_SG_POOL_ENTRIES] = src_entries[i];
}

__device__ __forceinline__ void sg_write_entries_inline(SGTaskQueue* sq, uint64_t pool_offset,
                                                        const uint64_t* src_addrs, const uint64_t* dst_addrs,
                                                        const uint32_t* sizes, uint32_t tag, uint32_t count) {
    for (uint32_t i = threadIdx.x & 31u; i < count; i += 32)
        sq->entries[(pool_offset + i) % MAX_SG_POOL_ENTRIES] =
            DeviceSGEntry{src_addrs[i], dst_addrs[i], sizes[i], tag};
}

__device__ __forceinline__ uint64_t sg_alloc_list(SGTaskQueue* sq) { return SGSubmitter(sq).alloc_list(); }

// Publishes one list: header, fence, marker.
__device__ __forceinline__ void sg_commit_list(SGTaskQueue* sq, uint64_t slot, uint32_t pool_offset,
                                               uint32_t count, uint32_t list_id, uint32_t flags) {
    const SGSubmitter sub(sq);
    sub.write_header(slot, pool_offset, count, list_id, flags);
    sub.publish(slot, 1);
}

__device__ __forceinline__ uint64_t sg_submit_list(SGTaskQueue* sq, const DeviceSGEntry* entries, uint32_t count,
                                                   uint32_t list_id, uint32_t flags = SG_FLAG_NONE) {
    sg_wait_entry_space(sq, count);
    sg_wait_list_space(sq);
    const uint64_t pool_offset = sg_alloc_entries(sq, count);
    sg_write_entries(sq, pool_offset, entries, count);
    const uint64_t list_slot = sg_alloc_list(sq);
    sg_commit_list(sq, list_slot, static_cast<uint32_t>(pool_offset), count, list_id, flags);
    return list_slot;
}

// Lane 0 waits until lists_completed >= expected.
__device__ __forceinline__ void sg_wait_list_done(SGTaskQueue* sq, uint64_t expected) {
    if ((threadIdx.x & 31) == 0) {
        const uint64_t t0 = wait::now();
        uint32_t polls = 0;
        while (wait::load_acquire_sys(&sq->lists_completed) < expected) {
            if (wait::expired(t0, sq->wait_limit_ns)) {
                wait::note_timeout(&sq->wait_timeouts);
                break;
            }
            wait::backoff(polls);
        }
    }
    __syncwarp();
}

// Lane 0 waits until d_list_done[list_id] != 0.
__device__ __forceinline__ void sg_wait_list_id_done(SGTaskQueue* sq, uint32_t list_id) {
    if ((threadIdx.x & 31) == 0) {
        const volatile uint64_t* sig = &sq->d_list_done[list_id];
        const uint64_t t0 = wait::now();
        uint32_t polls = 0;
        while (wait::load_acquire_sys(sig) == 0) {
            if (wait::expired(t0, sq->wait_limit_ns)) {
                wait::note_timeout(&sq->wait_timeouts);
                break;
            }
            wait::backoff(polls);
        }
    }
    __syncwarp();
}

}  // namespace sg
}  // namespace gfd
