#pragma once
// Warp-collective device primitives for the scatter-gather task queue.
//
// Same functions and protocol as the reference interface
// include/gfd/sg_device_primitives.cuh:28-243: reserve pool entries and a list slot
// with atomics, write the entries, then a three-step commit (fence, header, fence,
// marker sequence = slot + 1, fence).  Waits are bounded by sq->wait_limit_ns
// (0: GFD_DEVICE_WAIT_LIMIT_NS); a give-up increments sq->wait_timeouts.
// sg_wait_list_space additionally waits until the ring slot it will use has been
// released by the consumer (its marker is 0).

#include <cstdint>

#include "gfd/sg_task_queue.h"
#include "gfd/wait.cuh"

namespace gfd {
namespace sg {

// Lane 0 waits until the pool has room for `needed` more entries.
__device__ __forceinline__ void sg_wait_entry_space(SGTaskQueue* sq, uint32_t needed) {
    if ((threadIdx.x & 31) == 0) {
        const uint64_t t0 = wait::now();
        uint32_t polls = 0;
        for (;;) {
            const uint64_t alloc = sq->entry_alloc_idx;
            const uint64_t consumed = wait::load_acquire_sys(&sq->entry_consumed_idx);
            if (alloc - consumed <= static_cast<uint64_t>(MAX_SG_POOL_ENTRIES - needed)) break;
            if (wait::expired(t0, sq->wait_limit_ns)) {
                wait::note_timeout(&sq->wait_timeouts);
                break;
            }
            wait::backoff(polls);
        }
    }
    __syncwarp();
}

// Lane 0 waits until the list ring has a free slot.
__device__ __forceinline__ void sg_wait_list_space(SGTaskQueue* sq) {
    if ((threadIdx.x & 31) == 0) {
        const uint64_t t0 = wait::now();
        uint32_t polls = 0;
        for (;;) {
            const uint64_t alloc = sq->list_alloc_idx;
            const uint64_t read = wait::load_acquire_sys(&sq->list_read_idx);
            // the reference condition (with consumers that claimed ahead counted as no
            // backlog), plus: the slot's previous list has been released
            const uint64_t pending = alloc > read ? alloc - read : 0;
            if (pending < static_cast<uint64_t>(MAX_SG_LISTS - 1) &&
                wait::load_acquire_sys(&sq->lists[alloc % MAX_SG_LISTS].sequence) == 0)
                break;
            if (wait::expired(t0, sq->wait_limit_ns)) {
                wait::note_timeout(&sq->wait_timeouts);
                break;
            }
            wait::backoff(polls);
        }
    }
    __syncwarp();
}

__device__ __forceinline__ uint64_t sg_alloc_entries(SGTaskQueue* sq, uint32_t count) {
    unsigned long long base = 0;
    if ((threadIdx.x & 31) == 0)
        base = atomicAdd(reinterpret_cast<unsigned long long*>(const_cast<uint64_t*>(&sq->entry_alloc_idx)),
                         static_cast<unsigned long long>(count));
    return __shfl_sync(0xffffffffu, base, 0);
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

__device__ __forceinline__ uint64_t sg_alloc_list(SGTaskQueue* sq) {
    unsigned long long slot = 0;
    if ((threadIdx.x & 31) == 0)
        slot = atomicAdd(reinterpret_cast<unsigned long long*>(const_cast<uint64_t*>(&sq->list_alloc_idx)), 1ull);
    return __shfl_sync(0xffffffffu, slot, 0);
}

__device__ __forceinline__ void sg_commit_list(SGTaskQueue* sq, uint64_t slot, uint32_t pool_offset,
                                               uint32_t count, uint32_t list_id, uint32_t flags) {
    SGList* l = &sq->lists[slot % MAX_SG_LISTS];
    __threadfence_system();  // entries before the header
    __syncwarp();
    if ((threadIdx.x & 31) == 0) {
        l->pool_offset = pool_offset % MAX_SG_POOL_ENTRIES;
        l->count = count;
        l->list_id = list_id;
        l->flags = flags;
    }
    __syncwarp();
    __threadfence_system();  // header before the marker
    __syncwarp();
    if ((threadIdx.x & 31) == 0) l->sequence = slot + 1;
    __threadfence_system();
    __syncwarp();
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
