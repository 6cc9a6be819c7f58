#pragma once
// Device-side producer API for GPU-queued submission.
//
// Same functions, arguments and ring protocol as the reference interface
// include/gfd/device.cuh:47-176: a thread writes the descriptor of its token into
// slot base_slot + token_idx, the warp fences at system scope and then stores the
// commit marker sequence = slot + 1; waiters poll done_idx.  In this library the
// ring is consumed by the ring agent, a device-resident kernel (gfd_b200/csrc/agent.cu),
// which publishes done_idx only after the bytes have landed in HBM.
//
// Differences: every thread fences its own descriptor before storing its marker
// (the reference fences only from the warp leader), and wait_for_completion gives
// up after GFD_DEVICE_WAIT_LIMIT_NS (default 10 s) instead of spinning forever; a
// give-up increments queue->wait_timeouts (host-visible).  wait_for_completion_until
// returns whether the wait succeeded.

#include <cstdint>

#include "gfd/descriptor_queue.h"
#include "gfd/wait.cuh"

namespace gfd {
namespace device {

__device__ __forceinline__ void write_descriptor(DescriptorQueue* queue, uint64_t base_slot, int token_idx,
                                                 uint64_t src_addr, void* gpu_dst, uint32_t token_size,
                                                 int num_tokens, uint64_t user_data = 0) {
    const uint64_t slot = base_slot + static_cast<uint64_t>(token_idx);
    Descriptor* d = &queue->entries[slot % QUEUE_SIZE];
    d->src_addr = src_addr;
    d->dst_addr = reinterpret_cast<uint64_t>(gpu_dst) + static_cast<uint64_t>(token_idx) * token_size;
    d->size = token_size;
    d->flags = (token_idx == num_tokens - 1) ? FLAG_LAST_IN_BATCH : FLAG_NONE;
    d->user_data = user_data;
}

// Publishes this thread's descriptor (active == true) with the commit marker.
__device__ __forceinline__ void fence_and_commit(DescriptorQueue* queue, uint64_t base_slot, int token_idx,
                                                 bool active) {
    __threadfence_system();  // descriptor fields before the marker, on every lane
    __syncwarp();
    if (active) {
        const uint64_t slot = base_slot + static_cast<uint64_t>(token_idx);
        queue->entries[slot % QUEUE_SIZE].sequence = slot + 1;
    }
    __threadfence_system();  // marker out to the consumer
}

// Waits until done_idx >= expected_done or the time limit passes; true on success.
// Polls the device-memory mirror of done_idx when the consumer keeps one (many CTAs
// polling host memory throttle the consumer's own pulls) and confirms with one read of
// the host field, which stays the authority.
__device__ __forceinline__ bool wait_for_completion_until(DescriptorQueue* queue, uint64_t expected_done,
                                                          uint64_t limit_ns) {
    const QueueMirror* m = queue->mirror;
    const uint64_t t0 = wait::now();
    uint32_t polls = 0;
    for (;;) {
        const uint64_t d = m != nullptr ? m->done_idx : wait::load_acquire_sys(&queue->done_idx);
        if (d >= expected_done && (m == nullptr || wait::load_acquire_sys(&queue->done_idx) >= expected_done))
            return true;
        if (wait::expired(t0, limit_ns)) {
            wait::note_timeout(&queue->wait_timeouts);
            return false;
        }
        wait::backoff(polls);
    }
}

// One thread waits (then __syncthreads() to broadcast), as in the reference.
__device__ __forceinline__ void wait_for_completion(DescriptorQueue* queue, uint64_t expected_done) {
    wait_for_completion_until(queue, expected_done, GFD_DEVICE_WAIT_LIMIT_NS);
}

// Writes only if the slot is free (marker 0); false when the ring is full there.
__device__ __forceinline__ bool write_descriptor_safe(DescriptorQueue* queue, uint64_t base_slot, int token_idx,
                                                      uint64_t src_addr, void* gpu_dst, uint32_t token_size,
                                                      int num_tokens, uint64_t user_data = 0) {
    const uint64_t slot = base_slot + static_cast<uint64_t>(token_idx);
    if (queue->entries[slot % QUEUE_SIZE].sequence != 0) return false;
    write_descriptor(queue, base_slot, token_idx, src_addr, gpu_dst, token_size, num_tokens, user_data);
    return true;
}

__device__ __forceinline__ void write_and_commit(DescriptorQueue* queue, uint64_t base_slot, int token_idx,
                                                 bool active, uint64_t src_addr, void* gpu_dst,
                                                 uint32_t token_size, int num_tokens, uint64_t user_data = 0) {
    if (active) write_descriptor(queue, base_slot, token_idx, src_addr, gpu_dst, token_size, num_tokens, user_data);
    fence_and_commit(queue, base_slot, token_idx, active);
}

}  // namespace device
}  // namespace gfd
