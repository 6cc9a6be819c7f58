#pragma once
// Tile-level device primitives for hand-written warp-specialised kernels.
//
// Same functions and semantics as the reference interface
// include/gfd/device_primitives.cuh:24-209: tile claiming, chunk slot reservation,
// chunk / tile descriptor writing with FLAG_LAST_IN_TILE / FLAG_LAST_CHUNK_IN_TILE
// markers and user_data = (tile << 32) | global token index, two-phase commit, and
// waits on the cumulative per-tile counter.  Descriptors written here are drained
// by the library's GPU ring consumer, which adds each landed token to
// d_tile_chunk_done[tile] (or tile_chunk_done[tile] when no device copy exists).
//
// The waits (wait_chunk_done, wait_queue_space) are bounded by
// tq->scheduler.wait_limit_ns (0: GFD_DEVICE_WAIT_LIMIT_NS); a give-up increments
// tq->base.wait_timeouts and the function returns.  The _until variants report it.

#include <cstdint>

#include "gfd/tiled_queue.h"
#include "gfd/wait.cuh"

namespace gfd {
namespace device {

__device__ __forceinline__ uint32_t acquire_tile(TiledQueue* tq) {
    return atomicAdd(const_cast<uint32_t*>(&tq->scheduler.next_tile), 1u);
}

// Warp-collective: lane 0 reserves `count` consecutive slots; all lanes get the base.
__device__ __forceinline__ uint64_t acquire_chunk_slots(TiledQueue* tq, uint32_t count) {
    unsigned long long base = 0;
    if ((threadIdx.x & 31) == 0)
        base = atomicAdd(reinterpret_cast<unsigned long long*>(const_cast<uint64_t*>(&tq->base.write_idx)),
                         static_cast<unsigned long long>(count));
    return __shfl_sync(0xffffffffu, base, 0);
}

__device__ __forceinline__ void fill_tile_descriptor(TiledQueue* tq, uint64_t slot, uint32_t tile_id,
                                                     uint32_t global_idx, const void* cpu_base, void* gpu_base,
                                                     uint32_t token_size, uint32_t flags) {
    Descriptor* d = &tq->base.entries[slot % QUEUE_SIZE];
    const uint64_t off = static_cast<uint64_t>(global_idx) * token_size;
    d->src_addr = reinterpret_cast<uint64_t>(cpu_base) + off;
    d->dst_addr = reinterpret_cast<uint64_t>(gpu_base) + off;
    d->size = token_size;
    d->user_data = (static_cast<uint64_t>(tile_id) << 32) | global_idx;
    d->flags = flags;
}

// Warp-collective: descriptors of chunk `chunk_id` of tile `tile_id` (linear mapping).
__device__ __forceinline__ void write_chunk(TiledQueue* tq, uint64_t slot_base, uint32_t tile_id,
                                            uint32_t chunk_id, uint32_t tokens_per_chunk,
                                            uint32_t tokens_per_tile, const void* cpu_base, void* gpu_base,
                                            uint32_t token_size) {
    const uint32_t C = tokens_per_chunk;
    const uint32_t K = tokens_per_tile / C;
    for (uint32_t i = threadIdx.x & 31u; i < C; i += 32) {
        uint32_t flags = FLAG_NONE;
        if (i == C - 1) {
            flags |= FLAG_LAST_IN_TILE;
            if (chunk_id == K - 1) flags |= FLAG_LAST_CHUNK_IN_TILE;
        }
        const uint32_t global_idx = tile_id * tokens_per_tile + chunk_id * C + i;
        fill_tile_descriptor(tq, slot_base + i, tile_id, global_idx, cpu_base, gpu_base, token_size, flags);
    }
}

// Warp-collective two-phase commit of `count` slots from slot_base.
__device__ __forceinline__ void commit_chunk(TiledQueue* tq, uint64_t slot_base, uint32_t count) {
    __threadfence_system();
    __syncwarp();
    for (uint32_t i = threadIdx.x & 31u; i < count; i += 32) {
        const uint64_t slot = slot_base + i;
        tq->base.entries[slot % QUEUE_SIZE].sequence = slot + 1;
    }
    __threadfence_system();
    __syncwarp();
}

// One thread: waits until the tile's cumulative landed-token count reaches expected.
__device__ __forceinline__ bool wait_chunk_done_until(TiledQueue* tq, uint32_t tile_id, uint64_t expected,
                                                      uint64_t limit_ns) {
    const volatile uint64_t* sig = tq->d_tile_chunk_done ? &tq->d_tile_chunk_done[tile_id]
                                                         : &tq->tile_chunk_done[tile_id];
    const uint64_t t0 = wait::now();
    uint32_t polls = 0;
    while (wait::load_acquire_sys(sig) < expected) {
        if (wait::expired(t0, limit_ns)) {
            wait::note_timeout(&tq->base.wait_timeouts);
            return false;
        }
        wait::backoff(polls);
    }
    return true;
}

__device__ __forceinline__ void wait_chunk_done(TiledQueue* tq, uint32_t tile_id, uint64_t expected) {
    wait_chunk_done_until(tq, tile_id, expected, tq->scheduler.wait_limit_ns);
}

// Warp-collective: lane 0 waits until at least 2 * needed slots are free.
__device__ __forceinline__ void wait_queue_space(TiledQueue* tq, uint32_t needed) {
    if ((threadIdx.x & 31) == 0) {
        const QueueMirror* m = tq->base.mirror;
        const uint64_t t0 = wait::now();
        uint32_t polls = 0;
        uint64_t seen = ~0ull, w = 0;
        for (;;) {
            // the mirror never runs ahead of the host read_idx, so a slot it shows free
            // is free; write_idx (host) is re-read only when the consumer has moved
            uint64_t r = m != nullptr ? m->read_idx : wait::load_acquire_sys(&tq->base.read_idx);
            if (r != seen) {
                w = tq->base.write_idx;
                seen = r;
            }
            if (m != nullptr && r > w) r = wait::load_acquire_sys(&tq->base.read_idx);  // indices were reset
            if (w - r < static_cast<uint64_t>(QUEUE_SIZE) - 2ull * needed) break;
            if (wait::expired(t0, tq->scheduler.wait_limit_ns)) {
                wait::note_timeout(&tq->base.wait_timeouts);
                break;
            }
            wait::backoff(polls);
        }
    }
    __syncwarp();
}

__device__ __forceinline__ void submit_chunk(TiledQueue* tq, uint64_t slot_base, uint32_t tile_id,
                                             uint32_t chunk_id, uint32_t tokens_per_chunk,
                                             uint32_t tokens_per_tile, const void* cpu_base, void* gpu_base,
                                             uint32_t token_size) {
    write_chunk(tq, slot_base, tile_id, chunk_id, tokens_per_chunk, tokens_per_tile, cpu_base, gpu_base,
                token_size);
    commit_chunk(tq, slot_base, tokens_per_chunk);
}

// Warp-collective: all T descriptors of a tile in one reservation + one commit.
__device__ __forceinline__ void submit_tile(TiledQueue* tq, uint64_t slot_base, uint32_t tile_id, uint32_t T,
                                            uint32_t C, const void* cpu_base, void* gpu_base,
                                            uint32_t token_size) {
    for (uint32_t i = threadIdx.x & 31u; i < T; i += 32) {
        uint32_t flags = FLAG_NONE;
        if (i % C == C - 1) flags |= FLAG_LAST_IN_TILE;
        if (i == T - 1) flags |= FLAG_LAST_CHUNK_IN_TILE;
        fill_tile_descriptor(tq, slot_base + i, tile_id, tile_id * T + i, cpu_base, gpu_base, token_size, flags);
    }
    commit_chunk(tq, slot_base, T);
}

}  // namespace device
}  // namespace gfd
