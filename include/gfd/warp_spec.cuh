#pragma once
// Warp-specialised transfer + compute framework for linear tiles.
//
// Same user contract as the reference interface include/gfd/warp_spec.cuh:41-469:
// a compute functor with __device__ void operator()(gfd::warp_spec::ChunkView), the
// kernel macros GFD_WARP_SPEC_KERNEL / GFD_WARP_SPEC_KERNEL_DB, the kernel
// signature (TiledQueue*, void* gpu_buffer, const void* cpu_base, ComputeFn), tile
// claiming through tq->scheduler.next_tile, tile t covering tokens
// [t*T, (t+1)*T) at cpu_base / gpu_buffer + index * token_size, chunk k of a tile
// handed to compute warp k (in DB mode: two compute sets take alternate tiles).
// Tail tokens beyond total_tiles * T are not transferred, as in the reference.
//
// Page-table mode (library addition: a paged-KV block table turned straight into pull
// work, with no descriptors in between): when tq->scheduler.block_table is set, token g is read from
// cpu_base + block_table[g] * token_size instead of cpu_base + g * token_size; it still
// lands at gpu_buffer + g * token_size, so the functor's ChunkView is unchanged.
//
// B200 mechanism: no descriptors and no CPU poller.  The first P warps of the CTA
// are producers; they claim a tile and pull its chunks straight from pinned host
// memory into gpu_buffer (16-byte loads, U in flight per thread, gfd/pull.cuh),
// publishing "chunk c landed" in shared memory after a named barrier.  Compute
// warps wait on that flag and run the functor on data that is already in HBM.
// Because every tile has its own region of gpu_buffer, producers never wait for
// compute to free a buffer: they run up to kTileSlots tiles ahead, so the pull of
// tile i+1.. overlaps the compute of tile i.  P = warps in the block minus the
// compute warps (K, or 2K in DB mode), so the reference launch shape (one transfer
// warp) also works; WarpSpecSession launches P = 4 by default.
// Every wait is bounded by scheduler.wait_limit_ns (0: GFD_DEVICE_WAIT_LIMIT_NS); a
// give-up increments tq->base.wait_timeouts and makes the whole CTA wind down.

#include <cstdint>

#include "gfd/device_primitives.cuh"
#include "gfd/pull.cuh"
#include "gfd/wait.cuh"

namespace gfd {
namespace warp_spec {

constexpr int MAX_CHUNKS_PER_TILE = 16;

struct ChunkView {
    void* base_ptr;                // first token of the chunk in GPU memory
    uint32_t token_size;
    uint32_t size;                 // tokens in the chunk
    uint32_t tile_id;
    uint32_t chunk_id;
    uint32_t global_token_offset;  // global index of the chunk's first token
    int lane_id;

    template <typename T>
    __device__ __forceinline__ T* data(int local_token_idx) const {
        return reinterpret_cast<T*>(static_cast<char*>(base_ptr) +
                                    static_cast<uint64_t>(local_token_idx) * token_size);
    }
    __device__ __forceinline__ int global_idx(int local_token_idx) const {
        return static_cast<int>(global_token_offset) + local_token_idx;
    }
};

struct TileContext {
    uint32_t tile_id;
    uint32_t tokens_per_tile;
    uint32_t chunks_per_tile;
    uint32_t tokens_per_chunk;
    void* tile_base_ptr;
    uint32_t token_size;

    __device__ __forceinline__ ChunkView get_chunk(int chunk_id) const {
        ChunkView v;
        v.base_ptr = static_cast<char*>(tile_base_ptr) +
                     static_cast<uint64_t>(chunk_id) * tokens_per_chunk * token_size;
        v.token_size = token_size;
        v.size = tokens_per_chunk;
        v.tile_id = tile_id;
        v.chunk_id = static_cast<uint32_t>(chunk_id);
        v.global_token_offset = tile_id * tokens_per_tile + chunk_id * tokens_per_chunk;
        v.lane_id = static_cast<int>(threadIdx.x & 31);
        return v;
    }
};

// Reference shared-state layouts, kept for code that names them.
struct _WarpSpecState {
    uint32_t tile_id;
    volatile int chunks_ready;
    volatile int compute_done;
};
struct _WarpSpecStateDB {
    uint32_t tile_id[2];
    volatile int chunks_ready[2];
    volatile int compute_done[2];
    volatile int active_slot;
    volatile int tiles_dispatched;
};

// ---------------------------------------------------------------------------
constexpr int kTileSlots = 4;
constexpr uint32_t kSlotEmpty = 0xffffffffu;
constexpr uint32_t kTileEnd = 0xffffffffu;

struct _TileSlot {
    volatile uint32_t seq;    // local tile number held, kSlotEmpty when free
    volatile uint32_t tile;   // global tile id (kTileEnd: no more tiles)
    volatile uint32_t ready;  // chunks landed
    uint32_t done;            // compute warps finished with this tile
};

struct _TilePipe {
    _TileSlot slot[kTileSlots];
    volatile uint32_t abort;
    volatile uint32_t tile_bcast;
};

__device__ __forceinline__ void _producer_bar(uint32_t threads) {
    asm volatile("bar.sync 1, %0;" ::"r"(threads) : "memory");
}

// Bounded wait on a shared-memory condition; false if the pipe aborted or timed out.
template <typename Pred>
__device__ __forceinline__ bool _pipe_wait(volatile uint32_t* abort, Pred pred, uint64_t limit_ns,
                                           TiledQueue* tq) {
    const uint64_t t0 = wait::now();
    uint32_t polls = 0;
    while (!pred()) {
        if (*abort) return false;
        if (wait::expired(t0, limit_ns)) {
            *abort = 1;
            wait::note_timeout(&tq->base.wait_timeouts);
            if (tq->scheduler.stats) atomicAdd(&tq->scheduler.stats->timeouts, 1ull);
            return false;
        }
        wait::backoff(polls);
    }
    return true;
}

template <typename ComputeFn>
__device__ void _warp_spec_run(TiledQueue* tq, void* gpu_buffer, const void* cpu_base, ComputeFn& compute_fn,
                               uint32_t sets) {
    __shared__ _TilePipe pipe;
    const uint32_t warp = threadIdx.x >> 5;
    const uint32_t lane = threadIdx.x & 31;
    const uint32_t nwarps = blockDim.x >> 5;
    const uint32_t C = tq->scheduler.tokens_per_chunk;
    const uint32_t K = tq->scheduler.chunks_per_tile;
    const uint32_t T = tq->scheduler.tokens_per_tile;
    const uint32_t total = tq->scheduler.total_tiles;
    const uint32_t token_size = tq->scheduler.token_size;
    const uint64_t limit = tq->scheduler.wait_limit_ns;
    TransferStats* stats = tq->scheduler.stats;
    const uint32_t* table = tq->scheduler.block_table;
    const uint32_t nblocks = tq->scheduler.table_blocks;
    const int producers = static_cast<int>(nwarps) - static_cast<int>(sets * K);

    if (threadIdx.x < kTileSlots) {
        pipe.slot[threadIdx.x].seq = kSlotEmpty;
        pipe.slot[threadIdx.x].tile = kTileEnd;
        pipe.slot[threadIdx.x].ready = 0;
        pipe.slot[threadIdx.x].done = 0;
    }
    if (threadIdx.x == 0) pipe.abort = (producers < 1 || K == 0 || C == 0) ? 1u : 0u;
    __syncthreads();
    if (pipe.abort) {
        if (threadIdx.x == 0) wait::note_timeout(&tq->base.wait_timeouts);  // launch shape mismatch
        return;
    }

    if (warp < static_cast<uint32_t>(producers)) {
        // ---------------- producers ----------------
        const uint32_t pt = threadIdx.x;
        const uint32_t np = static_cast<uint32_t>(producers) * 32u;
        char* gbase = static_cast<char*>(gpu_buffer);
        const char* hbase = static_cast<const char*>(cpu_base);
        for (uint32_t j = 0;; ++j) {
            _TileSlot& s = pipe.slot[j % kTileSlots];
            if (pt == 0) {
                uint32_t tile = kTileEnd;
                if (_pipe_wait(&pipe.abort, [&] { return s.seq == kSlotEmpty; }, limit, tq)) {
                    tile = device::acquire_tile(tq);
                    if (tile >= total) tile = kTileEnd;
                }
                pipe.tile_bcast = tile;
            }
            _producer_bar(np);
            const uint32_t tile = pipe.tile_bcast;
            _producer_bar(np);
            if (tile == kTileEnd) {
                if (pt == 0 && !pipe.abort) {
                    // wake every compute set with an end marker on its next slot
                    for (uint32_t e = 0; e < sets; ++e) {
                        _TileSlot& se = pipe.slot[(j + e) % kTileSlots];
                        if (!_pipe_wait(&pipe.abort, [&] { return se.seq == kSlotEmpty; }, limit, tq)) break;
                        se.tile = kTileEnd;
                        se.ready = K;
                        se.done = 0;
                        __threadfence_block();
                        se.seq = j + e;
                    }
                }
                break;
            }
            if (pt == 0) {
                s.tile = tile;
                s.ready = 0;
                s.done = 0;
                __threadfence_block();
                s.seq = j;
            }
            const uint64_t chunk_bytes = static_cast<uint64_t>(C) * token_size;
            for (uint32_t c = 0; c < K; ++c) {
                const uint64_t g0 = static_cast<uint64_t>(tile) * T + static_cast<uint64_t>(c) * C;
                const uint64_t off = g0 * token_size;
                if (table == nullptr) {
                    pull::group_copy(gbase + off, hbase + off, chunk_bytes, pt, np);
                } else {
                    // gather: producer warp w moves tokens w, w + P, ... of the chunk.  Ids
                    // are checked here, on every launch, so the table may be rewritten on the
                    // device between launches; a token with a bad id is skipped and counted.
                    const uint32_t pw = pt >> 5;
                    for (uint32_t i = pw; i < C; i += static_cast<uint32_t>(producers)) {
                        const uint32_t blk = table[g0 + i];
                        if (blk >= nblocks) {
                            if ((pt & 31u) == 0 && stats != nullptr) atomicAdd(&stats->rejected, 1ull);
                            continue;
                        }
                        pull::warp_copy(gbase + off + static_cast<uint64_t>(i) * token_size,
                                        hbase + static_cast<uint64_t>(blk) * token_size, token_size);
                    }
                }
                _producer_bar(np);
                if (pt == 0) {
                    __threadfence_block();
                    s.ready = c + 1;
                }
            }
            if (pt == 0 && stats != nullptr) {
                atomicAdd(&stats->tokens, static_cast<unsigned long long>(T));
                atomicAdd(&stats->bytes, static_cast<unsigned long long>(T) * token_size);
            }
            if (pipe.abort) break;
        }
    } else {
        // ---------------- compute warps ----------------
        const uint32_t w = warp - static_cast<uint32_t>(producers);
        const uint32_t set = w / K;
        const uint32_t k = w % K;
        for (uint32_t j = set;; j += sets) {
            _TileSlot& s = pipe.slot[j % kTileSlots];
            int ok = 1;
            if (lane == 0) ok = _pipe_wait(&pipe.abort, [&] { return s.seq == j; }, limit, tq);
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) break;
            const uint32_t tile = s.tile;
            if (tile == kTileEnd) break;
            if (lane == 0) ok = _pipe_wait(&pipe.abort, [&] { return s.ready > k; }, limit, tq);
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) break;
            __threadfence_block();
            ChunkView v;
            v.base_ptr = static_cast<char*>(gpu_buffer) +
                         (static_cast<uint64_t>(tile) * T + static_cast<uint64_t>(k) * C) * token_size;
            v.token_size = token_size;
            v.size = C;
            v.tile_id = tile;
            v.chunk_id = k;
            v.global_token_offset = tile * T + k * C;
            v.lane_id = static_cast<int>(lane);
            compute_fn(v);
            __syncwarp();
            if (lane == 0) {
                __threadfence_block();
                if (atomicAdd(&s.done, 1u) + 1u == K) s.seq = kSlotEmpty;
            }
        }
    }
}

// Reference entry points (names kept): single buffer and double buffer.
template <typename ComputeFn>
__device__ void _warp_spec_tile_loop(TiledQueue* tq, void* gpu_buffer, const void* cpu_base, ComputeFn compute_fn) {
    _warp_spec_run(tq, gpu_buffer, cpu_base, compute_fn, 1u);
}

template <typename ComputeFn>
__device__ void _warp_spec_tile_loop_double_buffer(TiledQueue* tq, void* gpu_buffer, const void* cpu_base,
                                                   ComputeFn compute_fn) {
    _warp_spec_run(tq, gpu_buffer, cpu_base, compute_fn, 2u);
}

}  // namespace warp_spec
}  // namespace gfd

// Kernels are compiled for blocks of up to GFD_WARP_SPEC_MAX_THREADS threads (define it
// before including this header to change it): 640 covers the default 4 producer warps
// plus two compute sets of 8 warps.  The sessions refuse a launch shape above the
// kernel's limit instead of launching it.
#ifndef GFD_WARP_SPEC_MAX_THREADS
#define GFD_WARP_SPEC_MAX_THREADS 640
#endif

#define GFD_WARP_SPEC_KERNEL(kernel_name, ComputeFnType)                                          \
    __global__ void __launch_bounds__(GFD_WARP_SPEC_MAX_THREADS)                                 \
        kernel_name(gfd::TiledQueue* tq, void* gpu_buffer, const void* cpu_base,                 \
                    ComputeFnType compute_fn) {                                                  \
        gfd::warp_spec::_warp_spec_tile_loop(tq, gpu_buffer, cpu_base, compute_fn);              \
    }

#define GFD_WARP_SPEC_KERNEL_DB(kernel_name, ComputeFnType)                                       \
    __global__ void __launch_bounds__(GFD_WARP_SPEC_MAX_THREADS)                                 \
        kernel_name(gfd::TiledQueue* tq, void* gpu_buffer, const void* cpu_base,                 \
                    ComputeFnType compute_fn) {                                                  \
        gfd::warp_spec::_warp_spec_tile_loop_double_buffer(tq, gpu_buffer, cpu_base, compute_fn); \
    }
