#pragma once
// Tile scheduling block and per-tile completion counters for warp-specialised
// transfer/compute kernels.
//
// Byte-compatible with the reference interface include/gfd/tiled_queue.h:8-43.
// TileScheduler keeps its six named fields at the same offsets; this library
// stores its own launch parameters in the reference's 40 padding bytes
// (producer warp count, compute sets, wait limit, stats pointer, optional block
// table), which the reference never reads, so sizeof and every named offset are
// unchanged.

#include "gfd/descriptor_queue.h"
#include <cstdint>

namespace gfd {

constexpr int MAX_TILES = 1024;
constexpr uint32_t FLAG_LAST_IN_TILE = 4;        // last descriptor of a chunk
constexpr uint32_t FLAG_LAST_CHUNK_IN_TILE = 8;  // last descriptor of a tile

// Counters the framework kernels accumulate (device memory, owned by a session).
struct TransferStats {
    unsigned long long tokens;     // tokens (or SG entries) landed
    unsigned long long bytes;      // payload bytes landed
    unsigned long long timeouts;   // bounded waits that gave up
    unsigned long long rejected;   // page-table ids outside the source pool (tokens skipped)
};

struct alignas(64) TileScheduler {
    volatile uint32_t next_tile;   // atomicAdd by CTAs to claim a tile
    uint32_t total_tiles;
    uint32_t tokens_per_tile;
    uint32_t tokens_per_chunk;
    uint32_t chunks_per_tile;
    uint32_t token_size;
    // ---- library extension inside the reference's padding ----
    uint32_t producer_warps;       // warps per CTA that pull (0 means 1)
    uint32_t compute_sets;         // 1 = single buffer, 2 = double buffer
    uint64_t wait_limit_ns;        // bound on every in-kernel wait (0 = default)
    TransferStats* stats;          // device counters (may be null)
    const uint32_t* block_table;   // device array: token g reads block block_table[g] (null: linear)
    uint32_t table_blocks;         // blocks in the source pool; larger ids are rejected
    uint8_t _pad[64 - 24 - 8 - 8 - 8 - 8 - 4];
};

static_assert(sizeof(TileScheduler) == 64, "TileScheduler is 64 bytes");
static_assert(offsetof(TileScheduler, next_tile) == 0, "layout");
static_assert(offsetof(TileScheduler, total_tiles) == 4, "layout");
static_assert(offsetof(TileScheduler, tokens_per_tile) == 8, "layout");
static_assert(offsetof(TileScheduler, tokens_per_chunk) == 12, "layout");
static_assert(offsetof(TileScheduler, chunks_per_tile) == 16, "layout");
static_assert(offsetof(TileScheduler, token_size) == 20, "layout");

struct TiledQueue {
    DescriptorQueue base;
    TileScheduler scheduler;
    volatile uint64_t tile_chunk_done[MAX_TILES];  // cumulative tokens landed per tile
    uint64_t* d_tile_chunk_done;                   // device copy of the same counters
};

static_assert(offsetof(TiledQueue, scheduler) == sizeof(DescriptorQueue), "layout");
static_assert(offsetof(TiledQueue, tile_chunk_done) == sizeof(DescriptorQueue) + 64, "layout");
static_assert(offsetof(TiledQueue, d_tile_chunk_done) ==
              sizeof(DescriptorQueue) + 64 + 8 * MAX_TILES, "layout");

}  // namespace gfd
