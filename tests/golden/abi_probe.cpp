// Prints the size and field offsets of the host<->GPU wire structs as JSON.
// Compiled twice by tests/golden/make_golden.py / tests/test_abi.py: once against the
// reference headers (to make abi_layout.json) and once against include/gfd.
#include <cstddef>
#include <cstdio>
#include "gfd/descriptor_queue.h"
#include "gfd/tiled_queue.h"
#include "gfd/sg_task_queue.h"
#include "gfd/copy_engine.h"

#define F(T, f) printf("  \"" #T "." #f "\": %zu,\n", offsetof(T, f))
#define S(T) printf("  \"sizeof(" #T ")\": %zu,\n", sizeof(T))
#define A(T) printf("  \"alignof(" #T ")\": %zu,\n", alignof(T))

int main() {
    using namespace gfd;
    printf("{\n");
    S(Descriptor); A(Descriptor);
    F(Descriptor, src_addr); F(Descriptor, dst_addr); F(Descriptor, size); F(Descriptor, flags);
    F(Descriptor, user_data); F(Descriptor, sequence);
    S(DescriptorQueue); A(DescriptorQueue);
    F(DescriptorQueue, entries); F(DescriptorQueue, write_idx); F(DescriptorQueue, read_idx);
    F(DescriptorQueue, done_idx);
    S(TokenInfo); F(TokenInfo, cpu_addr); F(TokenInfo, token_id); F(TokenInfo, expert_id);
    S(TileScheduler); A(TileScheduler);
    F(TileScheduler, next_tile); F(TileScheduler, total_tiles); F(TileScheduler, tokens_per_tile);
    F(TileScheduler, tokens_per_chunk); F(TileScheduler, chunks_per_tile); F(TileScheduler, token_size);
    S(TiledQueue); A(TiledQueue);
    F(TiledQueue, base); F(TiledQueue, scheduler); F(TiledQueue, tile_chunk_done);
    F(TiledQueue, d_tile_chunk_done);
    S(DeviceSGEntry); A(DeviceSGEntry);
    F(DeviceSGEntry, src_addr); F(DeviceSGEntry, dst_addr); F(DeviceSGEntry, size); F(DeviceSGEntry, tag);
    S(SGList); A(SGList);
    F(SGList, pool_offset); F(SGList, count); F(SGList, list_id); F(SGList, flags); F(SGList, sequence);
    S(SGTaskQueue); A(SGTaskQueue);
    F(SGTaskQueue, lists); F(SGTaskQueue, entries); F(SGTaskQueue, list_alloc_idx);
    F(SGTaskQueue, entry_alloc_idx); F(SGTaskQueue, list_read_idx); F(SGTaskQueue, entry_consumed_idx);
    F(SGTaskQueue, lists_completed); F(SGTaskQueue, terminate); F(SGTaskQueue, d_list_done);
    S(SGEntry); F(SGEntry, dst); F(SGEntry, src); F(SGEntry, size);
    printf("  \"QUEUE_SIZE\": %d,\n  \"MAX_BATCH_SIZE\": %d,\n  \"BATCH_THRESHOLD\": %d,\n",
           QUEUE_SIZE, MAX_BATCH_SIZE, BATCH_THRESHOLD);
    printf("  \"BATCH_THRESHOLD_SMALL\": %d,\n  \"MAX_TILES\": %d,\n  \"MAX_SG_LISTS\": %d,\n",
           BATCH_THRESHOLD_SMALL, MAX_TILES, MAX_SG_LISTS);
    printf("  \"MAX_SG_POOL_ENTRIES\": %d,\n  \"FLAG_LAST_IN_BATCH\": %u,\n  \"FLAG_URGENT\": %u,\n",
           MAX_SG_POOL_ENTRIES, FLAG_LAST_IN_BATCH, FLAG_URGENT);
    printf("  \"FLAG_LAST_IN_TILE\": %u,\n  \"FLAG_LAST_CHUNK_IN_TILE\": %u,\n",
           FLAG_LAST_IN_TILE, FLAG_LAST_CHUNK_IN_TILE);
    printf("  \"SG_FLAG_HOST_SUBMITTED\": %u,\n  \"MAX_CE_CHANNELS\": %d,\n  \"MAX_SG_ENTRIES_PER_BATCH\": %d\n}\n",
           SG_FLAG_HOST_SUBMITTED, MAX_CE_CHANNELS, MAX_SG_ENTRIES_PER_BATCH);
    return 0;
}
