#pragma once
// Ring agent: the device-resident consumer of the GPU-written descriptor ring
// (GPU-queued submit).  Shared by the kernel (agent.cu) and its host side (ring.cu).
//
// One launch = 1 front CTA + `movers` mover CTAs, all resident at once:
//   front   polls the commit markers (one warp), copies each committed run of
//           descriptors out of the ring, clears their markers, advances read_idx,
//           validates every descriptor against cached ranges, counts per-tile tokens
//           and landed lists, merges contiguous descriptors into rows (block scan) and
//           publishes the run as a batch (up to kAgentSlots batches in flight);
//   movers  pull each batch's bytes (the pull kernel's body), and the last mover to
//           finish a batch applies its tile counts / list flags and publishes done_idx.
// A range the front has not seen yet is checked once by the host through a mailbox in
// pinned memory (the driver knows which allocations exist); the answer is cached in
// device memory for the rest of the launch.  The launch ends when stop is requested
// (after draining what is committed), after `linger_ns` with nothing committed (so
// that cudaDeviceSynchronize in the application returns), or -- in resident mode --
// after idle_limit_ns; the host relaunches it when the next marker is committed.
// Replaces the reference's CPU poller and batch processor (src/cpu_polling.cpp:337-436,
// src/batch_processor.cpp:69-831).

#include <cuda_runtime.h>

#include <cstdint>

#include "gfd/descriptor_queue.h"
#include "internal.h"

namespace gfdb {

constexpr int kAgentThreads = kPullThreads;      // the pull body assumes 8 warps
constexpr int kAgentMaxMovers = 32;
constexpr int kAgentDefaultMovers = 8;
constexpr uint32_t kAgentBatchMax = 8192;        // descriptors per batch (reference MAX_BATCH_SIZE)
constexpr uint32_t kAgentEagerBatch = 512;       // batch cap while the movers are idle
constexpr int kAgentSlots = 3;                   // batches in flight
constexpr int kAgentRanges = 128;                // cached validated ranges per kind
constexpr uint32_t kAgentTile = 1024;            // descriptors the front stages at a time
constexpr uint32_t kAgentMaxQueries = 64;        // mailbox queries per staged tile

struct AgentRanges {
    uint64_t lo[kAgentRanges];
    uint64_t hi[kAgentRanges];
    uint32_t n;
    uint32_t evict;  // next slot to replace once the table is full
};

struct AgentBatch {
    uint64_t begin, end;      // ring slots [begin, end)
    uint64_t total, per_cta;  // aligned stream bytes, stream bytes per mover
    uint32_t n_rows, n_misc;
    uint32_t n_tiles, n_lists, lists_landed;
    uint32_t ctas_done;       // movers finished with this batch
    uint32_t cta_first[kAgentMaxMovers];
    uint16_t tile_id[kEpiTiles];
    uint32_t tile_count[kEpiTiles];
    uint16_t list_id[kEpiLists];
    PullRow rows[kAgentBatchMax];
    PullRow misc[kAgentBatchMax];
};

// Device memory owned by the ring.  The launch counters (gen .. left) are zero when a
// launch starts: the front of the previous launch resets them once every mover has left
// (AgentHost::reset_ok), otherwise the host clears them on the ring's stream.  The host
// uploads the range tables before a launch when they changed.
struct AgentDev {
    AgentRanges src;     // pinned host sources
    AgentRanges dst;     // device destinations
    uint32_t gen;        // batches published in this launch
    uint32_t done;       // batches completed in this launch
    uint32_t exit;       // front -> movers: leave
    uint32_t started;    // CTAs running in this launch
    uint32_t left;       // movers that have left this launch
    uint32_t _pad;
    unsigned long long consumed;  // descriptors completed (all launches)
    unsigned long long batches;   // batches completed (all launches)
    AgentBatch batch[kAgentSlots];
};

// Control block in pinned, device-mapped host memory.
struct AgentHost {
    volatile uint32_t stop;      // host -> agent: drain what is committed, then exit
    volatile uint32_t resident;  // agent -> host: id of the launch whose CTAs all run
    volatile uint32_t status;    // agent -> host: exit reason of the last launch (kAgent*)
    volatile uint32_t exited;    // agent -> host: id of the last launch that finished
    volatile uint64_t next;      // agent -> host: slot the last launch stopped at
    // range mailbox: the front asks the host to check a range it has not seen
    volatile uint32_t q_seq;     // agent -> host: query number
    volatile uint32_t a_seq;     // host -> agent: number of the query answered
    volatile uint32_t q_kind;    // 0: source (pinned host memory), 1: destination (device memory)
    volatile uint32_t a_ok;      // 1: [a_lo, a_hi) is an allocation of the asked kind holding the range
    volatile uint64_t q_addr, q_size;
    volatile uint64_t a_lo, a_hi;
    // counters (agent -> host)
    volatile uint64_t rejected;   // descriptors rejected by validation
    volatile uint64_t first_bad;  // first rejected slot + 1 (0: none)
    volatile uint64_t queries;    // mailbox queries asked
    volatile uint64_t timeouts;   // waits that gave up (mailbox, slots, movers)
    volatile uint64_t exits[4];   // launches that ended, by reason (kAgentIdle, kAgentStopped, kAgentError)
    volatile uint32_t reset_ok;   // 1: the last launch left its counters zeroed
    volatile uint32_t _pad;
    // %globaltimer stamps of the last launch: front running, first batch published, last
    // batch completed, launch ended
    volatile uint64_t t_start, t_first, t_done, t_exit;
};

enum : uint32_t { kAgentRunning = 0, kAgentIdle = 1, kAgentStopped = 2, kAgentError = 3 };

struct AgentArgs {
    gfd::DescriptorQueue* q;
    gfd::QueueMirror* mirror;            // device copies of read_idx / done_idx (may be null)
    uint64_t* tile_done;                 // per-tile cumulative token counts (may be null)
    uint64_t* list_done;                 // per-list completion flags (may be null)
    volatile uint64_t* lists_completed;  // SGTaskQueue::lists_completed (may be null)
    AgentDev* dev;
    AgentHost* host;
    unsigned long long* bytes_ctr;       // payload bytes moved
    uint64_t start_slot;                 // first slot to consume
    uint64_t linger_ns;                  // exit after this long with nothing committed
    uint64_t idle_limit_ns;              // bound on idling in resident mode
    uint64_t wait_limit_ns;              // bound on every other wait
    uint32_t movers;                     // mover CTAs (1 .. kAgentMaxMovers)
    uint32_t launch_id;
    uint32_t resident;                   // 1: ignore linger_ns (idle_limit_ns still applies)
};

cudaError_t launch_agent(const AgentArgs& a, cudaStream_t st);
cudaError_t preload_agent();

}  // namespace gfdb
