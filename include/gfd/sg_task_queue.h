#pragma once
// Scatter-gather task queue: dynamic (src, dst, size) lists submitted by the host
// or by GPU code, consumed by the SG warp-specialised framework.
//
// Byte-compatible with the reference interface include/gfd/sg_task_queue.h:28-122
// (constants, DeviceSGEntry 24 B, SGList 32 B, SGTaskQueue field order with the
// cache-line separated indices). This library appends three fields inside the
// struct's existing 64-byte tail padding (stats pointer, wait limit, producer warp
// count, timeout counter); sizeof and every reference offset are unchanged.

#include <cstdint>
#include <cstddef>
#include "gfd/tiled_queue.h"

namespace gfd {

constexpr int MAX_SG_LISTS = 512;
constexpr int MAX_SG_POOL_ENTRIES = 16384;

constexpr uint32_t SG_FLAG_NONE = 0;
constexpr uint32_t SG_FLAG_HOST_SUBMITTED = 1;
// Library extension: the list's header and entries are in the session's device mirror
// (SGPollMirror::hdr / pool), written by a device submitter (SGSubmitter::
// write_header_device / publish_device); its host header, pool entries and marker are
// not written.
constexpr uint32_t SG_FLAG_DEVICE_ENTRIES = 2;

struct alignas(8) DeviceSGEntry {
    uint64_t src_addr;  // host source (pinned, device-mapped)
    uint64_t dst_addr;  // device destination
    uint32_t size;      // bytes
    uint32_t tag;       // caller's grouping tag
};

static_assert(sizeof(DeviceSGEntry) == 24, "DeviceSGEntry is 24 bytes");

struct alignas(16) SGList {
    uint32_t pool_offset;        // first entry (index into SGTaskQueue::entries)
    uint32_t count;              // number of entries
    uint32_t list_id;            // completion slot (d_list_done[list_id])
    uint32_t flags;              // SG_FLAG_*
    volatile uint64_t sequence;  // ring slot + 1 when committed, 0 when consumed
    // Reference: padding.  This library: absolute end of the list's pool entries,
    // written by the consumer once the list is fully processed (0 otherwise); lists
    // are then released in list order (see SGTaskQueue::lists_released).
    volatile uint64_t release_end;
};

static_assert(sizeof(SGList) == 32, "SGList is 32 bytes");

// Device-memory mirror of the list commit markers (library extension).  Many CTAs
// polling host memory at once throttle the GPU's reads of host memory for every SM (the
// pulls included), so consumers waiting for a list poll this mirror instead; one CTA at a
// time (the holder of `token`) reads a small window of markers from host memory, at
// most once per kMirrorPollNs, and publishes what it saw.
constexpr uint32_t kMirrorWindow = 16;         // markers read per poll round
constexpr uint64_t kMirrorPollNs = 2000;       // minimum time between poll rounds

// Header of a device-entry list (SG_FLAG_DEVICE_ENTRIES), kept in the mirror.
struct SGDeviceListHdr {
    uint32_t pool_offset;             // first entry (index into SGPollMirror::pool)
    uint32_t count;
    uint32_t list_id;
    uint32_t flags;
    unsigned long long first_entry;   // absolute pool index of the first entry
    volatile unsigned long long seq;  // list index + 1 once header and entries are written
};

// The consumers' shared counters live here too: concurrent accesses to one host-memory
// word from many SMs are serialised at about one PCIe round trip each (measured: 148 CTAs
// x 100 atomicAdd on one pinned word take 14 ms, a CAS loop far longer; in device memory
// 16 us).  The host-visible fields the API exposes (list_read_idx, lists_completed,
// entry_consumed_idx, the list markers) are published from these with one monotonic
// update per list.
struct SGPollMirror {
    unsigned int token;                        // 0 free, 1 held
    volatile unsigned int terminate;           // copy of SGTaskQueue::terminate
    volatile unsigned long long last_poll_ns;  // start of the last poll round
    volatile unsigned long long scan;          // lowest list index not yet seen committed
    unsigned long long claim;                  // next list index to claim (list_read_idx)
    unsigned long long completed;              // lists landed (lists_completed)
    unsigned long long released;               // lists released in order (lists_released)
    unsigned long long consumed;               // pool entries released (entry_consumed_idx)
    volatile unsigned long long committed[MAX_SG_LISTS];    // [i % MAX] = i + 1 once list i is committed
    volatile unsigned long long release_end[MAX_SG_LISTS];  // [i % MAX]: end of list i's entries once processed
    // Device-side submitters (sg_device_primitives.cuh) allocate here too: the counters
    // are seeded once per launch from entry_alloc_idx / list_alloc_idx (so lists the host
    // submitted first are counted) and published back with one monotonic update per
    // allocation; pool and ring space are judged from `consumed` and `slot_free`
    // without reading host memory.
    unsigned int alloc_state;                             // 0 unseeded, 1 seeding, 2 seeded
    unsigned long long entry_alloc;                       // entry_alloc_idx
    unsigned long long list_alloc;                        // list_alloc_idx
    volatile unsigned long long slot_free[MAX_SG_LISTS];  // [i % MAX] = i + 1 once list i's marker is cleared
    // Device-entry lists: a device submitter on the same GPU writes the entries and the
    // header here and commits in `committed` directly, so neither the submitter nor the
    // consumers cross PCIe for a list (under a saturated link a posted write to host
    // memory, a system fence or a host read each wait behind the payload reads).
    SGDeviceListHdr hdr[MAX_SG_LISTS];
    DeviceSGEntry pool[MAX_SG_POOL_ENTRIES];
};

struct SGTaskQueue {
    SGList lists[MAX_SG_LISTS];
    DeviceSGEntry entries[MAX_SG_POOL_ENTRIES];

    alignas(64) volatile uint64_t list_alloc_idx;      // producers
    alignas(64) volatile uint64_t entry_alloc_idx;     // producers
    alignas(64) volatile uint64_t list_read_idx;       // consumers claim lists here
    alignas(64) volatile uint64_t entry_consumed_idx;  // consumers release pool entries

    alignas(64) volatile uint64_t lists_completed;     // lists whose bytes have landed
    volatile uint32_t terminate;                       // set by the session to stop consumers
    volatile uint32_t timeout_site;  // reference: padding; here: last in-kernel wait that gave up

    uint64_t* d_list_done;  // device array [MAX_SG_LISTS]; non-zero once list_id landed

    // ---- library extension inside the reference's tail padding ----
    TransferStats* stats;          // device counters (may be null)
    uint64_t wait_limit_ns;        // bound on every in-kernel wait (0 = default)
    uint32_t producer_warps;       // pulling warps per CTA (0 means 1)
    volatile uint32_t wait_timeouts;
    volatile uint64_t lists_released;  // lists below this are released (marker cleared,
                                       // their entries counted in entry_consumed_idx)
    SGPollMirror* poll_mirror;         // device memory (may be null: consumers poll the
                                       // markers in host memory directly)
};

// Offsets of the reference layout (lists 16 KiB, entries 384 KiB, then one index
// per 64-byte line).
static_assert(offsetof(SGTaskQueue, entries) == 32 * MAX_SG_LISTS, "layout");
static_assert(offsetof(SGTaskQueue, list_alloc_idx) == 409600, "layout");
static_assert(offsetof(SGTaskQueue, entry_alloc_idx) == 409664, "layout");
static_assert(offsetof(SGTaskQueue, list_read_idx) == 409728, "layout");
static_assert(offsetof(SGTaskQueue, entry_consumed_idx) == 409792, "layout");
static_assert(offsetof(SGTaskQueue, lists_completed) == 409856, "layout");
static_assert(offsetof(SGTaskQueue, terminate) == 409864, "layout");
static_assert(offsetof(SGTaskQueue, d_list_done) == 409872, "layout");
static_assert(sizeof(SGTaskQueue) == 409920, "layout");
static_assert(offsetof(SGTaskQueue, poll_mirror) == 409912, "the extension fits the reference's tail padding");

namespace sg_compat {

// Linear token range -> SG entries (reference sg_task_queue.h:106-122 semantics):
// entry i covers token start_idx + i at cpu_base/gpu_base + (start_idx + i) * token_size.
inline void linear_to_sg_entries(DeviceSGEntry* entries, const void* cpu_base, void* gpu_base,
                                 uint32_t token_size, uint32_t start_idx, uint32_t count,
                                 uint32_t tag = 0) {
    const uint64_t src0 = reinterpret_cast<uint64_t>(cpu_base);
    const uint64_t dst0 = reinterpret_cast<uint64_t>(gpu_base);
    for (uint32_t i = 0; i < count; ++i) {
        const uint64_t off = static_cast<uint64_t>(start_idx + i) * token_size;
        entries[i] = DeviceSGEntry{src0 + off, dst0 + off, token_size, tag};
    }
}

}  // namespace sg_compat
}  // namespace gfd
