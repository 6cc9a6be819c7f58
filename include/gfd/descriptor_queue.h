#pragma once
// Host<->GPU descriptor ring: the wire format of GPU-queued submission.
//
// Byte-compatible with the reference interface include/gfd/descriptor_queue.h:9-53
// (same constants, same field order, sizes and alignment; static_asserts below pin
// every offset), so GPU producer code written against the reference keeps working.
//
// Protocol (unchanged):
//   producer   reserves slots [b, b+n), writes Descriptor fields, fences, then stores
//              sequence = slot + 1 (the commit marker);
//   consumer   accepts slot s only when sequence == s + 1, clears sequence to 0 after
//              it no longer needs the descriptor, advances read_idx;
//   completion done_idx = number of leading slots whose bytes have landed in GPU
//              memory; waiters test done_idx >= base_slot + count.
// In this library the consumer is the ring agent, a device-resident kernel
// (gfd_b200/csrc/agent.cu): it polls the commit markers, copies committed runs out and
// clears their markers, pulls the bytes and advances read_idx / done_idx.  The fields
// keep their meaning.

#include <cstdint>
#include <cstddef>

namespace gfd {

constexpr int QUEUE_SIZE = 16384;
constexpr int MAX_BATCH_SIZE = 8192;
constexpr int BATCH_THRESHOLD = 4096;
constexpr size_t ADAPTIVE_BATCH_TARGET_BYTES = 1024 * 1024;
constexpr int BATCH_THRESHOLD_SMALL = 1024;

constexpr uint32_t FLAG_NONE = 0;
constexpr uint32_t FLAG_LAST_IN_BATCH = 1;
constexpr uint32_t FLAG_URGENT = 2;

// One 64-byte ring entry.
struct alignas(64) Descriptor {
    uint64_t src_addr;           // host source (pinned, device-mapped)
    uint64_t dst_addr;           // device destination
    uint32_t size;               // bytes
    uint32_t flags;              // FLAG_*
    uint64_t user_data;          // (tile or list id << 32) | index, or user payload
    volatile uint64_t sequence;  // slot + 1 when committed, 0 when free
};

static_assert(sizeof(Descriptor) == 64, "Descriptor is 64 bytes");
static_assert(offsetof(Descriptor, src_addr) == 0, "layout");
static_assert(offsetof(Descriptor, dst_addr) == 8, "layout");
static_assert(offsetof(Descriptor, size) == 16, "layout");
static_assert(offsetof(Descriptor, flags) == 20, "layout");
static_assert(offsetof(Descriptor, user_data) == 24, "layout");
static_assert(offsetof(Descriptor, sequence) == 32, "layout");

// Device-memory copies of read_idx and done_idx (library extension), kept current by
// this library's ring consumer, which writes the host fields first.  Many CTAs polling
// host memory throttle every SM's reads of host memory (the consumer's own pulls
// included), so device-side waits poll these copies and confirm success with one read
// of the host field.
struct QueueMirror {
    volatile uint64_t read_idx;
    volatile uint64_t done_idx;
};

struct DescriptorQueue {
    Descriptor entries[QUEUE_SIZE];
    volatile uint64_t write_idx;  // producers: atomicAdd to reserve slots
    volatile uint64_t read_idx;   // consumer: slots below this are free to reuse
    volatile uint64_t done_idx;   // consumer: slots below this have landed
    // The reference leaves these 40 bytes as padding. This library keeps the size and
    // uses them for a count of device-side waits that gave up (bounded waits, see
    // device.cuh) and for the device-memory mirror of the indices (null when no ring
    // consumer of this library is attached; whoever resets the host indices resets the
    // mirror too).  Everything else stays zero.
    volatile uint32_t wait_timeouts;
    uint32_t _reserved;
    QueueMirror* mirror;
    uint8_t _padding[64 - 24 - 4 - 4 - 8];
};

static_assert(offsetof(DescriptorQueue, write_idx) == (size_t)QUEUE_SIZE * 64, "layout");
static_assert(offsetof(DescriptorQueue, read_idx) == (size_t)QUEUE_SIZE * 64 + 8, "layout");
static_assert(offsetof(DescriptorQueue, done_idx) == (size_t)QUEUE_SIZE * 64 + 16, "layout");
static_assert(sizeof(DescriptorQueue) == (size_t)QUEUE_SIZE * 64 + 64, "layout");
static_assert(offsetof(DescriptorQueue, mirror) == (size_t)QUEUE_SIZE * 64 + 32, "extension inside the padding");

// Per-token request record used by GPU producers (reference examples pass these in).
struct TokenInfo {
    uint64_t cpu_addr;
    uint32_t token_id;
    uint32_t expert_id;
};

static_assert(sizeof(TokenInfo) == 16, "TokenInfo is 16 bytes");

}  // namespace gfd
