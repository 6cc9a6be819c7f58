#pragma once
// Host side of a ring drain (GPU-queued submit), plain C++ so the CPU tests compile it on
// its own (tests/host_logic.cpp): finding the committed run at the ring's read position,
// the reference poller's batching rule, and the per-drain completion accounting (tokens
// per tile, lists whose last descriptor is in the drain).  Reference behaviour:
// src/cpu_polling.cpp:337-436 (scan and batching), src/batch_processor.cpp:69-446
// (per-tile and per-list completion).

#include <cstdint>

#include "gfd/descriptor_queue.h"
#include "gfd/sg_task_queue.h"
#include "gfd/tiled_queue.h"

namespace gfdb {

// Flags that end a batch at once: the producer marked a batch, tile or list boundary.
constexpr uint32_t kUrgentFlags = gfd::FLAG_LAST_IN_BATCH | gfd::FLAG_URGENT | gfd::FLAG_LAST_IN_TILE |
                                  gfd::FLAG_LAST_CHUNK_IN_TILE;

// Length of the committed run at slot `next` (at most max_n): consecutive slots whose
// marker equals slot + 1, read with acquire loads.  *urgent: a slot of the run carries a
// boundary flag.
inline uint32_t committed_run(const gfd::DescriptorQueue* q, uint64_t next, uint32_t max_n, bool* urgent) {
    uint32_t n = 0;
    *urgent = false;
    while (n < max_n) {
        const gfd::Descriptor* d = &q->entries[(next + n) % gfd::QUEUE_SIZE];
        const uint64_t seq = __atomic_load_n(&d->sequence, __ATOMIC_ACQUIRE);
        if (seq != next + n + 1) break;
        if (d->flags & kUrgentFlags) *urgent = true;
        ++n;
    }
    return n;
}

// The reference poller's batching: a run goes at once when forced, when a boundary flag
// is in it, or when it reached BATCH_THRESHOLD_SMALL slots; otherwise once the producers
// have stopped extending it for `quiet_ns`.
class BatchGate {
public:
    explicit BatchGate(uint64_t quiet_ns = 20000) : quiet_ns_(quiet_ns) {}

    bool ready(uint32_t n, bool urgent, bool force, uint64_t now_ns) {
        if (n == 0) {
            pending_n_ = 0;
            return false;
        }
        if (!force && !urgent && n < static_cast<uint32_t>(gfd::BATCH_THRESHOLD_SMALL)) {
            if (n != pending_n_) {
                pending_n_ = n;
                pending_since_ = now_ns;
                return false;
            }
            if (now_ns - pending_since_ < quiet_ns_) return false;
        }
        pending_n_ = 0;
        return true;
    }

    void reset() { pending_n_ = 0; }

private:
    uint64_t quiet_ns_;
    uint32_t pending_n_ = 0;
    uint64_t pending_since_ = 0;
};

// Completion accounting of one drain.  add() each descriptor's flags and user_data
// ((tile or list id << 32) | index): a tiled queue counts every descriptor toward its tile
// (ids below MAX_TILES; the per-tile counters are cumulative token counts), an SG queue
// counts a list as landed at the descriptor flagged FLAG_LAST_IN_TILE (ids below
// MAX_SG_LISTS).  `counts` is caller-owned scratch of MAX_TILES zeros, left zeroed by
// finish().
class DrainAccounting {
public:
    DrainAccounting(bool tiled, bool sg, uint32_t* counts, uint16_t* tile_id, uint32_t* tile_count,
                    uint16_t* list_id, uint32_t max_lists)
        : tiled_(tiled), sg_(sg), counts_(counts), tile_id_(tile_id), tile_count_(tile_count), list_id_(list_id),
          max_lists_(max_lists) {}

    void add(uint32_t flags, uint64_t user_data) {
        const uint32_t id = static_cast<uint32_t>(user_data >> 32);
        if (tiled_ && id < static_cast<uint32_t>(gfd::MAX_TILES) && counts_[id]++ == 0) tile_id_[n_tiles_++] = static_cast<uint16_t>(id);
        if (sg_ && (flags & gfd::FLAG_LAST_IN_TILE) && id < static_cast<uint32_t>(gfd::MAX_SG_LISTS)) {
            if (n_lists_ < max_lists_) list_id_[n_lists_++] = static_cast<uint16_t>(id);
            ++lists_landed_;
        }
    }

    // Writes the per-tile counts next to their ids (in first-seen order) and clears the
    // scratch.
    void finish() {
        for (uint32_t k = 0; k < n_tiles_; ++k) {
            tile_count_[k] = counts_[tile_id_[k]];
            counts_[tile_id_[k]] = 0;
        }
    }

    uint32_t n_tiles() const { return n_tiles_; }
    uint32_t n_lists() const { return n_lists_; }
    uint32_t lists_landed() const { return lists_landed_; }

private:
    bool tiled_, sg_;
    uint32_t* counts_;
    uint16_t* tile_id_;
    uint32_t* tile_count_;
    uint16_t* list_id_;
    uint32_t max_lists_;
    uint32_t n_tiles_ = 0, n_lists_ = 0, lists_landed_ = 0;
};

}  // namespace gfdb
