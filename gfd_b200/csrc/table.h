#pragma once
// Host-built pull tables: the part of a gather call that turns an entry list into the
// work the pull kernel does.  Plain C++ (no CUDA), so the CPU tests compile it on its
// own (tests/host_logic.cpp).
//
// A "row" is one contiguous (src, dst, len) span.  Rows whose src, dst and len are all
// multiples of 16 form the aligned byte stream: row r owns stream bytes
// [start_r, start_r + len_r), and each pull CTA takes an equal, piece-aligned part of the
// stream.  Entries that continue the previous aligned entry in both src and dst extend
// its row (run merging); entries with any misaligned field become "misc" rows, copied one
// warp per row with narrower accesses, and end the current run.  Same bytes land as when
// the entries are copied one by one in list order (the reference's semantics,
// src/parallel_gather.cpp:10-27): entries never overlap in their destinations in a valid
// call, and a merged row copies exactly the bytes of the entries it covers.

#include <cstdint>
#include <vector>

namespace gfdb {

struct PullRow {
    uint64_t src;
    uint64_t dst;
    uint64_t len;
    uint64_t start;
};
static_assert(sizeof(PullRow) == 32, "PullRow is 32 bytes");

// Run-merging table builder: add() the entries of one call in order.
class TableBuilder {
public:
    TableBuilder(PullRow* rows, std::vector<PullRow>* misc) : rows_(rows), misc_(misc) {}

    void add(uint64_t src, uint64_t dst, uint64_t size) {
        if (size == 0) return;
        if (((src | dst | size) & 15u) != 0) {
            misc_->push_back(PullRow{src, dst, size, 0});
            chain_ = false;
            return;
        }
        if (chain_ && src == src_end_ && dst == dst_end_) {
            rows_[n_rows_ - 1].len += size;
        } else {
            rows_[n_rows_++] = PullRow{src, dst, size, total_};
        }
        total_ += size;
        chain_ = true;
        src_end_ = src + size;
        dst_end_ = dst + size;
    }

    uint32_t n_rows() const { return n_rows_; }
    uint64_t total() const { return total_; }  // aligned stream bytes

    // Re-packs the stream without the rows taken out by `take` (called with each row;
    // returns true to remove it), recomputing the starts.  Used to move long rows to the
    // copy engine.
    template <typename Take>
    void remove_rows(Take take) {
        uint32_t w = 0;
        uint64_t off = 0;
        for (uint32_t r = 0; r < n_rows_; ++r) {
            if (take(rows_[r])) continue;
            PullRow x = rows_[r];
            x.start = off;
            off += x.len;
            rows_[w++] = x;
        }
        n_rows_ = w;
        total_ = off;
        chain_ = false;
    }

private:
    PullRow* rows_;
    std::vector<PullRow>* misc_;
    uint32_t n_rows_ = 0;
    uint64_t total_ = 0;
    bool chain_ = false;
    uint64_t src_end_ = 0, dst_end_ = 0;
};

// Appends the span (src, dst, len) to `runs`, extending the last run instead when the
// span continues it in both source and destination.  Any alignment: this is for the copy
// engine, which has none to keep.  Empty spans are dropped.
inline void append_run(std::vector<PullRow>* runs, uint64_t src, uint64_t dst, uint64_t len) {
    if (len == 0) return;
    if (!runs->empty()) {
        PullRow& b = runs->back();
        if (b.src + b.len == src && b.dst + b.len == dst) {
            b.len += len;
            return;
        }
    }
    runs->push_back(PullRow{src, dst, len, 0});
}

// A copy-engine copy: `height` rows of `width` bytes, row i from src + i * spitch to
// dst + i * dpitch (height 1: one plain copy).
struct CeCopy {
    uint64_t dst, src, width, height, dpitch, spitch;
};

// Groups consecutive runs of one length whose sources and destinations advance by
// constant pitches (each at least the length, below 2^31) into 2D copies, so an evenly
// strided gather -- a 2x-stride token layout, say -- costs one copy-engine call instead
// of one per token.  Runs are (src, dst, len) in call order; the copies keep that order.
inline void group_strided(const PullRow* runs, size_t n, std::vector<CeCopy>* out) {
    constexpr uint64_t kMaxPitch = (1ull << 31) - 1;
    size_t i = 0;
    while (i < n) {
        CeCopy c{runs[i].dst, runs[i].src, runs[i].len, 1, runs[i].len, runs[i].len};
        size_t j = i + 1;
        if (j < n && runs[j].len == c.width && runs[j].src > runs[i].src && runs[j].dst > runs[i].dst) {
            const uint64_t sp = runs[j].src - runs[i].src, dp = runs[j].dst - runs[i].dst;
            if (sp >= c.width && dp >= c.width && sp <= kMaxPitch && dp <= kMaxPitch) {
                c.spitch = sp;
                c.dpitch = dp;
                while (j < n && runs[j].len == c.width && runs[j].src - runs[j - 1].src == sp &&
                       runs[j].dst - runs[j - 1].dst == dp && runs[j].src > runs[j - 1].src &&
                       runs[j].dst > runs[j - 1].dst)
                    ++j;
                c.height = j - i;
            } else {
                j = i + 1;
            }
        } else {
            j = i + 1;
        }
        out->push_back(c);
        i = j;
    }
}

// First row of each pull CTA: CTA c covers stream bytes [c * per, (c + 1) * per) and
// starts in the last row whose start is at or below c * per (rows sorted by start).
inline void partition_ctas(const PullRow* rows, uint32_t n_rows, uint64_t per, int grid, uint32_t* first) {
    uint32_t r = 0;
    for (int c = 0; c < grid; ++c) {
        const uint64_t target = static_cast<uint64_t>(c) * per;
        while (r + 1 < n_rows && rows[r + 1].start <= target) ++r;
        first[c] = r;
    }
}

}  // namespace gfdb
