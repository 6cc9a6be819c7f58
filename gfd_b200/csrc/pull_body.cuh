#pragma once
// The body of the SM pull, shared by pull_kernel (gather.cu: one launch per request) and
// the ring agent (agent.cu: a resident kernel that drains the descriptor ring), so both
// move bytes with exactly the same code.
//
// Row tables (table.h: PullRow) describe an aligned byte stream: row r owns stream bytes
// [start_r, start_r + len_r) and maps them to (src_r, dst_r).  A CTA copies a contiguous
// stream range: it stages the rows covering the range in shared memory, kRowWindow at a
// time, and its 8 warps move 4 KiB pieces -- lane l owns 16-byte words l, l+32, ... of
// the piece, issues all 8 loads, then the 8 stores.  Rows that are not 16-byte aligned
// ("misc" rows) are copied one warp per row.
//
// Bulk-copy variant (pull_stream_range_bulk): the same windows and pieces, but a warp
// moves a piece with cp.async.bulk -- host memory -> shared memory, completion on an
// mbarrier (expect_tx = the piece's bytes), then a bulk store shared memory -> HBM --
// through two 4 KiB buffers per warp, so a piece's store drains while the next piece
// loads.  Each lane issues the copies of one row segment of the piece.  No multicast; the
// source is this process's pinned host memory.  Selected by GFD_GATHER_BULK_STAGE.

#include <cstdint>

#include "gfd/pull.cuh"
#include "internal.h"

namespace gfdb {

// Largest r in [0, n) with rows[r].start <= pos (rows sorted by start, rows[0].start <= pos).
__device__ __forceinline__ int find_row(const PullRow* rows, int n, uint64_t pos) {
    int lo = 0, hi = n - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (rows[mid].start <= pos) lo = mid;
        else hi = mid - 1;
    }
    return lo;
}

// Copies stream bytes [lo, hi) (lo < hi) of the table `rows` (n_rows rows, stream length
// `total`).  r0 is the row holding byte lo; rows r0 .. r_end-1 cover the range.  With
// lens_from_starts, row lengths are not stored and come from the next row's start (GPU-built
// tables).  srow: kRowWindow rows of shared memory.  Every thread of the CTA calls it.
__device__ __forceinline__ void pull_stream_range(const PullRow* rows, uint32_t n_rows, uint64_t total,
                                                  bool lens_from_starts, uint64_t lo, uint64_t hi, uint32_t r0,
                                                  uint32_t r_end, PullRow* srow) {
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    uint64_t pos = lo;
    while (pos < hi) {
        const uint32_t left = r_end - r0;
        const int nw = left < static_cast<uint32_t>(kRowWindow) ? static_cast<int>(left) : kRowWindow;
        __syncthreads();  // previous window fully consumed
        if (threadIdx.x < nw) srow[threadIdx.x] = rows[r0 + threadIdx.x];
        if (lens_from_starts) {  // uniform over the block
            const unsigned tid = threadIdx.x, last = static_cast<unsigned>(nw) - 1;
            uint64_t nx = 0;
            if (tid == last) nx = r0 + nw < n_rows ? rows[r0 + nw].start : total;
            __syncthreads();
            uint64_t len = 0;
            if (tid < last) nx = srow[tid + 1].start;
            if (tid <= last) len = nx - srow[tid].start;
            __syncthreads();
            if (tid <= last) srow[tid].len = len;
        }
        __syncthreads();
        const uint64_t wend = srow[nw - 1].start + srow[nw - 1].len;
        const uint64_t whi = wend < hi ? wend : hi;

        for (uint64_t pb = pos + static_cast<uint64_t>(warp) * kPiece; pb < whi;
             pb += static_cast<uint64_t>(kPullWarps) * kPiece) {
            int r = find_row(srow, nw, pb);
            uint4 v[kPullUnroll];
            char* d[kPullUnroll];
#pragma unroll
            for (int u = 0; u < kPullUnroll; ++u) {
                const uint64_t g = pb + static_cast<uint64_t>(u * 32 + lane) * 16u;
                d[u] = nullptr;
                if (g < whi) {
                    while (r + 1 < nw && g >= srow[r + 1].start) ++r;
                    const uint64_t off = g - srow[r].start;
                    v[u] = gfd::pull::ld_host_v4(reinterpret_cast<const char*>(srow[r].src) + off);
                    d[u] = reinterpret_cast<char*>(srow[r].dst) + off;
                }
            }
#pragma unroll
            for (int u = 0; u < kPullUnroll; ++u)
                if (d[u] != nullptr) gfd::pull::st_v4(d[u], v[u]);
        }
        pos = whi;
        r0 += static_cast<uint32_t>(nw);
    }
}

// ---------------------------------------------------------------------------
// Bulk-copy staging
// ---------------------------------------------------------------------------
constexpr int kBulkBuffers = 2;                                      // per warp
constexpr uint64_t kBulkWaitNs = 2000000000ull;                      // bound on one piece's load
constexpr size_t kBulkBufBytes = static_cast<size_t>(kPullWarps) * kBulkBuffers * kPiece;
// dynamic shared memory of the bulk pull: buffers, then the row window, then the barriers
constexpr size_t kBulkSmem = kBulkBufBytes + kRowWindow * sizeof(PullRow) +
                             static_cast<size_t>(kPullWarps) * kBulkBuffers * sizeof(uint64_t);

struct BulkStage {
    char* buf;          // [kPullWarps][kBulkBuffers][kPiece], 128-byte aligned
    uint64_t* bar;      // [kPullWarps][kBulkBuffers] mbarriers
    uint32_t phase;     // this warp's parity bit per buffer (bit b)
    uint32_t next;      // buffer the next piece uses
    bool failed;        // a load wait ran out: the warp stops moving pieces
};

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Lane 0 of every warp initialises the warp's barriers (arrival count 1).
__device__ __forceinline__ void bulk_init(BulkStage& bs) {
    const int warp = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0)
        for (int b = 0; b < kBulkBuffers; ++b)
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_addr(&bs.bar[warp * kBulkBuffers + b]))
                         : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    __syncwarp();
    bs.phase = 0;
    bs.next = 0;
    bs.failed = false;
}

// Rows r .. of the window that overlap [pb, pe): lane-parallel, 32 segments a round.
// Calls f(seg_lo, row) for each overlapping row (seg_lo = first stream byte of the segment).
template <typename F>
__device__ __forceinline__ void for_segments(const PullRow* srow, int nw, uint64_t pb, uint64_t pe, F&& f) {
    const int lane = threadIdx.x & 31;
    const int r0 = find_row(srow, nw, pb);
    for (int base = r0; base < nw; base += 32) {
        const int r = base + lane;
        const bool in = r < nw && srow[r].start < pe;
        if (in) {
            const uint64_t lo = srow[r].start > pb ? srow[r].start : pb;
            const uint64_t end = srow[r].start + srow[r].len;
            if (end > lo) f(lo, (end < pe ? end : pe) - lo, srow[r]);
        }
        if (!__any_sync(0xffffffffu, in) || srow[base + 31 < nw ? base + 31 : nw - 1].start >= pe) break;
    }
}

// One warp moves its pieces of [pos, whi) through its two buffers.
__device__ __forceinline__ void bulk_pieces(const PullRow* srow, int nw, uint64_t pos, uint64_t whi,
                                            BulkStage& bs) {
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    for (uint64_t pb = pos + static_cast<uint64_t>(warp) * kPiece; pb < whi && !bs.failed;
         pb += static_cast<uint64_t>(kPullWarps) * kPiece) {
        const uint64_t pe = pb + kPiece < whi ? pb + kPiece : whi;
        const uint32_t b = bs.next;
        bs.next ^= 1u;
        char* buf = bs.buf + (static_cast<size_t>(warp) * kBulkBuffers + b) * kPiece;
        const uint32_t bar = smem_addr(&bs.bar[warp * kBulkBuffers + b]);
        // the store that last read this buffer (issued one piece ago at most) is done reading
        asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
        __syncwarp();
        if (lane == 0)
            asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar),
                         "r"(static_cast<uint32_t>(pe - pb))
                         : "memory");
        __syncwarp();
        for_segments(srow, nw, pb, pe, [&](uint64_t lo, uint64_t n, const PullRow& row) {
            asm volatile(
                "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                    smem_addr(buf + (lo - pb))),
                "l"(row.src + (lo - row.start)), "r"(static_cast<uint32_t>(n)), "r"(bar)
                : "memory");
        });
        // bounded wait for the piece's bytes
        const uint32_t parity = (bs.phase >> b) & 1u;
        const uint64_t t0 = gfd::pull::globaltimer_ns();
        uint32_t done = 0;
        while (true) {
            asm volatile(
                "{\n\t.reg .pred p;\n\t"
                "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                "selp.u32 %0, 1, 0, p;\n\t}"
                : "=r"(done)
                : "r"(bar), "r"(parity)
                : "memory");
            if (done || gfd::pull::globaltimer_ns() - t0 > kBulkWaitNs) break;
        }
        if (!__all_sync(0xffffffffu, done != 0)) {  // leave the buffers to the copies in flight
            bs.failed = true;
            break;
        }
        bs.phase ^= 1u << b;
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        for_segments(srow, nw, pb, pe, [&](uint64_t lo, uint64_t n, const PullRow& row) {
            asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(row.dst + (lo - row.start)),
                         "r"(smem_addr(buf + (lo - pb))), "r"(static_cast<uint32_t>(n))
                         : "memory");
        });
        asm volatile("cp.async.bulk.commit_group;" ::: "memory");
    }
}

// Waits until the warp's bulk stores have written HBM; after a failed load wait, also
// gives the loads still in flight a bounded time to land before the CTA's shared memory
// is released.  Returns true when every piece moved.
__device__ __forceinline__ bool bulk_finish(BulkStage& bs) {
    asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
    asm volatile("fence.proxy.async;" ::: "memory");
    if (bs.failed) {
        const int warp = threadIdx.x >> 5;
        for (int b = 0; b < kBulkBuffers; ++b) {
            const uint32_t bar = smem_addr(&bs.bar[warp * kBulkBuffers + b]);
            const uint32_t parity = (bs.phase >> b) & 1u;
            const uint64_t t0 = gfd::pull::globaltimer_ns();
            uint32_t done = 0;
            while (!done && gfd::pull::globaltimer_ns() - t0 < kBulkWaitNs)
                asm volatile(
                    "{\n\t.reg .pred p;\n\t"
                    "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                    "selp.u32 %0, 1, 0, p;\n\t}"
                    : "=r"(done)
                    : "r"(bar), "r"(parity)
                    : "memory");
        }
    }
    return !bs.failed;
}

// pull_stream_range with the bulk-copy mover (same arguments; srow in dynamic shared
// memory, bs initialised by bulk_init).
__device__ __forceinline__ void pull_stream_range_bulk(const PullRow* rows, uint32_t n_rows, uint64_t total,
                                                       bool lens_from_starts, uint64_t lo, uint64_t hi,
                                                       uint32_t r0, uint32_t r_end, PullRow* srow,
                                                       BulkStage& bs) {
    uint64_t pos = lo;
    while (pos < hi) {
        const uint32_t left = r_end - r0;
        const int nw = left < static_cast<uint32_t>(kRowWindow) ? static_cast<int>(left) : kRowWindow;
        __syncthreads();
        if (threadIdx.x < nw) srow[threadIdx.x] = rows[r0 + threadIdx.x];
        if (lens_from_starts) {
            const unsigned tid = threadIdx.x, last = static_cast<unsigned>(nw) - 1;
            uint64_t nx = 0;
            if (tid == last) nx = r0 + nw < n_rows ? rows[r0 + nw].start : total;
            __syncthreads();
            uint64_t len = 0;
            if (tid < last) nx = srow[tid + 1].start;
            if (tid <= last) len = nx - srow[tid].start;
            __syncthreads();
            if (tid <= last) srow[tid].len = len;
        }
        __syncthreads();
        const uint64_t wend = srow[nw - 1].start + srow[nw - 1].len;
        const uint64_t whi = wend < hi ? wend : hi;
        bulk_pieces(srow, nw, pos, whi, bs);
        pos = whi;
        r0 += static_cast<uint32_t>(nw);
    }
}

// Misaligned rows: warp gw of nwarps takes rows gw, gw + nwarps, ...  Returns the bytes
// this warp moved (every lane gets the same value).
__device__ __forceinline__ uint64_t pull_misc_rows(const PullRow* misc, uint32_t n_misc, uint32_t gw,
                                                   uint32_t nwarps) {
    uint64_t moved = 0;
    for (uint32_t m = gw; m < n_misc; m += nwarps) {
        const PullRow row = misc[m];
        gfd::pull::warp_copy<kPullUnroll, true>(reinterpret_cast<void*>(row.dst),
                                                reinterpret_cast<const void*>(row.src), row.len);
        moved += row.len;
    }
    return moved;
}

}  // namespace gfdb
