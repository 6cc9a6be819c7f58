// SM-pull gather kernels for sm_100a.
//
//  pull_kernel  moves a row table (see internal.h) from pinned, device-mapped host
//               memory into HBM (and, with the roles swapped, HBM into pinned host
//               memory: the device -> host scatter).  The aligned byte stream is split into equal
//               contiguous CTA ranges; each CTA stages the rows that cover its range
//               in shared memory (256 rows per window) and its 8 warps move 4 KiB
//               pieces: lane l of a warp owns 16-byte words l, l+32, ... of the
//               piece, issues all 8 loads, then the 8 stores.  Rows that are not
//               16-byte aligned ("misc") are copied one warp per row afterwards.
//               The last CTA to finish (device counter) raises a host-mapped
//               completion word, which lets the host wait without a CUDA call.
//
//  plan_kernel  builds the same row table on the GPU for entry lists that live in
//               device memory (routing kernels, the descriptor ring): it validates
//               each entry against the allowed source pools and destination
//               windows, marks run heads (an entry starts a new row unless it
//               continues its predecessor in both src and dst), compacts heads with
//               a warp ballot + block prefix scan, computes each row's stream
//               offset with a 64-bit block prefix sum of sizes, and finally the
//               first row of every pull CTA.
//
// Replaces the reference's CPU gather (src/parallel_gather.cpp:10-116), its
// contiguity detection / radix sort / coalescing (src/batch_processor.cpp:15-53,
// 605-831; src/direct_submit.cpp:41-59) and the CE DMA issue
// (src/copy_engine.cpp:89-153).  Output bytes are identical by construction: each
// destination byte receives exactly the source byte the entry maps to it.

#include <cuda_runtime.h>
#include <cstdint>

#include "gfd/pull.cuh"
#include "internal.h"
#include "pull_body.cuh"

namespace gfdb {

using gfd::pull::ld_host_v4;
using gfd::pull::st_v4;

__device__ __forceinline__ void st_release_sys_u64(volatile uint64_t* p, uint64_t v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Completion of a ring drain, run by every thread of the pull kernel's last CTA after all
// CTAs have counted in (their stores are visible at device scope): per-tile token counts
// and per-list flags first, then lists_completed, read_idx and done_idx in host memory,
// then their device-memory copies, which never run ahead of the host fields.  Same
// effects as the reference's batch completion (src/batch_processor.cpp:69-446).
__device__ __noinline__ void ring_epilogue(const RingDrain& d) {
    __threadfence();  // this thread's writes below follow every CTA's payload stores
    if (d.tables != nullptr) {
        if (d.tile_done != nullptr)
            for (uint32_t i = threadIdx.x; i < d.n_tiles; i += blockDim.x) {
                volatile uint64_t* p = &d.tile_done[d.tables->tile_id[i]];
                *p = *p + d.tables->tile_count[i];  // ids are distinct within a drain; drains run in order
            }
        if (d.list_done != nullptr)
            for (uint32_t i = threadIdx.x; i < d.n_lists; i += blockDim.x)
                *reinterpret_cast<volatile uint64_t*>(&d.list_done[d.tables->list_id[i]]) = 1;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        if (d.lists_completed != nullptr && d.lists_landed != 0)
            *d.lists_completed = *d.lists_completed + d.lists_landed;
        // drains complete in slot order on one stream: both indices only grow
        *d.read_idx = d.end;
        *d.done_idx = d.end;
        __threadfence_system();
        if (d.mirror_done != nullptr) {
            *d.mirror_read = d.end;
            if (*d.mirror_done < d.end) *d.mirror_done = d.end;
            __threadfence();
        }
    }
}

// The parameter block is __grid_constant__: the inline row and first-row tables are read
// in place (parameter space), without a per-thread copy.
__global__ void __launch_bounds__(kPullThreads) pull_kernel(const __grid_constant__ PullArgs a) {
    __shared__ PullRow srow[kRowWindow];
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    // launched behind the plan with programmatic stream serialization: the CTAs become
    // resident while the plan runs and wait here until it has completed and its table is
    // visible (without that launch attribute this returns at once)
    asm volatile("griddepcontrol.wait;" ::: "memory");

    PullGeometry geo = a.geo;
    if (a.hdr != nullptr) geo = a.hdr->geo;
    const PullRow* rows = a.rows != nullptr ? a.rows : a.rows_inline;
    const bool lens_from_starts = (geo.flags & kLensFromStarts) != 0;
    const PullRow* misc = a.misc != nullptr ? a.misc : a.rows_inline + geo.n_rows;

    const uint64_t lo = static_cast<uint64_t>(blockIdx.x) * geo.per_cta;
    const uint64_t hi = lo + geo.per_cta < geo.total ? lo + geo.per_cta : geo.total;
    uint64_t moved = 0;

    if (lo < hi) {
        const uint32_t* first = a.cta_first != nullptr ? a.cta_first : a.cta_first_inline;
        const uint32_t r0 = first[blockIdx.x];
        // rows this CTA needs end at the next CTA's first row (inclusive): stage only those
        uint32_t r_end = geo.n_rows;
        if (hi < geo.total && blockIdx.x + 1 < gridDim.x) {
            const uint32_t nxt = first[blockIdx.x + 1] + 1;
            if (nxt < r_end) r_end = nxt;
        }
        pull_stream_range(rows, geo.n_rows, geo.total, lens_from_starts, lo, hi, r0, r_end, srow);
        if (threadIdx.x == 0) moved = hi - lo;
    }

    // Rows without 16-byte alignment: one warp per row.
    const uint64_t mm = pull_misc_rows(misc, geo.n_misc, blockIdx.x * kPullWarps + warp, gridDim.x * kPullWarps);
    if (lane == 0) moved += mm;

    if (a.bytes_ctr != nullptr && lane == 0 && moved != 0)
        atomicAdd(a.bytes_ctr, static_cast<unsigned long long>(moved));

    if (a.done_ctr != nullptr) {
        __shared__ int s_last;
        __syncthreads();
        if (threadIdx.x == 0) {
            // the CTA's stores (ordered before this thread by the barrier) become visible
            // before its count: device scope for HBM destinations, system scope when the
            // destinations are host memory read by the CPU after the completion word
            if (a.sys_fence) __threadfence_system();
            else __threadfence();
            const unsigned prev = atomicAdd(a.done_ctr, 1u);
            s_last = prev == gridDim.x - 1;
            if (s_last) *a.done_ctr = 0u;  // ready for the next launch on this counter
        }
        __syncthreads();
        if (s_last) {
            if (a.drain.read_idx != nullptr) ring_epilogue(a.drain);
            if (threadIdx.x == 0) {
                __threadfence_system();
                if (a.done_flag != nullptr) st_release_sys_u64(a.done_flag, a.done_value);
            }
        }
    }
}

// The same pull with the bulk-copy mover (pull_body.cuh: pull_stream_range_bulk):
// host -> device only, selected by GFD_GATHER_BULK_STAGE.  A CTA whose load wait ran out
// still counts in, with a failure mark in the high bits of the launch's counter; the last
// CTA then leaves the completion word unset, so the caller's wait ends in a timeout
// instead of returning with bytes missing (the next launch on the counter starts clean).
constexpr unsigned kBulkFailMark = 1u << 20;  // above any CTA count (grid <= kMaxPullGrid)
static_assert(kMaxPullGrid < static_cast<int>(kBulkFailMark), "CTA count fits below the failure mark");

__global__ void __launch_bounds__(kPullThreads) pull_bulk_kernel(const __grid_constant__ PullArgs a) {
    extern __shared__ __align__(128) char bulk_smem[];
    BulkStage bs;
    bs.buf = bulk_smem;
    PullRow* srow = reinterpret_cast<PullRow*>(bulk_smem + kBulkBufBytes);
    bs.bar = reinterpret_cast<uint64_t*>(bulk_smem + kBulkBufBytes + kRowWindow * sizeof(PullRow));
    bulk_init(bs);
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    PullGeometry geo = a.geo;
    if (a.hdr != nullptr) geo = a.hdr->geo;
    const PullRow* rows = a.rows != nullptr ? a.rows : a.rows_inline;
    const bool lens_from_starts = (geo.flags & kLensFromStarts) != 0;
    const PullRow* misc = a.misc != nullptr ? a.misc : a.rows_inline + geo.n_rows;

    const uint64_t lo = static_cast<uint64_t>(blockIdx.x) * geo.per_cta;
    const uint64_t hi = lo + geo.per_cta < geo.total ? lo + geo.per_cta : geo.total;
    uint64_t moved = 0;
    if (lo < hi) {
        const uint32_t* first = a.cta_first != nullptr ? a.cta_first : a.cta_first_inline;
        const uint32_t r0 = first[blockIdx.x];
        uint32_t r_end = geo.n_rows;
        if (hi < geo.total && blockIdx.x + 1 < gridDim.x) {
            const uint32_t nxt = first[blockIdx.x + 1] + 1;
            if (nxt < r_end) r_end = nxt;
        }
        pull_stream_range_bulk(rows, geo.n_rows, geo.total, lens_from_starts, lo, hi, r0, r_end, srow, bs);
        if (threadIdx.x == 0) moved = hi - lo;
    }
    __shared__ int s_failed;
    if (threadIdx.x == 0) s_failed = 0;
    __syncthreads();
    if (!bulk_finish(bs) && lane == 0) s_failed = 1;

    const uint64_t mm = pull_misc_rows(misc, geo.n_misc, blockIdx.x * kPullWarps + warp, gridDim.x * kPullWarps);
    if (lane == 0) moved += mm;
    if (a.bytes_ctr != nullptr && lane == 0 && moved != 0)
        atomicAdd(a.bytes_ctr, static_cast<unsigned long long>(moved));

    if (a.done_ctr != nullptr) {
        __shared__ int s_last;
        __syncthreads();
        __shared__ int s_clean;
        if (threadIdx.x == 0) {
            __threadfence();
            const unsigned add = 1u + (s_failed ? kBulkFailMark : 0u);
            const unsigned prev = atomicAdd(a.done_ctr, add);
            s_last = (prev & (kBulkFailMark - 1u)) == gridDim.x - 1;
            s_clean = ((prev + add) & ~(kBulkFailMark - 1u)) == 0u;
            if (s_last) *a.done_ctr = 0u;
        }
        __syncthreads();
        if (s_last && threadIdx.x == 0) {
            __threadfence_system();
            if (a.done_flag != nullptr && s_clean) st_release_sys_u64(a.done_flag, a.done_value);
        }
    }
}

// ---------------------------------------------------------------------------
// GPU plan: entry list -> row table.
//
// A list of at most one tile (4096 entries) is planned by plan_kernel, one CTA.  Longer
// lists take three launches so the work spreads over the SMs:
//   plan_count_kernel  one CTA per tile: classify the tile's entries (start of a run,
//                      continuation, misaligned "misc", rejected) and write its totals;
//   plan_scan_kernel   one CTA: exclusive scan of the tile totals, the list's totals,
//                      the header, the first-row entries of pull CTAs past the stream;
//   plan_emit_kernel   one CTA per tile: classify again (the tile is L2-resident), write
//                      rows and misc rows at the scanned offsets, and the first row of
//                      every pull CTA whose stream range starts inside the tile.
// GPU-built rows carry their stream start only; the pull kernel derives each row's
// length from the next row's start (PullGeometry::flags & kLensFromStarts).
// ---------------------------------------------------------------------------
constexpr int kPlanThreads = 1024;
constexpr int kPlanItems = 4;                        // consecutive entries per thread
constexpr uint32_t kPlanTile = kPlanThreads * kPlanItems;
// dynamic shared memory: src, dst, size of one tile + the entry before it
constexpr size_t kPlanSmem = 3 * (kPlanTile + 1) * sizeof(uint64_t);
// plan_emit_kernel also keeps the stream starts of the tile's rows
constexpr size_t kEmitSmem = kPlanSmem + kPlanTile * sizeof(uint64_t);

struct EntryView {
    uint64_t src, dst, size;
    bool valid;    // passes validation and size > 0
    bool aligned;  // src, dst and size multiples of 16
};

__device__ __forceinline__ bool in_range(const RangeTable& t, uint32_t i, uint64_t p, uint64_t n) {
    return p >= t.lo[i] && n <= t.hi[i] - t.lo[i] && p - t.lo[i] <= t.hi[i] - t.lo[i] - n;
}

// Range check with a per-thread hint: consecutive entries almost always fall in the
// range the previous one did, so the table is searched only on a miss.
__device__ __forceinline__ bool in_table(const RangeTable& t, uint64_t p, uint64_t n, uint32_t& hint) {
    if (hint < t.n && in_range(t, hint, p, n)) return true;
    for (uint32_t i = 0; i < t.n; ++i)
        if (in_range(t, i, p, n)) {
            hint = i;
            return true;
        }
    return false;
}

// One tile of entries staged in shared memory; slot 0 holds the entry before the tile.
struct PlanTile {
    uint64_t* src;
    uint64_t* dst;
    uint64_t* size;
};

__device__ __forceinline__ uint64_t ld_sys_u64(const void* p) {
    uint64_t v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ const char* record(const PlanArgs& a, uint64_t i) {
    return reinterpret_cast<const char*>(a.entries) + i * sizeof(gfd_sg_entry);
}

// Stores word f of a gfd_sg_entry (dst, src, size) into tile slot `sl`.
__device__ __forceinline__ void put_word(const PlanTile& tile, uint32_t sl, uint32_t f, uint64_t v) {
    if (f == 0) tile.dst[sl] = v;
    else if (f == 1) tile.src[sl] = v;
    else tile.size[sl] = v;
}

// Loads entries [base, base + cnt) into slots 1..cnt and, when base > 0, entry base - 1
// into slot 0.  Consecutive threads read consecutive words of the 3-word records, so a
// warp's loads coalesce into full sectors; each thread issues a batch of loads before
// storing any of them.
__device__ __forceinline__ void load_tile(const PlanArgs& a, uint64_t base, uint32_t cnt, const PlanTile& tile) {
    const uint32_t nw = cnt * 3u;
    constexpr int kW = 8;
    for (uint32_t w0 = 0; w0 < nw; w0 += kW * kPlanThreads) {
        uint64_t v[kW];
#pragma unroll
        for (int q = 0; q < kW; ++q) {
            const uint32_t w = w0 + threadIdx.x + q * kPlanThreads;
            if (w < nw) {
                const uint32_t k = w / 3u, f = w - k * 3u;
                v[q] = ld_sys_u64(record(a, base + k) + 8u * f);
            }
        }
#pragma unroll
        for (int q = 0; q < kW; ++q) {
            const uint32_t w = w0 + threadIdx.x + q * kPlanThreads;
            if (w < nw) {
                const uint32_t k = w / 3u, f = w - k * 3u;
                put_word(tile, k + 1, f, v[q]);
            }
        }
    }
    if (base > 0 && threadIdx.x < 3u)
        put_word(tile, 0, threadIdx.x, ld_sys_u64(record(a, base - 1) + 8u * threadIdx.x));
}

__device__ __forceinline__ EntryView view_entry(const PlanArgs& a, const PlanTile& tile, uint32_t j,
                                                uint32_t& src_hint, uint32_t& dst_hint) {
    EntryView e;
    e.src = tile.src[j];
    e.dst = tile.dst[j];
    e.size = tile.size[j];
    const bool ok = in_table(a.src_ok, e.src, e.size, src_hint) && in_table(a.dst_ok, e.dst, e.size, dst_hint);
    e.valid = ok && e.size > 0;
    e.aligned = ((e.src | e.dst | e.size) & 15u) == 0;
    return e;
}

template <typename T>
__device__ __forceinline__ T warp_incl_scan(T x, int lane) {
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const T y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    return x;
}

// Classification of the thread's tile entries 4t .. 4t+3 (slots 4t+1 .. 4t+4).
struct Classified {
    uint32_t heads, miscs;       // rows started here, misaligned rows
    uint32_t hbits, mbits, sbits;  // per entry: starts a row / misc / part of the stream
    uint64_t bytes;              // stream bytes of the thread's entries
    uint64_t bad;                // first rejected entry index, or ~0
};

__device__ __forceinline__ Classified classify(const PlanArgs& a, const PlanTile& tile, uint64_t base, uint32_t cnt,
                                               uint32_t& src_hint, uint32_t& dst_hint) {
    Classified c{0, 0, 0, 0, 0, 0, ~0ull};
    const uint32_t j0 = threadIdx.x * kPlanItems;
    if (j0 >= cnt) return c;
    EntryView prev = view_entry(a, tile, j0, src_hint, dst_hint);  // slot j0 = the entry before j0
    const bool has_prev = base + j0 > 0;
#pragma unroll
    for (int k = 0; k < kPlanItems; ++k) {
        const uint32_t j = j0 + k;
        if (j >= cnt) break;
        const EntryView e = view_entry(a, tile, j + 1, src_hint, dst_hint);
        if (e.size > 0 && !e.valid && c.bad == ~0ull) c.bad = base + j;
        if (e.valid && e.aligned) {
            const bool cont = (k > 0 || has_prev) && prev.valid && prev.aligned && prev.src + prev.size == e.src &&
                              prev.dst + prev.size == e.dst;
            if (!cont) {
                c.hbits |= 1u << k;
                ++c.heads;
            }
            c.sbits |= 1u << k;
            c.bytes += e.size;
        } else if (e.valid) {
            c.mbits |= 1u << k;
            ++c.miscs;
        }
        prev = e;
    }
    return c;
}

struct BlockScan {
    uint32_t heads, miscs;   // exclusive prefix of this thread
    uint64_t bytes;
    uint32_t t_heads, t_miscs;  // block totals
    uint64_t t_bytes;
};

struct ScanSmem {
    unsigned long long bytes[33];
    uint32_t heads[33];
    uint32_t miscs[33];
};

// Block-wide exclusive scan of the per-thread counts (callers sync before reusing `sm`).
__device__ __forceinline__ BlockScan block_scan(const Classified& c, ScanSmem& sm) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t ih = warp_incl_scan<uint32_t>(c.heads, lane);
    const uint32_t im = warp_incl_scan<uint32_t>(c.miscs, lane);
    const unsigned long long ib = warp_incl_scan<unsigned long long>(c.bytes, lane);
    if (lane == 31) {
        sm.bytes[warp] = ib;
        sm.heads[warp] = ih;
        sm.miscs[warp] = im;
    }
    __syncthreads();
    if (warp == 0) {
        const unsigned long long wb = sm.bytes[lane];
        const uint32_t wh = sm.heads[lane], wm = sm.miscs[lane];
        const unsigned long long xb = warp_incl_scan<unsigned long long>(wb, lane);
        const uint32_t xh = warp_incl_scan<uint32_t>(wh, lane);
        const uint32_t xm = warp_incl_scan<uint32_t>(wm, lane);
        sm.bytes[lane] = xb - wb;
        sm.heads[lane] = xh - wh;
        sm.miscs[lane] = xm - wm;
        if (lane == 31) {
            sm.bytes[32] = xb;
            sm.heads[32] = xh;
            sm.miscs[32] = xm;
        }
    }
    __syncthreads();
    BlockScan o;
    o.heads = sm.heads[warp] + ih - c.heads;
    o.miscs = sm.miscs[warp] + im - c.miscs;
    o.bytes = sm.bytes[warp] + ib - c.bytes;
    o.t_heads = sm.heads[32];
    o.t_miscs = sm.miscs[32];
    o.t_bytes = sm.bytes[32];
    return o;
}

// Writes the thread's rows (start offsets; lengths come from successive starts) and misc
// rows.  `hstart` (may be null) receives the start of each row at its rank in the tile.
__device__ __forceinline__ void write_rows(const PlanArgs& a, const PlanTile& tile, const Classified& c, uint32_t r,
                                           uint32_t m, uint64_t off, uint64_t* hstart, uint32_t hlocal) {
    if ((c.sbits | c.mbits) == 0) return;
#pragma unroll
    for (int k = 0; k < kPlanItems; ++k) {
        const uint32_t sl = threadIdx.x * kPlanItems + k + 1;
        if (c.sbits & (1u << k)) {
            if (c.hbits & (1u << k)) {
                a.rows[r++] = PullRow{tile.src[sl], tile.dst[sl], 0, off};
                if (hstart != nullptr) hstart[hlocal] = off;
                ++hlocal;
            }
            off += tile.size[sl];
        } else if (c.mbits & (1u << k)) {
            a.misc[m++] = PullRow{tile.src[sl], tile.dst[sl], tile.size[sl], 0};
        }
    }
}

__device__ __forceinline__ uint64_t plan_per_cta(uint64_t total, uint32_t grid) {
    uint64_t per = (total + grid - 1) / grid;
    per = (per + kPiece - 1) / kPiece * kPiece;
    return per == 0 ? kPiece : per;
}

__device__ __forceinline__ void write_header(const PlanArgs& a, uint64_t total, uint64_t per, uint32_t n_rows,
                                             uint32_t n_misc, uint64_t bad) {
    PlanHeader h;
    h.geo.total = total;
    h.geo.per_cta = per;
    h.geo.flags = kLensFromStarts;
    h.geo.n_rows = n_rows;
    h.geo.n_misc = n_misc;
    h.bad_entry = bad;
    h.status = (bad == ~0ull) ? GFD_OK : GFD_ERR_INVALID;
    h.list_done = 0;   // the short-list kernel's between-launch state
    h.list_nbad = 0;
    *a.hdr = h;
}

__device__ __forceinline__ void launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// First row of pull CTA c: the last row starting at or before c * per (0 past the stream).
// hstart: the rows' stream starts in shared memory.
__device__ __forceinline__ void first_rows_from_starts(const PlanArgs& a, const uint64_t* hstart, uint32_t n_rows,
                                                       uint64_t total) {
    const uint64_t per = plan_per_cta(total, a.grid);
    for (uint32_t c = threadIdx.x; c < a.grid; c += kPlanThreads) {
        const uint64_t target = static_cast<uint64_t>(c) * per;
        uint32_t first = 0;
        if (target < total && n_rows > 0) {
            uint32_t l = 0, h = n_rows - 1;
            while (l < h) {
                const uint32_t mid = (l + h + 1) >> 1;
                if (hstart[mid] <= target) l = mid;
                else h = mid - 1;
            }
            first = l;
        }
        a.cta_first[c] = first;
    }
}

__global__ void __launch_bounds__(kPlanThreads) plan_kernel(PlanArgs a) {
    extern __shared__ uint64_t s_dyn[];
    __shared__ ScanSmem s_scan;
    __shared__ unsigned long long s_bad;
    const PlanTile tile{s_dyn, s_dyn + (kPlanTile + 1), s_dyn + 2 * (kPlanTile + 1)};
    const int t = threadIdx.x;
    uint32_t src_hint = 0, dst_hint = 0;
    if (t == 0) s_bad = ~0ull;
    launch_dependents();  // the pull may start launching; it waits for this grid to finish
    if (a.n <= kPlanTile) {
        // one tile: the row starts stay in shared memory for the first-row search
        uint64_t* hstart = s_dyn + 3 * (kPlanTile + 1);
        const uint32_t cnt = static_cast<uint32_t>(a.n);
        load_tile(a, 0, cnt, tile);
        __syncthreads();
        const Classified c = classify(a, tile, 0, cnt, src_hint, dst_hint);
        if (c.bad != ~0ull) atomicMin(&s_bad, c.bad);
        const BlockScan so = block_scan(c, s_scan);
        write_rows(a, tile, c, so.heads, so.miscs, so.bytes, hstart, so.heads);
        __syncthreads();
        first_rows_from_starts(a, hstart, so.t_heads, so.t_bytes);
        if (t == 0) write_header(a, so.t_bytes, plan_per_cta(so.t_bytes, a.grid), so.t_heads, so.t_miscs, s_bad);
        return;
    }
    uint64_t cb = 0;  // carries (identical in every thread)
    uint32_t ch = 0, cm = 0;

    for (uint64_t base = 0; base < a.n; base += kPlanTile) {
        const uint32_t cnt = static_cast<uint32_t>(a.n - base < kPlanTile ? a.n - base : kPlanTile);
        load_tile(a, base, cnt, tile);
        __syncthreads();
        const Classified c = classify(a, tile, base, cnt, src_hint, dst_hint);
        if (c.bad != ~0ull) atomicMin(&s_bad, c.bad);
        const BlockScan so = block_scan(c, s_scan);
        write_rows(a, tile, c, ch + so.heads, cm + so.miscs, cb + so.bytes, nullptr, 0);
        cb += so.t_bytes;
        ch += so.t_heads;
        cm += so.t_miscs;
        __syncthreads();  // tile and scan scratch free for the next tile
    }

    const uint64_t total = cb;
    const uint32_t n_rows = ch;
    const uint64_t per = plan_per_cta(total, a.grid);
    for (uint32_t c = t; c < a.grid; c += kPlanThreads) {
        const uint64_t target = static_cast<uint64_t>(c) * per;
        uint32_t first = 0;
        if (target < total && n_rows > 0) {
            uint32_t l = 0, h = n_rows - 1;
            while (l < h) {
                const uint32_t mid = (l + h + 1) >> 1;
                if (a.rows[mid].start <= target) l = mid;
                else h = mid - 1;
            }
            first = l;
        }
        a.cta_first[c] = first;
    }
    if (t == 0) write_header(a, total, per, n_rows, cm, s_bad);
}

__global__ void __launch_bounds__(kPlanThreads) plan_count_kernel(PlanArgs a) {
    extern __shared__ uint64_t s_dyn[];
    __shared__ ScanSmem s_scan;
    __shared__ unsigned long long s_bad;
    const PlanTile tile{s_dyn, s_dyn + (kPlanTile + 1), s_dyn + 2 * (kPlanTile + 1)};
    uint32_t src_hint = 0, dst_hint = 0;
    if (threadIdx.x == 0) s_bad = ~0ull;
    const uint64_t base = static_cast<uint64_t>(blockIdx.x) * kPlanTile;
    const uint32_t cnt = static_cast<uint32_t>(a.n - base < kPlanTile ? a.n - base : kPlanTile);
    load_tile(a, base, cnt, tile);
    __syncthreads();
    const Classified c = classify(a, tile, base, cnt, src_hint, dst_hint);
    if (c.bad != ~0ull) atomicMin(&s_bad, c.bad);
    const BlockScan so = block_scan(c, s_scan);  // ends with a barrier: s_bad is final
    if (threadIdx.x == 0) a.tiles[blockIdx.x] = TileTotals{so.t_bytes, s_bad, so.t_heads, so.t_miscs};
}

// One CTA: tiles[nt + i] = exclusive prefix of tiles[0..i), tiles[2 nt] = list totals.
__global__ void __launch_bounds__(kPlanThreads) plan_scan_kernel(PlanArgs a, uint32_t nt) {
    __shared__ ScanSmem s_scan;
    __shared__ unsigned long long s_bad;
    if (threadIdx.x == 0) s_bad = ~0ull;
    __syncthreads();
    uint64_t cb = 0;
    uint32_t ch = 0, cm = 0;
    for (uint32_t b = 0; b < nt; b += kPlanThreads) {
        const uint32_t i = b + threadIdx.x;
        Classified c{0, 0, 0, 0, 0, 0, ~0ull};
        if (i < nt) {
            const TileTotals x = a.tiles[i];
            c.heads = x.heads;
            c.miscs = x.misc;
            c.bytes = x.bytes;
            if (x.bad != ~0ull) atomicMin(&s_bad, x.bad);
        }
        const BlockScan so = block_scan(c, s_scan);
        if (i < nt) a.tiles[nt + i] = TileTotals{cb + so.bytes, 0, ch + so.heads, cm + so.miscs};
        cb += so.t_bytes;
        ch += so.t_heads;
        cm += so.t_miscs;
        __syncthreads();
    }
    const uint64_t per = plan_per_cta(cb, a.grid);
    // pull CTAs whose range starts past the stream do no stream work
    for (uint32_t c = threadIdx.x; c < a.grid; c += kPlanThreads)
        if (static_cast<uint64_t>(c) * per >= cb) a.cta_first[c] = 0;
    if (threadIdx.x == 0) {
        a.tiles[2 * nt] = TileTotals{cb, s_bad, ch, cm};
        write_header(a, cb, per, ch, cm, s_bad);
    }
}

__global__ void __launch_bounds__(kPlanThreads) plan_emit_kernel(PlanArgs a, uint32_t nt) {
    extern __shared__ uint64_t s_dyn[];
    __shared__ ScanSmem s_scan;
    launch_dependents();
    const PlanTile tile{s_dyn, s_dyn + (kPlanTile + 1), s_dyn + 2 * (kPlanTile + 1)};
    uint64_t* hstart = s_dyn + 3 * (kPlanTile + 1);
    uint32_t src_hint = 0, dst_hint = 0;
    const uint64_t base = static_cast<uint64_t>(blockIdx.x) * kPlanTile;
    const uint32_t cnt = static_cast<uint32_t>(a.n - base < kPlanTile ? a.n - base : kPlanTile);
    const TileTotals carry = a.tiles[nt + blockIdx.x];
    const TileTotals mine = a.tiles[blockIdx.x];
    const uint64_t total = a.tiles[2 * nt].bytes;
    load_tile(a, base, cnt, tile);
    __syncthreads();
    const Classified c = classify(a, tile, base, cnt, src_hint, dst_hint);
    const BlockScan so = block_scan(c, s_scan);
    write_rows(a, tile, c, carry.heads + so.heads, carry.misc + so.miscs, carry.bytes + so.bytes, hstart, so.heads);
    __syncthreads();
    if (mine.bytes == 0) return;
    // first row of every pull CTA whose range starts in this tile's stream bytes
    const uint64_t per = plan_per_cta(total, a.grid);
    const uint64_t lo = carry.bytes, hi = carry.bytes + mine.bytes;
    const uint64_t c_lo = (lo + per - 1) / per;
    uint64_t c_hi = (hi + per - 1) / per;
    if (c_hi > a.grid) c_hi = a.grid;
    for (uint64_t cc = c_lo + threadIdx.x; cc < c_hi; cc += kPlanThreads) {
        const uint64_t target = cc * per;
        // last row of this tile starting at or before target (rows are in start order)
        int l = -1, h = static_cast<int>(mine.heads) - 1;
        while (l < h) {
            const int mid = (l + h + 1) >> 1;
            if (hstart[mid] <= target) l = mid;
            else h = mid - 1;
        }
        a.cta_first[cc] = l >= 0 ? carry.heads + static_cast<uint32_t>(l) : carry.heads - 1;
    }
}

int pull_grid_for(uint64_t total_bytes, int num_sms) {
    const uint64_t pieces = (total_bytes + kPiece - 1) / kPiece;
    uint64_t grid = static_cast<uint64_t>(num_sms) * 2;
    // one 4 KiB piece per warp, at most two CTAs per SM
    const uint64_t want = (pieces + kPullWarps - 1) / kPullWarps;
    if (want < grid) grid = want;
    if (grid < 1) grid = 1;
    return static_cast<int>(grid);
}

// With lazy module loading, the first launch of a kernel loads its code and can be
// serialised behind kernels already running -- e.g. a user kernel spinning on
// done_idx that this very launch is supposed to satisfy.  Contexts load the library's
// kernels up front instead.
__global__ void list_pull_kernel(const __grid_constant__ ListArgs a);

cudaError_t preload_gather_kernels() {
    cudaFuncAttributes fa;
    cudaError_t e = cudaFuncGetAttributes(&fa, pull_kernel);
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, pull_bulk_kernel);
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, list_pull_kernel);
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, plan_kernel);
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, plan_count_kernel);
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, plan_scan_kernel);
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, plan_emit_kernel);
    // the plan tiles (~96-128 KiB) live in dynamic shared memory above the 48 KiB default
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(pull_bulk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(kBulkSmem));
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(plan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kEmitSmem));
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(plan_count_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(kPlanSmem));
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(plan_emit_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(kEmitSmem));
    return e;
}

size_t plan_tile_slots(uint64_t n) { return 2 * ((n + kPlanTile - 1) / kPlanTile) + 1; }

cudaError_t launch_pull(const PullArgs& a, int grid, cudaStream_t st, bool bulk, bool after_plan) {
    if (bulk) {
        pull_bulk_kernel<<<grid, kPullThreads, kBulkSmem, st>>>(a);
        return cudaGetLastError();
    }
    if (after_plan) {
        // programmatic dependent launch: the pull's CTAs launch while the plan runs
        cudaLaunchConfig_t cfg = {};
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.gridDim = dim3(static_cast<unsigned>(grid));
        cfg.blockDim = dim3(kPullThreads);
        cfg.dynamicSmemBytes = 0;
        cfg.stream = st;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        return cudaLaunchKernelEx(&cfg, pull_kernel, a);
    }
    pull_kernel<<<grid, kPullThreads, 0, st>>>(a);
    return cudaGetLastError();
}

// Short device lists: CTA c works on entry c mod n, together with the other CTAs that
// map to the same entry; the entry is cut into 4 KiB chunks shared out over those CTAs'
// warps.  With at least two CTAs per SM in the grid, a list of small entries gets about
// one CTA per entry and a list of a few large entries spreads over the whole GPU, and no
// CTA reads more than its own entry (no plan, no scan).  Entries are checked against the
// source ranges and the destination window first; rejected ones are skipped and the first
// is reported through the header by the last CTA to finish, as the plan path does.
// Chunks keep an entry's relative alignment, so aligned entries copy with 16-byte accesses.
constexpr uint64_t kListChunk = 4096;

__global__ void __launch_bounds__(kPullThreads) list_pull_kernel(const __grid_constant__ ListArgs a) {
    __shared__ uint64_t s_e[3];
    __shared__ int s_ok;
    const uint32_t warp = threadIdx.x >> 5;
    const uint32_t i = blockIdx.x % a.n;
    const uint32_t part = blockIdx.x / a.n, parts = (gridDim.x - 1 - i) / a.n + 1;  // CTAs on entry i
    if (threadIdx.x < 3) s_e[threadIdx.x] = reinterpret_cast<const uint64_t*>(a.entries + i)[threadIdx.x];
    __syncthreads();
    const uint64_t dst = s_e[0], src = s_e[1], size = s_e[2];
    if (threadIdx.x == 0) {
        bool ok = size == 0 ||
                  (size <= a.dst_hi - a.dst_lo && dst >= a.dst_lo && dst - a.dst_lo <= a.dst_hi - a.dst_lo - size);
        if (ok && size != 0) {
            bool in_src = false;
            for (uint32_t r = 0; r < a.n_src; ++r)
                in_src = in_src || (size <= a.src_hi[r] - a.src_lo[r] && src >= a.src_lo[r] &&
                                    src - a.src_lo[r] <= a.src_hi[r] - a.src_lo[r] - size);
            ok = in_src;
        }
        if (!ok && part == 0) atomicMax(&a.hdr->list_nbad, ~static_cast<unsigned long long>(i));
        s_ok = ok ? 1 : 0;
    }
    __syncthreads();
    if (s_ok && size != 0) {
        const uint64_t chunks = (size + kListChunk - 1) / kListChunk;
        const uint64_t step = static_cast<uint64_t>(parts) * kPullWarps;
        for (uint64_t k = static_cast<uint64_t>(part) * kPullWarps + warp; k < chunks; k += step) {
            const uint64_t off = k * kListChunk;
            const uint64_t len = size - off < kListChunk ? size - off : kListChunk;
            gfd::pull::warp_copy<kPullUnroll, true>(reinterpret_cast<void*>(dst + off), reinterpret_cast<const void*>(src + off),
                                              len);
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        const unsigned prev = atomicAdd(&a.hdr->list_done, 1u);
        if (prev == gridDim.x - 1) {  // last CTA: publish, and leave the fields at 0 for the next launch
            const unsigned long long v = atomicExch(&a.hdr->list_nbad, 0ull);
            a.hdr->list_done = 0u;
            a.hdr->bad_entry = v != 0 ? ~v : ~0ull;
            a.hdr->status = v != 0 ? static_cast<uint32_t>(GFD_ERR_INVALID) : static_cast<uint32_t>(GFD_OK);
            __threadfence();
        }
    }
}

cudaError_t launch_list_pull(const ListArgs& a, int num_sms, cudaStream_t st) {
    // at least one CTA per entry and two per SM, so a few large entries spread over the GPU
    const uint32_t floor = static_cast<uint32_t>(2 * num_sms);
    const int grid = static_cast<int>(a.n > floor ? a.n : floor);
    list_pull_kernel<<<grid, kPullThreads, 0, st>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_plan(const PlanArgs& a, cudaStream_t st) {
    if (a.n <= kPlanTile || a.tiles == nullptr) {
        plan_kernel<<<1, kPlanThreads, a.n <= kPlanTile ? kEmitSmem : kPlanSmem, st>>>(a);
        return cudaGetLastError();
    }
    const uint32_t nt = static_cast<uint32_t>((a.n + kPlanTile - 1) / kPlanTile);
    plan_count_kernel<<<nt, kPlanThreads, kPlanSmem, st>>>(a);
    plan_scan_kernel<<<1, kPlanThreads, 0, st>>>(a, nt);
    plan_emit_kernel<<<nt, kPlanThreads, kEmitSmem, st>>>(a, nt);
    return cudaGetLastError();
}

}  // namespace gfdb
