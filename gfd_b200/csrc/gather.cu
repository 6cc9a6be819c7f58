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

namespace gfdb {

using gfd::pull::ld_host_v4;
using gfd::pull::st_v4;

__device__ __forceinline__ void st_release_sys_u64(volatile uint64_t* p, uint64_t v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

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

// The parameter block is __grid_constant__: the inline row and first-row tables are read
// in place (parameter space), without a per-thread copy.
__global__ void __launch_bounds__(kPullThreads) pull_kernel(const __grid_constant__ PullArgs a) {
    __shared__ PullRow srow[kRowWindow];
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    PullGeometry geo = a.geo;
    if (a.hdr != nullptr) geo = a.hdr->geo;
    const PullRow* rows = a.rows != nullptr ? a.rows : a.rows_inline;
    const PullRow* misc = a.misc != nullptr ? a.misc : a.rows_inline + geo.n_rows;

    const uint64_t lo = static_cast<uint64_t>(blockIdx.x) * geo.per_cta;
    const uint64_t hi = lo + geo.per_cta < geo.total ? lo + geo.per_cta : geo.total;
    uint64_t moved = 0;

    if (lo < hi) {
        const uint32_t* first = a.cta_first != nullptr ? a.cta_first : a.cta_first_inline;
        uint32_t r0 = first[blockIdx.x];
        // rows this CTA needs end at the next CTA's first row (inclusive): stage only those
        uint32_t r_end = geo.n_rows;
        if (hi < geo.total && blockIdx.x + 1 < gridDim.x) {
            const uint32_t nxt = first[blockIdx.x + 1] + 1;
            if (nxt < r_end) r_end = nxt;
        }
        uint64_t pos = lo;
        while (pos < hi) {
            const uint32_t left = r_end - r0;
            const int nw = left < static_cast<uint32_t>(kRowWindow) ? static_cast<int>(left) : kRowWindow;
            __syncthreads();  // previous window fully consumed
            if (threadIdx.x < nw) srow[threadIdx.x] = rows[r0 + threadIdx.x];
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
                        v[u] = ld_host_v4(reinterpret_cast<const char*>(srow[r].src) + off);
                        d[u] = reinterpret_cast<char*>(srow[r].dst) + off;
                    }
                }
#pragma unroll
                for (int u = 0; u < kPullUnroll; ++u)
                    if (d[u] != nullptr) st_v4(d[u], v[u]);
            }
            pos = whi;
            r0 += static_cast<uint32_t>(nw);
        }
        if (threadIdx.x == 0) moved = hi - lo;
    }

    // Rows without 16-byte alignment: one warp per row.
    const uint32_t gw = blockIdx.x * kPullWarps + warp;
    const uint32_t nwarps = gridDim.x * kPullWarps;
    for (uint32_t m = gw; m < geo.n_misc; m += nwarps) {
        const PullRow row = misc[m];
        gfd::pull::warp_copy<kPullUnroll>(reinterpret_cast<void*>(row.dst),
                                          reinterpret_cast<const void*>(row.src), row.len);
        if (lane == 0) moved += row.len;
    }

    if (a.bytes_ctr != nullptr && lane == 0 && moved != 0)
        atomicAdd(a.bytes_ctr, static_cast<unsigned long long>(moved));

    if (a.done_ctr != nullptr) {
        __syncthreads();
        if (threadIdx.x == 0) {
            // the CTA's stores (ordered before this thread by the barrier) become visible
            // before its count: device scope for HBM destinations, system scope when the
            // destinations are host memory read by the CPU after the completion word
            if (a.sys_fence) __threadfence_system();
            else __threadfence();
            const unsigned prev = atomicAdd(a.done_ctr, 1u);
            if (prev == gridDim.x - 1) {
                *a.done_ctr = 0u;  // ready for the next launch on this counter
                __threadfence_system();
                if (a.done_flag != nullptr) st_release_sys_u64(a.done_flag, a.done_value);
            }
        }
    }
}

// ---------------------------------------------------------------------------
// plan_kernel: one CTA of 1024 threads, tiles of 4096 entries (4 per thread).
// ---------------------------------------------------------------------------
constexpr int kPlanThreads = 1024;
constexpr int kPlanItems = 4;                        // consecutive entries per thread
constexpr uint32_t kPlanTile = kPlanThreads * kPlanItems;
// dynamic shared memory: src, dst, size of one tile + the previous tile's last entry
constexpr size_t kPlanSmem = 3 * (kPlanTile + 1) * sizeof(uint64_t);

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

// One tile of entries staged in shared memory (slot 0 holds the previous tile's last
// entry, so every entry can be compared with its predecessor).
struct PlanTile {
    uint64_t* src;
    uint64_t* dst;
    uint64_t* size;
};

// Loads entries [base, base + cnt) into tile slots 1..cnt.  Consecutive threads read
// consecutive words of the records (gfd_sg_entry: all 3 words; ring descriptor: its first
// 4 words), so a warp's loads coalesce into full sectors instead of one small request
// per field.  Ring descriptors also hand their flags and user_data to `meta_*` for the
// finalize kernel, which then never reads the ring again.
__device__ __forceinline__ uint64_t ld_sys_u64(const void* p) {
    uint64_t v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// Each thread issues all of its loads before using any of them, so a tile costs one
// memory latency rather than one per word.
__device__ __forceinline__ void load_tile(const PlanArgs& a, uint64_t base, uint32_t cnt, const PlanTile& tile) {
    if (a.kind == 0) {
        constexpr int kW = 6;  // words per batch; 3 per entry, two batches per tile
        const char* rec0 = static_cast<const char*>(a.entries) + base * a.stride;
        const uint32_t nw = cnt * 3u;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            uint64_t v[kW];
#pragma unroll
            for (int q = 0; q < kW; ++q) {
                const uint32_t w = threadIdx.x + (h * kW + q) * kPlanThreads;
                if (w < nw) {
                    const uint32_t k = w / 3u, f = w - k * 3u;
                    v[q] = ld_sys_u64(rec0 + k * a.stride + 8u * f);
                }
            }
#pragma unroll
            for (int q = 0; q < kW; ++q) {
                const uint32_t w = threadIdx.x + (h * kW + q) * kPlanThreads;
                if (w < nw) {
                    const uint32_t k = w / 3u, f = w - k * 3u;
                    if (f == 0) tile.dst[k + 1] = v[q];
                    else if (f == 1) tile.src[k + 1] = v[q];
                    else tile.size[k + 1] = v[q];
                }
            }
        }
    } else {
        constexpr int kW = 8;  // words per batch; 4 per descriptor, two batches per tile
        const uint32_t nw = cnt * 4u;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            uint64_t v[kW];
#pragma unroll
            for (int q = 0; q < kW; ++q) {
                const uint32_t w = threadIdx.x + (h * kW + q) * kPlanThreads;
                if (w < nw) {
                    const uint64_t slot = (a.ring_begin + base + (w >> 2)) % a.ring_size;
                    v[q] = ld_sys_u64(static_cast<const char*>(a.entries) + slot * a.stride + 8u * (w & 3u));
                }
            }
#pragma unroll
            for (int q = 0; q < kW; ++q) {
                const uint32_t w = threadIdx.x + (h * kW + q) * kPlanThreads;
                if (w >= nw) continue;
                const uint32_t k = w >> 2, f = w & 3u;
                if (f == 0) {
                    tile.src[k + 1] = v[q];
                } else if (f == 1) {
                    tile.dst[k + 1] = v[q];
                } else if (f == 2) {
                    tile.size[k + 1] = v[q] & 0xffffffffull;  // size (u32), flags in the high half
                    if (a.meta_flags != nullptr) a.meta_flags[base + k] = static_cast<uint32_t>(v[q] >> 32);
                } else if (a.meta_user != nullptr) {
                    a.meta_user[base + k] = v[q];
                }
            }
        }
    }
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

__global__ void __launch_bounds__(kPlanThreads) plan_kernel(PlanArgs a) {
    extern __shared__ uint64_t s_dyn[];
    __shared__ unsigned long long s_wbytes[32];
    __shared__ uint32_t s_wheads[32];
    __shared__ uint32_t s_wmisc[32];
    __shared__ unsigned long long s_carry_bytes;
    __shared__ uint32_t s_carry_heads, s_carry_misc;
    __shared__ unsigned long long s_bad;

    const PlanTile tile{s_dyn, s_dyn + (kPlanTile + 1), s_dyn + 2 * (kPlanTile + 1)};
    const int t = threadIdx.x;
    uint32_t src_hint = 0, dst_hint = 0;
    const int lane = t & 31, warp = t >> 5;
    if (t == 0) {
        s_carry_bytes = 0;
        s_carry_heads = 0;
        s_carry_misc = 0;
        s_bad = ~0ull;
    }
    __syncthreads();

    for (uint64_t base = 0; base < a.n; base += kPlanTile) {
        const uint32_t cnt = static_cast<uint32_t>(a.n - base < kPlanTile ? a.n - base : kPlanTile);
        load_tile(a, base, cnt, tile);
        __syncthreads();
        // thread t owns tile entries 4t .. 4t+3 (slots 4t+1 .. 4t+4; predecessor of the
        // first is slot 4t)
        uint32_t heads = 0, miscs = 0, hbits = 0, mbits = 0, sbits = 0;  // head / misc / stream entries
        uint64_t bytes = 0;
        EntryView prev = view_entry(a, tile, static_cast<uint32_t>(t) * kPlanItems, src_hint, dst_hint);
        const bool has_prev = base + static_cast<uint64_t>(t) * kPlanItems > 0;
#pragma unroll
        for (int k = 0; k < kPlanItems; ++k) {
            const uint32_t j = static_cast<uint32_t>(t) * kPlanItems + k;
            if (j >= cnt) break;
            const EntryView e = view_entry(a, tile, j + 1, src_hint, dst_hint);
            if (e.size > 0 && !e.valid) atomicMin(&s_bad, static_cast<unsigned long long>(base + j));
            if (e.valid && e.aligned) {
                const bool cont = (k > 0 || has_prev) && prev.valid && prev.aligned &&
                                  prev.src + prev.size == e.src && prev.dst + prev.size == e.dst;
                if (!cont) {
                    hbits |= 1u << k;
                    ++heads;
                }
                sbits |= 1u << k;
                bytes += e.size;
            } else if (e.valid) {
                mbits |= 1u << k;
                ++miscs;
            }
            prev = e;
        }
        // block exclusive scan of the per-thread counts
        const uint32_t ih = warp_incl_scan<uint32_t>(heads, lane);
        const uint32_t im = warp_incl_scan<uint32_t>(miscs, lane);
        const unsigned long long ib = warp_incl_scan<unsigned long long>(bytes, lane);
        if (lane == 31) {
            s_wbytes[warp] = ib;
            s_wheads[warp] = ih;
            s_wmisc[warp] = im;
        }
        __syncthreads();
        if (warp == 0) {
            const unsigned long long wb = s_wbytes[lane];
            const uint32_t wh = s_wheads[lane], wm = s_wmisc[lane];
            const unsigned long long xb = warp_incl_scan<unsigned long long>(wb, lane);
            const uint32_t xh = warp_incl_scan<uint32_t>(wh, lane);
            const uint32_t xm = warp_incl_scan<uint32_t>(wm, lane);
            s_wbytes[lane] = xb - wb;  // exclusive per-warp offsets
            s_wheads[lane] = xh - wh;
            s_wmisc[lane] = xm - wm;
        }
        __syncthreads();
        const unsigned long long cb = s_carry_bytes;
        const uint32_t ch = s_carry_heads, cm = s_carry_misc;
        uint32_t r = ch + s_wheads[warp] + (ih - heads);
        uint32_t m = cm + s_wmisc[warp] + (im - miscs);
        unsigned long long off = cb + s_wbytes[warp] + (ib - bytes);
        if (sbits | mbits) {
#pragma unroll
            for (int k = 0; k < kPlanItems; ++k) {
                const uint32_t sl = static_cast<uint32_t>(t) * kPlanItems + k + 1;
                if (sbits & (1u << k)) {
                    if (hbits & (1u << k)) a.rows[r++] = PullRow{tile.src[sl], tile.dst[sl], 0, off};
                    off += tile.size[sl];
                } else if (mbits & (1u << k)) {
                    a.misc[m++] = PullRow{tile.src[sl], tile.dst[sl], tile.size[sl], 0};
                }
            }
        }
        __syncthreads();
        if (t == kPlanThreads - 1) {
            s_carry_bytes = cb + s_wbytes[31] + ib;
            s_carry_heads = ch + s_wheads[31] + ih;
            s_carry_misc = cm + s_wmisc[31] + im;
        }
        // the tile's last entry becomes the next tile's predecessor (slot 0)
        if (t == 0) {
            tile.src[0] = tile.src[cnt];
            tile.dst[0] = tile.dst[cnt];
            tile.size[0] = tile.size[cnt];
        }
        __syncthreads();
    }

    const uint64_t total = s_carry_bytes;
    const uint32_t n_rows = s_carry_heads;
    // row lengths from successive starts (loads of a batch issued before its stores)
    for (uint32_t r0 = t; r0 < n_rows; r0 += 4 * kPlanThreads) {
        uint64_t st[4], nx[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const uint32_t r = r0 + q * kPlanThreads;
            if (r < n_rows) {
                st[q] = a.rows[r].start;
                nx[q] = (r + 1 < n_rows) ? a.rows[r + 1].start : total;
            }
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const uint32_t r = r0 + q * kPlanThreads;
            if (r < n_rows) a.rows[r].len = nx[q] - st[q];
        }
    }
    uint64_t per = (total + a.grid - 1) / a.grid;
    per = (per + kPiece - 1) / kPiece * kPiece;
    if (per == 0) per = kPiece;
    __syncthreads();
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
    if (t == 0) {
        PlanHeader h;
        h.geo.total = total;
        h.geo.per_cta = per;
        h.geo.uniform = 0;
        h.geo.n_rows = n_rows;
        h.geo.n_misc = s_carry_misc;
        h.bad_entry = s_bad;
        h.status = (s_bad == ~0ull) ? GFD_OK : GFD_ERR_INVALID;
        h._pad = 0;
        *a.hdr = h;
    }
}

int pull_grid_for(uint64_t total_bytes, int num_sms) {
    const uint64_t pieces = (total_bytes + kPiece - 1) / kPiece;
    uint64_t grid = static_cast<uint64_t>(num_sms) * 2;
    // small jobs: about two pieces per warp-set so every CTA does some work
    const uint64_t want = (pieces + kPullWarps - 1) / kPullWarps;
    if (want < grid) grid = want;
    if (grid < 1) grid = 1;
    return static_cast<int>(grid);
}

// With lazy module loading, the first launch of a kernel loads its code and can be
// serialised behind kernels already running -- e.g. a user kernel spinning on
// done_idx that this very launch is supposed to satisfy.  Contexts load the library's
// kernels up front instead.
cudaError_t preload_gather_kernels() {
    cudaFuncAttributes fa;
    cudaError_t e = cudaFuncGetAttributes(&fa, pull_kernel);
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, plan_kernel);
    // the plan's tile (~96 KiB) lives in dynamic shared memory above the 48 KiB default
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(plan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kPlanSmem));
    return e;
}

cudaError_t launch_pull(const PullArgs& a, int grid, cudaStream_t st) {
    pull_kernel<<<grid, kPullThreads, 0, st>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_plan(const PlanArgs& a, cudaStream_t st) {
    plan_kernel<<<1, kPlanThreads, kPlanSmem, st>>>(a);
    return cudaGetLastError();
}

}  // namespace gfdb
