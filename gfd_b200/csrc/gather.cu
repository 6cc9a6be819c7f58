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
// plan_kernel: one CTA of 1024 threads.
// ---------------------------------------------------------------------------
constexpr int kPlanThreads = 1024;

struct EntryView {
    uint64_t src, dst, size;
    bool valid;    // passes validation and size > 0
    bool aligned;  // src, dst and size multiples of 16
};

__device__ __forceinline__ bool in_table(const RangeTable& t, uint64_t p, uint64_t n) {
    for (uint32_t i = 0; i < t.n; ++i)
        if (p >= t.lo[i] && n <= t.hi[i] - t.lo[i] && p - t.lo[i] <= t.hi[i] - t.lo[i] - n) return true;
    return false;
}

// One tile of entries staged in shared memory by coalesced 8-byte loads (slot 0 holds the
// previous tile's last entry, so every entry can be compared with its predecessor).
struct PlanTile {
    uint64_t src[kPlanThreads + 1];
    uint64_t dst[kPlanThreads + 1];
    uint64_t size[kPlanThreads + 1];
};

// Loads entries [base, base + cnt) into tile slots 1..cnt.  Consecutive threads read
// consecutive words of the records (gfd_sg_entry: all 3 words; ring descriptor: its first
// 4 words), so a warp's loads coalesce into full sectors instead of one small request
// per field.  Ring descriptors also hand their flags and user_data to `meta_*` for the
// finalize kernel, which then never reads the ring again.
__device__ __forceinline__ void load_tile(const PlanArgs& a, uint64_t base, uint32_t cnt, PlanTile& tile) {
    if (a.kind == 0) {
        const char* rec0 = static_cast<const char*>(a.entries) + base * a.stride;
        for (uint32_t w = threadIdx.x; w < cnt * 3u; w += kPlanThreads) {
            const uint32_t k = w / 3u, f = w - k * 3u;
            const uint64_t v = *reinterpret_cast<const volatile uint64_t*>(rec0 + k * a.stride + 8u * f);
            if (f == 0) tile.dst[k + 1] = v;
            else if (f == 1) tile.src[k + 1] = v;
            else tile.size[k + 1] = v;
        }
    } else {
        for (uint32_t w = threadIdx.x; w < cnt * 4u; w += kPlanThreads) {
            const uint32_t k = w >> 2, f = w & 3u;
            const uint64_t slot = (a.ring_begin + base + k) % a.ring_size;
            const char* rec = static_cast<const char*>(a.entries) + slot * a.stride;
            const uint64_t v = *reinterpret_cast<const volatile uint64_t*>(rec + 8u * f);
            if (f == 0) {
                tile.src[k + 1] = v;
            } else if (f == 1) {
                tile.dst[k + 1] = v;
            } else if (f == 2) {
                tile.size[k + 1] = v & 0xffffffffull;  // size (u32), flags in the high half
                if (a.meta_flags != nullptr) a.meta_flags[base + k] = static_cast<uint32_t>(v >> 32);
            } else if (a.meta_user != nullptr) {
                a.meta_user[base + k] = v;
            }
        }
    }
}

__device__ __forceinline__ EntryView view_entry(const PlanArgs& a, const PlanTile& tile, uint32_t j,
                                                bool* rejected) {
    EntryView e;
    e.src = tile.src[j];
    e.dst = tile.dst[j];
    e.size = tile.size[j];
    const bool ok = in_table(a.src_ok, e.src, e.size) && in_table(a.dst_ok, e.dst, e.size);
    *rejected = (e.size > 0) && !ok;
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
    __shared__ unsigned long long s_wbytes[32];
    __shared__ uint32_t s_wheads[32];
    __shared__ uint32_t s_wmisc[32];
    __shared__ unsigned long long s_carry_bytes;
    __shared__ uint32_t s_carry_heads, s_carry_misc;
    __shared__ unsigned long long s_bad;
    __shared__ PlanTile s_tile;

    const int t = threadIdx.x;
    const int lane = t & 31, warp = t >> 5;
    if (t == 0) {
        s_carry_bytes = 0;
        s_carry_heads = 0;
        s_carry_misc = 0;
        s_bad = ~0ull;
    }
    __syncthreads();

    for (uint64_t base = 0; base < a.n; base += kPlanThreads) {
        const uint32_t cnt = static_cast<uint32_t>(a.n - base < kPlanThreads ? a.n - base : kPlanThreads);
        load_tile(a, base, cnt, s_tile);
        __syncthreads();
        const uint64_t i = base + t;
        EntryView e{0, 0, 0, false, false};
        bool head = false, misc = false, rejected = false;
        uint64_t sbytes = 0;
        if (i < a.n) {
            e = view_entry(a, s_tile, t + 1, &rejected);
            if (rejected) atomicMin(&s_bad, static_cast<unsigned long long>(i));
            if (e.valid && e.aligned) {
                sbytes = e.size;
                head = true;
                if (i > 0) {
                    bool prej;
                    const EntryView p = view_entry(a, s_tile, t, &prej);
                    if (p.valid && p.aligned && p.src + p.size == e.src && p.dst + p.size == e.dst)
                        head = false;
                }
            } else if (e.valid) {
                misc = true;
            }
        }
        // warp level: ballot for the 32-bit flags, shuffle scan for bytes
        const unsigned hmask = __ballot_sync(0xffffffffu, head);
        const unsigned mmask = __ballot_sync(0xffffffffu, misc);
        const unsigned lt = (1u << lane) - 1u;
        const uint32_t head_rank = __popc(hmask & lt);
        const uint32_t misc_rank = __popc(mmask & lt);
        const unsigned long long bincl = warp_incl_scan<unsigned long long>(sbytes, lane);
        if (lane == 31) {
            s_wbytes[warp] = bincl;
            s_wheads[warp] = __popc(hmask);
            s_wmisc[warp] = __popc(mmask);
        }
        __syncthreads();
        if (warp == 0) {
            const unsigned long long wb = s_wbytes[lane];
            const uint32_t wh = s_wheads[lane], wm = s_wmisc[lane];
            const unsigned long long ib = warp_incl_scan<unsigned long long>(wb, lane);
            const uint32_t ih = warp_incl_scan<uint32_t>(wh, lane);
            const uint32_t im = warp_incl_scan<uint32_t>(wm, lane);
            s_wbytes[lane] = ib - wb;  // exclusive per-warp offsets
            s_wheads[lane] = ih - wh;
            s_wmisc[lane] = im - wm;
        }
        __syncthreads();
        const unsigned long long cb = s_carry_bytes;
        const uint32_t ch = s_carry_heads, cm = s_carry_misc;
        if (head) {
            const uint32_t r = ch + s_wheads[warp] + head_rank;
            a.rows[r] = PullRow{e.src, e.dst, 0, cb + s_wbytes[warp] + (bincl - sbytes)};
        }
        if (misc) {
            const uint32_t m = cm + s_wmisc[warp] + misc_rank;
            a.misc[m] = PullRow{e.src, e.dst, e.size, 0};
        }
        __syncthreads();
        if (t == kPlanThreads - 1) {
            s_carry_bytes = cb + s_wbytes[31] + bincl;
            s_carry_heads = ch + s_wheads[31] + head_rank + (head ? 1u : 0u);
            s_carry_misc = cm + s_wmisc[31] + misc_rank + (misc ? 1u : 0u);
        }
        // the tile's last entry becomes the next tile's predecessor (slot 0)
        if (t == 0) {
            s_tile.src[0] = s_tile.src[cnt];
            s_tile.dst[0] = s_tile.dst[cnt];
            s_tile.size[0] = s_tile.size[cnt];
        }
        __syncthreads();
    }

    const uint64_t total = s_carry_bytes;
    const uint32_t n_rows = s_carry_heads;
    // row lengths from successive starts
    for (uint32_t r = t; r < n_rows; r += kPlanThreads) {
        const uint64_t end = (r + 1 < n_rows) ? a.rows[r + 1].start : total;
        a.rows[r].len = end - a.rows[r].start;
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
    return e;
}

cudaError_t launch_pull(const PullArgs& a, int grid, cudaStream_t st) {
    pull_kernel<<<grid, kPullThreads, 0, st>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_plan(const PlanArgs& a, cudaStream_t st) {
    plan_kernel<<<1, kPlanThreads, 0, st>>>(a);
    return cudaGetLastError();
}

}  // namespace gfdb
