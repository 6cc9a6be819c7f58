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
