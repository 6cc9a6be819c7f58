#pragma once
// Device-side data movers for pinned, device-mapped host memory -> HBM.
//
// This is the B200 replacement for the reference's CPU data path
// (AVX-512 streaming gather, src/parallel_gather.cpp:10-27, followed by a copy
// engine DMA, src/copy_engine.cpp:89-153): SM threads read host memory over PCIe
// with 16-byte vector loads that bypass L1 (ld.global.nc.L1::no_allocate.v4) and
// store straight to HBM.  A warp covers 512 contiguous bytes per load instruction
// (4 full 128-byte lines per request), and each thread keeps U loads in flight
// before its stores, so a 256-thread CTA has U * 4 KiB outstanding.
//
// Every routine writes exactly [dst, dst + n) and reads [src, src + n) -- except the
// warp-level shift path (warp_copy<U, true>) for sources and destinations that differ in
// their low two address bits, which reads the aligned 4-byte words covering the source
// range (at most three bytes on either side, in the same words and pages).  Heads and tails that are not
// 16-byte aligned are moved with narrower accesses.
//
// Included by the framework headers (warp_spec.cuh, sg_warp_spec.cuh), so it is
// compiled into user kernels as well as into libgfd_b200.

#include <cstdint>

namespace gfd {
namespace pull {

constexpr int kUnroll = 8;  // 16-byte loads in flight per thread

__device__ __forceinline__ uint4 ld_host_v4(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

__device__ __forceinline__ uint64_t ld_host_u64(const void* p) {
    uint64_t r;
    asm volatile("ld.global.nc.L1::no_allocate.u64 %0, [%1];" : "=l"(r) : "l"(p));
    return r;
}

__device__ __forceinline__ uint32_t ld_host_u32(const void* p) {
    uint32_t r;
    asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(r) : "l"(p));
    return r;
}

__device__ __forceinline__ uint32_t ld_host_u8(const void* p) {
    uint32_t r;
    asm volatile("ld.global.nc.L1::no_allocate.u8 %0, [%1];" : "=r"(r) : "l"(p));
    return r;
}

__device__ __forceinline__ void st_v4(void* p, uint4 v) {
    asm volatile("st.global.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z),
                 "r"(v.w)
                 : "memory");
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

// Vector body: nv 16-byte words, thread t of nt, U words in flight per thread.
template <int U>
__device__ __forceinline__ void copy_words16(char* dst, const char* src, uint64_t nv, uint32_t t,
                                             uint32_t nt) {
    const uint64_t sb = static_cast<uint64_t>(nt) * 16u;  // bytes between a thread's words
    const uint64_t nb = nv * 16u;
    uint64_t o = static_cast<uint64_t>(t) * 16u;
    for (; o + (U - 1) * sb < nb; o += U * sb) {
        uint4 r[U];
        const char* s = src + o;
#pragma unroll
        for (int u = 0; u < U; ++u) r[u] = ld_host_v4(s + u * sb);
        char* d = dst + o;
#pragma unroll
        for (int u = 0; u < U; ++u) st_v4(d + u * sb, r[u]);
    }
    // fewer than U words left for this thread: U/2 in flight at a time, each load
    // predicated on its word existing.  Re-reading an in-range word instead would cost
    // link bandwidth (repeated requests to one host line are not merged: 45.0 vs 51.4
    // GB/s for 14,336-byte rows), and U/2 keeps the framework kernels within their
    // register budget.
    constexpr int H = U > 1 ? U / 2 : 1;
    for (; o < nb; o += H * sb) {
        uint4 r[H];
#pragma unroll
        for (int u = 0; u < H; ++u)
            if (o + u * sb < nb) r[u] = ld_host_v4(src + o + u * sb);
#pragma unroll
        for (int u = 0; u < H; ++u)
            if (o + u * sb < nb) st_v4(dst + o + u * sb, r[u]);
    }
}

template <typename W, int U>
__device__ __forceinline__ void copy_words_narrow(char* dst, const char* src, uint64_t nw,
                                                  uint32_t t, uint32_t nt) {
    const uint64_t stride = static_cast<uint64_t>(nt);
    for (uint64_t v = t; v < nw; v += U * stride) {
        W r[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const uint64_t i = v + u * stride;
            if (i < nw) {
                if (sizeof(W) == 8) r[u] = (W)ld_host_u64(src + i * 8);
                else r[u] = (W)ld_host_u32(src + i * 4);
            }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const uint64_t i = v + u * stride;
            if (i < nw) reinterpret_cast<W*>(dst)[i] = r[u];
        }
    }
}

__device__ __forceinline__ void copy_bytes(char* dst, const char* src, uint64_t n, uint32_t t,
                                           uint32_t nt) {
    for (uint64_t i = t; i < n; i += nt) dst[i] = static_cast<char>(ld_host_u8(src + i));
}

// One warp, destination 4-byte aligned, source off by r = src & 3 (1..3): each 4-byte
// destination word is funnel-shifted out of two consecutive source-aligned words.  Every
// source word is loaded once (a lane takes its neighbour's word with a shuffle; lane 31
// loads the word after its block), U words in flight per lane.  The aligned words
// covering [src, src + 4 * nw) are read whole: up to three bytes before src and after the
// last byte, always inside the aligned words (and so the pages) that hold the range.
template <int U>
__device__ __noinline__ void copy_shift4_warp(uint32_t* dw, const char* src, uint64_t nw, uint32_t lane) {
    const uint32_t r = static_cast<uint32_t>(reinterpret_cast<uint64_t>(src) & 3u);
    const uint32_t* sw = reinterpret_cast<const uint32_t*>(src - r);
    for (uint64_t j0 = 0; j0 < nw; j0 += 32u * U) {
        uint32_t lo[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const uint64_t j = j0 + static_cast<uint64_t>(u) * 32u + lane;
            lo[u] = j <= nw ? ld_host_u32(sw + j) : 0u;  // word nw holds the last source bytes
        }
        const uint64_t after = j0 + 32u * U;  // first word of the next block
        const uint32_t extra = (lane == 31 && after <= nw) ? ld_host_u32(sw + after) : 0u;
#pragma unroll
        for (int u = 0; u < U; ++u) {
            uint32_t hi = __shfl_down_sync(0xffffffffu, lo[u], 1);
            const uint32_t row_next = u + 1 < U ? __shfl_sync(0xffffffffu, lo[u + 1 < U ? u + 1 : u], 0) : extra;
            if (lane == 31) hi = row_next;
            const uint64_t j = j0 + static_cast<uint64_t>(u) * 32u + lane;
            if (j < nw) dw[j] = __funnelshift_r(lo[u], hi, 8u * r);
        }
    }
}

// Cooperative copy of one span by nt threads (thread index t).  Any alignment.
template <int U = kUnroll>
__device__ __forceinline__ void group_copy(void* dst_, const void* src_, uint64_t n, uint32_t t,
                                           uint32_t nt) {
    char* dst = static_cast<char*>(dst_);
    const char* src = static_cast<const char*>(src_);
    const uint64_t s = reinterpret_cast<uint64_t>(src);
    const uint64_t d = reinterpret_cast<uint64_t>(dst);
    uint32_t gran = 1;
    if (((s ^ d) & 15) == 0) gran = 16;
    else if (((s ^ d) & 7) == 0) gran = 8;
    else if (((s ^ d) & 3) == 0) gran = 4;
    if (gran == 1 || n < 2 * gran) {
        copy_bytes(dst, src, n, t, nt);
        return;
    }
    uint64_t head = (gran - (s & (gran - 1))) & (gran - 1);
    copy_bytes(dst, src, head, t, nt);
    dst += head;
    src += head;
    n -= head;
    const uint64_t nw = n / gran;
    if (gran == 16) copy_words16<U>(dst, src, nw, t, nt);
    else if (gran == 8) copy_words_narrow<uint64_t, U>(dst, src, nw, t, nt);
    else copy_words_narrow<uint32_t, U>(dst, src, nw, t, nt);
    const uint64_t body = nw * gran;
    copy_bytes(dst + body, src + body, n - body, t, nt);
}

// Whole-warp copy (all 32 lanes call with identical arguments).  With Shift, sources and
// destinations that differ in their low two address bits take the funnel-shift path
// (4-byte words) instead of byte copies; the frameworks' kernels, which keep a tight
// register budget, call it without.
template <int U = kUnroll, bool Shift = false>
__device__ __forceinline__ void warp_copy(void* dst_, const void* src_, uint64_t n) {
    const uint32_t lane = threadIdx.x & 31u;
    if (Shift) {
        char* dst = static_cast<char*>(dst_);
        const char* src = static_cast<const char*>(src_);
        const uint64_t d = reinterpret_cast<uint64_t>(dst);
        if (((reinterpret_cast<uint64_t>(src) ^ d) & 3u) != 0 && n >= 64) {
            const uint64_t head = (4u - (d & 3u)) & 3u;
            copy_bytes(dst, src, head, lane, 32u);
            const uint64_t nw = (n - head) >> 2;
            copy_shift4_warp<U>(reinterpret_cast<uint32_t*>(dst + head), src + head, nw, lane);
            const uint64_t done = head + nw * 4u;
            copy_bytes(dst + done, src + done, n - done, lane, 32u);
            return;
        }
    }
    group_copy<U>(dst_, src_, n, lane, 32u);
}

}  // namespace pull
}  // namespace gfd
