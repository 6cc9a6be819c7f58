// Ring agent kernel: the device-resident consumer of the descriptor ring (see agent.h).
//
// CTA 0 ("front") owns the ring: warp 0 polls the commit markers, then the whole CTA
// copies each committed run out (four 8-byte fields per 64-byte descriptor), clears the
// markers, validates, accounts and plans the run into a batch of pull rows; CTAs 1..M
// ("movers") pull the batches with the pull kernel's body (pull_body.cuh).  Every wait is
// bounded on %globaltimer; a wait that gives up is counted in AgentHost::timeouts and
// ends the launch with kAgentError, so the host sees a status instead of a stuck GPU.
//
// Memory ordering follows the ring protocol of the reference (include/gfd/device.cuh:
// 78-100): producers write a descriptor, fence at system scope, then store
// sequence = slot + 1.  The front reads the markers (relaxed, system scope), fences
// (acquire), and only then reads the fields; it clears the markers of a batch only after
// every field of the batch has been read (and the batch handed to the movers), and
// publishes read_idx after its clears are visible.
// done_idx is published by the last mover of a batch after a system-scope fence that
// follows every mover's payload stores, so a kernel that sees done_idx >= slot + 1 sees
// the bytes.

#include <cuda_runtime.h>

#include <cstdint>

#include "agent.h"
#include "gfd/sg_task_queue.h"
#include "gfd/tiled_queue.h"
#include "gfd/wait.cuh"
#include "pull_body.cuh"

namespace gfdb {
namespace {

__device__ __forceinline__ uint64_t ld_relaxed_sys(const void* p) {
    uint64_t v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void st_relaxed_sys(void* p, uint64_t v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void st_release_gpu(uint32_t* p, uint32_t v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ void fence_acquire_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

__device__ __forceinline__ bool in_range(const AgentRanges& t, uint32_t i, uint64_t p, uint64_t n) {
    const uint64_t lo = t.lo[i], hi = t.hi[i];
    return p >= lo && n <= hi - lo && p - lo <= hi - lo - n;
}

// Range check with a per-thread hint (consecutive descriptors almost always hit the range
// the previous one did).
__device__ __forceinline__ bool known(const AgentRanges& t, uint64_t p, uint64_t n, uint32_t& hint) {
    const uint32_t cnt = t.n < kAgentRanges ? t.n : kAgentRanges;
    if (hint < cnt && in_range(t, hint, p, n)) return true;
    for (uint32_t i = 0; i < cnt; ++i)
        if (in_range(t, i, p, n)) {
            hint = i;
            return true;
        }
    return false;
}

__device__ __forceinline__ void note_timeout(const AgentArgs& a) {
    atomicAdd(reinterpret_cast<unsigned long long*>(const_cast<uint64_t*>(&a.host->timeouts)), 1ull);
}

// Asks the host whether [p, p + n) lies in an allocation of the given kind (0: pinned host
// memory mapped at the same address, 1: device memory of this GPU) and caches the
// allocation's range in the front's table `t`.  One thread; bounded.
__device__ bool ask_host(const AgentArgs& a, AgentRanges& t, uint32_t kind, uint64_t p, uint64_t n, uint32_t& seq) {
    AgentHost* h = a.host;
    ++seq;
    h->q_kind = kind;
    h->q_addr = p;
    h->q_size = n;
    __threadfence_system();
    h->q_seq = seq;
    __threadfence_system();
    atomicAdd(reinterpret_cast<unsigned long long*>(const_cast<uint64_t*>(&h->queries)), 1ull);
    const uint64_t t0 = gfd::wait::now();
    uint32_t polls = 0;
    while (gfd::wait::load_acquire_sys(&h->a_seq) != seq) {
        if (gfd::wait::expired(t0, a.wait_limit_ns)) {
            note_timeout(a);
            return false;
        }
        gfd::wait::backoff(polls);
    }
    if (gfd::wait::load_acquire_sys(&h->a_ok) == 0) return false;
    const uint64_t lo = h->a_lo, hi = h->a_hi;
    if (!(lo <= p && n <= hi - lo && p - lo <= hi - lo - n)) return false;
    // the host also keeps the range, so the next launch's tables hold it
    const uint32_t i = t.n < kAgentRanges ? t.n++ : (t.evict++ % kAgentRanges);
    t.lo[i] = lo;
    t.hi[i] = hi;
    return true;
}

// ---------------------------------------------------------------------------
// Front
// ---------------------------------------------------------------------------
struct ScanParts {
    unsigned long long bytes[33];
    uint32_t heads[33];
    uint32_t miscs[33];
};

struct FrontSmem {
    AgentRanges tab[2];             // [0] sources, [1] destinations: the launch's tables, plus
                                    // ranges learnt from the host during the launch
    // one staged tile of descriptors; index 0 holds the descriptor before the tile
    uint64_t src[kAgentTile + 1];
    uint64_t dst[kAgentTile + 1];
    uint64_t sf[kAgentTile + 1];    // size | flags << 32
    uint64_t user[kAgentTile + 1];
    uint32_t counts[kEpiTiles];     // tokens per tile id in the current batch
    ScanParts scan;
    unsigned long long first_bad;   // first rejected slot in the batch, or ~0
    uint32_t bad, need_query, n_lists, lists_landed, n_tiles;
    uint32_t run, stop, exit_reason, go;
};

struct MoverSmem {
    PullRow srow[kRowWindow];
    uint32_t batch_ok;
    uint32_t last;
};

template <typename T>
__device__ __forceinline__ T warp_incl_scan(T x, int lane) {
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const T y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    return x;
}

struct Counts {
    uint32_t heads, miscs;
    unsigned long long bytes;
};

// Block-wide exclusive scan of per-thread counts; *tot gets the block totals.
__device__ __forceinline__ Counts block_scan(const Counts& c, ScanParts& sm, Counts* tot) {
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
        const int nw = kAgentThreads / 32;
        const unsigned long long wb = lane < nw ? sm.bytes[lane] : 0ull;
        const uint32_t wh = lane < nw ? sm.heads[lane] : 0u, wm = lane < nw ? sm.miscs[lane] : 0u;
        const unsigned long long xb = warp_incl_scan<unsigned long long>(wb, lane);
        const uint32_t xh = warp_incl_scan<uint32_t>(wh, lane);
        const uint32_t xm = warp_incl_scan<uint32_t>(wm, lane);
        if (lane < nw) {
            sm.bytes[lane] = xb - wb;
            sm.heads[lane] = xh - wh;
            sm.miscs[lane] = xm - wm;
        }
        if (lane == 31) {
            sm.bytes[32] = xb;
            sm.heads[32] = xh;
            sm.miscs[32] = xm;
        }
    }
    __syncthreads();
    Counts o;
    o.heads = sm.heads[warp] + ih - c.heads;
    o.miscs = sm.miscs[warp] + im - c.miscs;
    o.bytes = sm.bytes[warp] + ib - c.bytes;
    tot->heads = sm.heads[32];
    tot->miscs = sm.miscs[32];
    tot->bytes = sm.bytes[32];
    __syncthreads();  // scratch free for the next scan
    return o;
}

// Committed run at `next` (at most cap slots), read by warp 0: the first window is one
// marker per lane, later windows sixteen per lane.  Lane 0 also reads the stop word.
__device__ __forceinline__ uint32_t poll_run(const AgentArgs& a, uint64_t next, uint32_t cap, uint32_t* stop) {
    const uint32_t lane = threadIdx.x & 31;
    if (lane == 0) *stop = a.host->stop;
    uint32_t n = 0;
    bool first = true;
    while (n < cap) {
        const uint32_t w = first ? 1u : 16u;
        const uint32_t n0 = n;  // the window starts at slot next + n0
        uint64_t seq[16];
#pragma unroll
        for (uint32_t k = 0; k < 16; ++k) {
            seq[k] = 0;
            const uint32_t i = k * 32u + lane;
            if (k < w && i < cap - n0)
                seq[k] = ld_relaxed_sys(
                    const_cast<const uint64_t*>(&a.q->entries[(next + n0 + i) % gfd::QUEUE_SIZE].sequence));
        }
        bool gap = false;
#pragma unroll
        for (uint32_t k = 0; k < 16; ++k) {
            if (k >= w || gap) break;
            const uint32_t i = k * 32u + lane;
            const bool ok = i < cap - n0 && seq[k] == next + n0 + i + 1;
            const uint32_t mask = __ballot_sync(0xffffffffu, ok);
            if (mask == 0xffffffffu) {
                n += 32;
            } else {
                n += static_cast<uint32_t>(__ffs(~mask)) - 1;
                gap = true;
            }
        }
        if (gap) break;
        first = false;
    }
    return n < cap ? n : cap;
}

// Copies slots [s, s + n) out of the ring into batch B: fields, validation, per-tile /
// per-list accounting, run merging and the movers' row tables.
__device__ void plan_batch(const AgentArgs& a, FrontSmem& sm, AgentBatch* B, uint64_t s, uint32_t n, uint32_t& seq) {
    const uint32_t tid = threadIdx.x;
    const bool tiled = a.tile_done != nullptr, sg = a.list_done != nullptr || a.lists_completed != nullptr;
    uint32_t src_hint = 0, dst_hint = 0;
    if (tid == 0) {
        sm.first_bad = ~0ull;
        sm.bad = 0;
        sm.need_query = 0;
        sm.n_lists = 0;
        sm.lists_landed = 0;
        sm.n_tiles = 0;
    }
    unsigned long long c_bytes = 0;  // carries over the tiles (uniform)
    uint32_t c_heads = 0, c_miscs = 0;
    __syncthreads();

    for (uint32_t base = 0; base < n; base += kAgentTile) {
        const uint32_t cnt = n - base < kAgentTile ? n - base : kAgentTile;
        // 1. fields: word f of descriptor d is read by thread (4 d + f) mod 256, so a warp
        //    reads eight descriptors' 32-byte heads per instruction; all loads in flight
        {
            constexpr int kW = kAgentTile * 4 / kAgentThreads;  // 16 words per thread
            uint64_t v[kW];
#pragma unroll
            for (int j = 0; j < kW; ++j) {
                const uint32_t w = tid + static_cast<uint32_t>(j) * kAgentThreads;
                const uint32_t d = w >> 2, f = w & 3u;
                v[j] = 0;
                if (d < cnt) {
                    const gfd::Descriptor* e = &a.q->entries[(s + base + d) % gfd::QUEUE_SIZE];
                    v[j] = ld_relaxed_sys(reinterpret_cast<const char*>(e) + 8u * f);
                }
            }
#pragma unroll
            for (int j = 0; j < kW; ++j) {
                const uint32_t w = tid + static_cast<uint32_t>(j) * kAgentThreads;
                const uint32_t d = w >> 2, f = w & 3u;
                if (d < cnt) {
                    uint64_t* dstv = f == 0 ? sm.src : f == 1 ? sm.dst : f == 2 ? sm.sf : sm.user;
                    dstv[d + 1] = v[j];
                }
            }
        }
        __syncthreads();
        // 2. ranges never seen before are checked by the host, once (the markers are
        //    cleared by release_slots once the batch is published)
        const uint32_t j0 = tid * 4u + 1u;  // this thread's slots in the tile (1-based)
        for (uint32_t k = 0; k < 4; ++k) {
            const uint32_t j = j0 + k;
            if (j > cnt) break;
            const uint64_t size = sm.sf[j] & 0xffffffffull;
            if (size != 0 && (!known(sm.tab[0], sm.src[j], size, src_hint) || !known(sm.tab[1], sm.dst[j], size, dst_hint)))
                sm.need_query = 1;
        }
        __syncthreads();
        if (sm.need_query) {
            if (tid == 0) {
                uint32_t asked = 0, h0 = 0, h1 = 0;
                for (uint32_t j = 1; j <= cnt; ++j) {
                    const uint64_t size = sm.sf[j] & 0xffffffffull;
                    if (size == 0) continue;
                    if (!known(sm.tab[0], sm.src[j], size, h0) && asked < kAgentMaxQueries) {
                        ++asked;
                        ask_host(a, sm.tab[0], 0, sm.src[j], size, seq);
                    }
                    if (!known(sm.tab[1], sm.dst[j], size, h1) && asked < kAgentMaxQueries) {
                        ++asked;
                        ask_host(a, sm.tab[1], 1, sm.dst[j], size, seq);
                    }
                }
                sm.need_query = 0;
            }
            __syncthreads();
        }
        // 3. classify the thread's four consecutive descriptors
        Counts c{0, 0, 0};
        uint32_t hbits = 0, mbits = 0, sbits = 0;
        {
            const bool has_prev0 = base + j0 - 1 > 0;
            uint64_t psrc = sm.src[j0 - 1], pdst = sm.dst[j0 - 1];
            uint64_t psize = sm.sf[j0 - 1] & 0xffffffffull;
            bool pchain = has_prev0 && psize != 0 && ((psrc | pdst | psize) & 15u) == 0 &&
                          known(sm.tab[0], psrc, psize, src_hint) && known(sm.tab[1], pdst, psize, dst_hint);
            for (uint32_t k = 0; k < 4; ++k) {
                const uint32_t j = j0 + k;
                if (j > cnt) break;
                const uint64_t src = sm.src[j], dst = sm.dst[j], size = sm.sf[j] & 0xffffffffull;
                const uint32_t flags = static_cast<uint32_t>(sm.sf[j] >> 32);
                const uint32_t id = static_cast<uint32_t>(sm.user[j] >> 32);
                if (tiled && id < static_cast<uint32_t>(gfd::MAX_TILES)) atomicAdd(&sm.counts[id], 1u);
                if (sg && (flags & gfd::FLAG_LAST_IN_TILE) && id < static_cast<uint32_t>(gfd::MAX_SG_LISTS)) {
                    const uint32_t li = atomicAdd(&sm.n_lists, 1u);
                    if (li < static_cast<uint32_t>(kEpiLists)) B->list_id[li] = static_cast<uint16_t>(id);
                    atomicAdd(&sm.lists_landed, 1u);
                }
                const bool valid = size != 0 && known(sm.tab[0], src, size, src_hint) &&
                                   known(sm.tab[1], dst, size, dst_hint);
                if (size != 0 && !valid) {
                    atomicAdd(&sm.bad, 1u);
                    atomicMin(&sm.first_bad, static_cast<unsigned long long>(s + base + j - 1));
                }
                const bool aligned = ((src | dst | size) & 15u) == 0;
                bool chain = false;
                if (valid && aligned) {
                    if (!(pchain && psrc + psize == src && pdst + psize == dst)) {
                        hbits |= 1u << k;
                        ++c.heads;
                    }
                    sbits |= 1u << k;
                    c.bytes += size;
                    chain = true;
                } else if (valid) {
                    mbits |= 1u << k;
                    ++c.miscs;
                }
                psrc = src;
                pdst = dst;
                psize = size;
                pchain = chain;
            }
        }
        // 4. rows at their scanned positions
        Counts tot;
        const Counts o = block_scan(c, sm.scan, &tot);
        if (sbits | mbits) {
            uint32_t r = c_heads + o.heads, m = c_miscs + o.miscs;
            uint64_t off = c_bytes + o.bytes;
            for (uint32_t k = 0; k < 4; ++k) {
                const uint32_t j = j0 + k;
                if (j > cnt) break;
                const uint64_t size = sm.sf[j] & 0xffffffffull;
                if (sbits & (1u << k)) {
                    // a continuation only extends the stream; row lengths come from the
                    // starts once the whole batch is planned
                    if (hbits & (1u << k)) B->rows[r++] = PullRow{sm.src[j], sm.dst[j], 0, off};
                    off += size;
                } else if (mbits & (1u << k)) {
                    B->misc[m++] = PullRow{sm.src[j], sm.dst[j], size, 0};
                }
            }
        }
        c_heads += tot.heads;
        c_miscs += tot.miscs;
        c_bytes += tot.bytes;
        __syncthreads();
        if (tid == 0) {  // the tile's last descriptor precedes the next tile
            sm.src[0] = sm.src[cnt];
            sm.dst[0] = sm.dst[cnt];
            sm.sf[0] = sm.sf[cnt];
            sm.user[0] = sm.user[cnt];
        }
        __syncthreads();
    }
    // row lengths from successive starts (a row may continue across threads and tiles), and
    // each mover's first row: the row holding the first byte of its range
    uint64_t per = (c_bytes + a.movers - 1) / a.movers;
    per = (per + kPiece - 1) / kPiece * kPiece;
    if (per == 0) per = kPiece;
    __syncthreads();
    for (uint32_t r = tid; r < c_heads; r += kAgentThreads) {
        const uint64_t start = B->rows[r].start;
        const uint64_t end = r + 1 < c_heads ? B->rows[r + 1].start : c_bytes;
        B->rows[r].len = end - start;
        for (uint64_t m = (start + per - 1) / per; m * per < end && m < a.movers; ++m)
            B->cta_first[m] = r;
    }
    for (uint32_t m = tid; m < a.movers; m += kAgentThreads)
        if (static_cast<uint64_t>(m) * per >= c_bytes) B->cta_first[m] = 0;  // no stream work
    // per-tile counts, compacted (ids distinct within a batch); the scratch is zeroed again
    for (uint32_t t = tid; t < static_cast<uint32_t>(kEpiTiles); t += kAgentThreads) {
        const uint32_t v = sm.counts[t];
        if (v != 0) {
            const uint32_t k = atomicAdd(&sm.n_tiles, 1u);
            B->tile_id[k] = static_cast<uint16_t>(t);
            B->tile_count[k] = v;
            sm.counts[t] = 0;
        }
    }
    __syncthreads();
    if (tid == 0) {
        B->begin = s;
        B->end = s + n;
        B->total = c_bytes;
        B->per_cta = per;
        B->n_rows = c_heads;
        B->n_misc = c_miscs;
        B->n_tiles = sm.n_tiles;
        B->n_lists = sm.n_lists < static_cast<uint32_t>(kEpiLists) ? sm.n_lists : static_cast<uint32_t>(kEpiLists);
        B->lists_landed = sm.lists_landed;
        B->ctas_done = 0;
        if (sm.bad != 0) {
            atomicAdd(reinterpret_cast<unsigned long long*>(const_cast<uint64_t*>(&a.host->rejected)),
                      static_cast<unsigned long long>(sm.bad));
            if (a.host->first_bad == 0) a.host->first_bad = sm.first_bad + 1;
        }
    }
    __syncthreads();
}

// Clears the markers of slots [s, s + n) -- every field of them was read in plan_batch --
// and makes the clears visible before the caller publishes read_idx.
__device__ void release_slots(const AgentArgs& a, uint64_t s, uint32_t n) {
    for (uint32_t d = threadIdx.x; d < n; d += kAgentThreads)
        st_relaxed_sys(const_cast<uint64_t*>(&a.q->entries[(s + d) % gfd::QUEUE_SIZE].sequence), 0ull);
    __threadfence_system();
    __syncthreads();
}

__device__ void front(const AgentArgs& a, FrontSmem& sm) {
    const uint32_t tid = threadIdx.x;
    AgentDev* dev = a.dev;
    for (uint32_t t = tid; t < static_cast<uint32_t>(kEpiTiles); t += kAgentThreads) sm.counts[t] = 0;
    {
        const uint64_t* g = reinterpret_cast<const uint64_t*>(&dev->src);
        uint64_t* l = reinterpret_cast<uint64_t*>(&sm.tab[0]);
        static_assert(sizeof(AgentRanges) % 8 == 0 && offsetof(AgentDev, dst) == sizeof(AgentRanges), "tables");
        for (uint32_t i = tid; i < 2 * sizeof(AgentRanges) / 8; i += kAgentThreads) l[i] = g[i];
    }
    uint32_t seq = a.host->q_seq;  // mailbox numbering continues across launches
    uint64_t next = a.start_slot;
    uint32_t gen = 0;
    uint64_t last_active = gfd::wait::now();
    uint64_t grow_since = 0;
    uint32_t polls = 0;
    uint32_t reason = kAgentRunning;
    if (tid == 0) {
        a.host->t_start = last_active;
        a.host->t_first = 0;
        a.host->reset_ok = 0;
    }
    // no batch is published before every mover runs: each mover then sees every batch of
    // the launch from the first one (a mover that starts late finds `exit` set and leaves)
    if (tid == 0) {
        const uint64_t t0 = gfd::wait::now();
        uint32_t p = 0;
        sm.exit_reason = kAgentRunning;
        while (ld_acquire_gpu(&dev->started) != gridDim.x) {
            if (gfd::wait::expired(t0, a.wait_limit_ns)) {
                note_timeout(a);
                sm.exit_reason = kAgentError;
                break;
            }
            gfd::wait::backoff(p);
        }
    }
    __syncthreads();
    reason = sm.exit_reason;
    for (; reason == kAgentRunning;) {
        uint32_t done = 0;
        if (tid == 0) done = ld_acquire_gpu(&dev->done);
        done = __shfl_sync(0xffffffffu, done, 0);
        if (threadIdx.x < 32) {
            const uint32_t cap = gen == done ? kAgentEagerBatch : kAgentBatchMax;
            uint32_t stop = 0;
            const uint32_t n = poll_run(a, next, cap, &stop);
            if (tid == 0) {
                sm.run = n;
                sm.stop = stop;
                sm.go = 0;
                sm.exit_reason = kAgentRunning;
                const uint64_t now = gfd::wait::now();
                if (n == 0) {
                    grow_since = 0;
                    const uint64_t idle = now - last_active;
                    if (gen == done && stop) sm.exit_reason = kAgentStopped;
                    else if (gen == done && ((!a.resident && idle > a.linger_ns) || idle > a.idle_limit_ns))
                        sm.exit_reason = kAgentIdle;
                } else if (n < 256 && gen != done && !stop) {
                    // the movers are busy and the run is short: give it a few microseconds
                    // to grow before it becomes a batch of its own
                    if (grow_since == 0) grow_since = now;
                    sm.go = now - grow_since > 4000;
                } else {
                    sm.go = 1;
                }
                last_active = n != 0 ? now : last_active;
            }
            __syncwarp();
        }
        __syncthreads();
        if (sm.exit_reason != kAgentRunning) {
            reason = sm.exit_reason;
            break;
        }
        if (!sm.go) {
            if (tid == 0) {
                ++polls;
                if (polls > 32) __nanosleep(sm.run == 0 ? (polls > 256 ? 1000 : 200) : 500);
            }
            __syncthreads();
            continue;
        }
        polls = 0;
        const uint32_t n = sm.run;
        fence_acquire_sys();  // the fields below are read after the markers that published them
        // a free batch slot
        if (tid == 0) {
            const uint64_t t0 = gfd::wait::now();
            uint32_t p = 0;
            sm.exit_reason = kAgentRunning;
            while (gen - ld_acquire_gpu(&dev->done) >= static_cast<uint32_t>(kAgentSlots)) {
                if (gfd::wait::expired(t0, a.wait_limit_ns)) {
                    note_timeout(a);
                    sm.exit_reason = kAgentError;
                    break;
                }
                gfd::wait::backoff(p);
            }
        }
        __syncthreads();
        if (sm.exit_reason != kAgentRunning) {
            reason = sm.exit_reason;
            break;
        }
        AgentBatch* B = &dev->batch[gen % kAgentSlots];
        plan_batch(a, sm, B, next, n, seq);
        if (tid == 0) {  // the movers start on the batch at once
            __threadfence();
            st_release_gpu(&dev->gen, gen + 1);
            if (gen == 0) a.host->t_first = gfd::wait::now();
        }
        // then the slots go back to the producers
        release_slots(a, next, n);
        if (tid == 0) {
            *reinterpret_cast<volatile uint64_t*>(&a.q->read_idx) = next + n;
            if (a.mirror != nullptr) a.mirror->read_idx = next + n;
            __threadfence();
        }
        ++gen;
        next += n;
        grow_since = 0;
        last_active = gfd::wait::now();
        __syncthreads();
    }
    if (tid == 0) {
        // every published batch completes before the movers are told to leave
        const uint64_t t0 = gfd::wait::now();
        uint32_t p = 0;
        while (ld_acquire_gpu(&dev->done) != gen) {
            if (gfd::wait::expired(t0, a.wait_limit_ns)) {
                note_timeout(a);
                reason = kAgentError;
                break;
            }
            gfd::wait::backoff(p);
        }
        st_release_gpu(&dev->exit, 1u);
        // once every mover has left, zero the launch counters for the next launch (the
        // host clears them itself when this does not happen in time)
        bool clean = false;
        {
            const uint64_t t1 = gfd::wait::now();
            uint32_t p1 = 0;
            for (;;) {
                if (ld_acquire_gpu(&dev->left) == a.movers) {
                    clean = true;
                    break;
                }
                if (gfd::wait::expired(t1, a.wait_limit_ns)) {
                    note_timeout(a);
                    break;
                }
                gfd::wait::backoff(p1);
            }
        }
        if (clean) {
            dev->gen = 0;
            dev->done = 0;
            dev->exit = 0;
            dev->started = 0;
            dev->left = 0;
            __threadfence();
        }
        a.host->next = next;
        a.host->status = reason;
        a.host->exits[reason < 4 ? reason : 0] += 1;
        a.host->reset_ok = clean ? 1u : 0u;
        a.host->t_exit = gfd::wait::now();
        __threadfence_system();
        a.host->exited = a.launch_id;
        __threadfence_system();
    }
}

// ---------------------------------------------------------------------------
// Movers
// ---------------------------------------------------------------------------
// Completion of batch B by the last mover: per-tile counts, per-list flags, then
// lists_completed and done_idx in host memory, then the device copy of done_idx
// (reference src/batch_processor.cpp:69-446 publishes the same effects).
__device__ void complete_batch(const AgentArgs& a, const AgentBatch* B) {
    __threadfence();  // after every mover's payload stores (they fenced before counting in)
    if (a.tile_done != nullptr)
        for (uint32_t i = threadIdx.x; i < B->n_tiles; i += blockDim.x) {
            volatile uint64_t* p = &a.tile_done[B->tile_id[i]];
            *p = *p + B->tile_count[i];  // batches complete in order, ids distinct within one
        }
    if (a.list_done != nullptr)
        for (uint32_t i = threadIdx.x; i < B->n_lists; i += blockDim.x)
            *reinterpret_cast<volatile uint64_t*>(&a.list_done[B->list_id[i]]) = 1;
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        if (a.lists_completed != nullptr && B->lists_landed != 0)
            *a.lists_completed = *a.lists_completed + B->lists_landed;
        *reinterpret_cast<volatile uint64_t*>(&a.q->done_idx) = B->end;
        __threadfence_system();
        if (a.mirror != nullptr && a.mirror->done_idx < B->end) a.mirror->done_idx = B->end;
        atomicAdd(&a.dev->consumed, static_cast<unsigned long long>(B->end - B->begin));
        atomicAdd(&a.dev->batches, 1ull);
        a.host->t_done = gfd::wait::now();
        __threadfence();
    }
}

__device__ void mover(const AgentArgs& a, MoverSmem& sm) {
    const uint32_t m = blockIdx.x - 1;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    AgentDev* dev = a.dev;
    const uint64_t bound = a.idle_limit_ns + a.wait_limit_ns;
    for (uint32_t b = 0;; ++b) {
        if (threadIdx.x == 0) {
            const uint64_t t0 = gfd::wait::now();
            uint32_t p = 0;
            sm.batch_ok = 0;
            for (;;) {
                if (ld_acquire_gpu(&dev->gen) > b) {
                    sm.batch_ok = 1;
                    break;
                }
                if (ld_acquire_gpu(&dev->exit) != 0) break;
                if (gfd::wait::expired(t0, bound)) {
                    note_timeout(a);
                    break;
                }
                ++p;
                if (p > 64) __nanosleep(p < 1024 ? 64 : 512);
            }
        }
        __syncthreads();
        if (!sm.batch_ok) {
            if (threadIdx.x == 0) {
                __threadfence();
                atomicAdd(&dev->left, 1u);
            }
            return;
        }
        // each thread acquires the publication itself: the slot's previous batch may still
        // sit in this SM's L1
        (void)ld_acquire_gpu(&dev->gen);
        AgentBatch* B = &dev->batch[b % kAgentSlots];
        const uint64_t total = B->total, per = B->per_cta;
        const uint32_t n_rows = B->n_rows;
        const uint64_t lo = static_cast<uint64_t>(m) * per;
        const uint64_t hi = lo + per < total ? lo + per : total;
        uint64_t moved = 0;
        if (lo < hi) {
            const uint32_t r0 = B->cta_first[m];
            uint32_t r_end = n_rows;
            if (hi < total && m + 1 < a.movers) {
                const uint32_t nxt = B->cta_first[m + 1] + 1;
                if (nxt < r_end) r_end = nxt;
            }
            pull_stream_range(B->rows, n_rows, total, false, lo, hi, r0, r_end, sm.srow);
            if (threadIdx.x == 0) moved = hi - lo;
        }
        const uint64_t mm = pull_misc_rows(B->misc, B->n_misc, m * kPullWarps + warp, a.movers * kPullWarps);
        if (lane == 0) moved += mm;
        if (a.bytes_ctr != nullptr && lane == 0 && moved != 0)
            atomicAdd(a.bytes_ctr, static_cast<unsigned long long>(moved));
        __syncthreads();
        if (threadIdx.x == 0) {
            __threadfence();  // this CTA's stores (ordered by the barrier) before its count
            const uint32_t prev = atomicAdd(&B->ctas_done, 1u);
            sm.last = prev == a.movers - 1;
        }
        __syncthreads();
        if (sm.last) {
            complete_batch(a, B);
            if (threadIdx.x == 0) {
                B->ctas_done = 0;
                __threadfence();
                st_release_gpu(&dev->done, b + 1);
            }
        }
        __syncthreads();
    }
}

union AgentSmem {
    FrontSmem front;
    MoverSmem mover;
};

__global__ void __launch_bounds__(kAgentThreads) ring_agent_kernel(const __grid_constant__ AgentArgs a) {
    __shared__ AgentSmem smem;
    if (threadIdx.x == 0) {
        // the host waits for every CTA of the launch to run before returning from start
        if (atomicAdd(&a.dev->started, 1u) == gridDim.x - 1) {
            a.host->resident = a.launch_id;
            __threadfence_system();
        }
    }
    if (blockIdx.x == 0) front(a, smem.front);
    else mover(a, smem.mover);
}

}  // namespace

cudaError_t launch_agent(const AgentArgs& a, cudaStream_t st) {
    ring_agent_kernel<<<1 + a.movers, kAgentThreads, 0, st>>>(a);
    return cudaGetLastError();
}

cudaError_t preload_agent() {
    cudaFuncAttributes fa;
    return cudaFuncGetAttributes(&fa, ring_agent_kernel);
}

}  // namespace gfdb
