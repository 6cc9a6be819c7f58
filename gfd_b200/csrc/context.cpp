// libgfd_b200 host side: contexts, host pools, entry validation, host-built pull
// tables and the direct-submit entry points of the C ABI (include/gfd_b200.h).

#include <cuda.h>
#include <cuda_runtime.h>
#include <sys/mman.h>
#include <sys/syscall.h>
#include <time.h>
#include <unistd.h>

#include <algorithm>
#include <cerrno>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <new>

#if defined(__x86_64__)
#include <immintrin.h>
#endif

#include "host_mem.h"
#include "internal.h"
#include "numa_pool.h"

namespace gfdb {

uint64_t now_ns() {
    timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return static_cast<uint64_t>(ts.tv_sec) * 1000000000ull + static_cast<uint64_t>(ts.tv_nsec);
}

static inline void cpu_relax() {
#if defined(__x86_64__)
    _mm_pause();
#endif
}

int set_error(gfd_ctx* ctx, int code, const char* fmt, ...) {
    if (ctx != nullptr) {
        char buf[512];
        va_list ap;
        va_start(ap, fmt);
        vsnprintf(buf, sizeof(buf), fmt, ap);
        va_end(ap);
        ctx->last_error = buf;
    }
    return code;
}

int cuda_error(gfd_ctx* ctx, cudaError_t e, const char* what) {
    return set_error(ctx, GFD_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

// ---------------------------------------------------------------------------
// RangeSet
// ---------------------------------------------------------------------------
bool RangeSet::contains(uint64_t p, uint64_t n) const { return find(p, n) != nullptr; }

const Range* RangeSet::find(uint64_t p, uint64_t n) const {
    // last range with lo <= p
    auto it = std::upper_bound(v_.begin(), v_.end(), p,
                               [](uint64_t x, const Range& r) { return x < r.lo; });
    if (it == v_.begin()) return nullptr;
    --it;
    const bool in = p >= it->lo && n <= it->hi - it->lo && p - it->lo <= it->hi - it->lo - n;
    return in ? &*it : nullptr;
}

void RangeSet::add(const Range& r) {
    const auto overlaps = [&](const Range& x) { return x.lo < r.hi && r.lo < x.hi; };
    // a range this library pinned stays until it is freed / unregistered: a driver-learnt
    // range overlapping it is not recorded
    if (!r.owned && !r.registered)
        for (const Range& x : v_)
            if (overlaps(x) && (x.owned || x.registered)) return;
    // drop ranges that overlap the new one (stale entries of freed allocations)
    v_.erase(std::remove_if(v_.begin(), v_.end(), overlaps), v_.end());
    auto it = std::lower_bound(v_.begin(), v_.end(), r.lo,
                               [](const Range& x, uint64_t lo) { return x.lo < lo; });
    v_.insert(it, r);
}

bool RangeSet::remove(uint64_t lo, Range* out) {
    for (auto it = v_.begin(); it != v_.end(); ++it) {
        if (it->lo == lo) {
            if (out) *out = *it;
            v_.erase(it);
            return true;
        }
    }
    return false;
}

std::vector<Range> RangeSet::snapshot() const { return v_; }

// ---------------------------------------------------------------------------
// Driver entry points and context scopes
// ---------------------------------------------------------------------------
template <typename F>
static void resolve(const char* name, F* out) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q) == cudaSuccess && q == cudaDriverEntryPointSuccess)
        *out = reinterpret_cast<F>(p);
    cudaGetLastError();
}

const Driver& driver() {
    static Driver d;
    static std::once_flag once;
    std::call_once(once, [] {
        resolve("cuCtxGetCurrent", &d.ctx_get_current);
        resolve("cuCtxSetCurrent", &d.ctx_set_current);
        resolve("cuCtxPushCurrent", &d.ctx_push);
        resolve("cuCtxPopCurrent", &d.ctx_pop);
        resolve("cuDeviceGet", &d.device_get);
        resolve("cuDevicePrimaryCtxRetain", &d.primary_retain);
        resolve("cuDevicePrimaryCtxRelease", &d.primary_release);
        resolve("cuPointerGetAttributes", &d.ptr_attrs);
        resolve("cuCtxGetId", &d.ctx_get_id);  // optional (CUDA 12.0+)
        d.ok = d.ctx_get_current && d.ctx_set_current && d.ctx_push && d.ctx_pop && d.device_get &&
               d.primary_retain && d.primary_release && d.ptr_attrs;
    });
    return d;
}

CtxScope::CtxScope(CUcontext c) {
    const Driver& d = driver();
    if (!d.ok || c == nullptr) return;
    CUcontext cur = nullptr;
    d.ctx_get_current(&cur);
    if (cur != c) pushed_ = d.ctx_push(c) == CUDA_SUCCESS;
}

CtxScope::~CtxScope() {
    if (pushed_) {
        CUcontext popped = nullptr;
        driver().ctx_pop(&popped);
    }
}

struct PtrInfo {
    unsigned mem_type = 0;
    int ordinal = -1;
    uint64_t dev_ptr = 0;
    uint64_t range_lo = 0;
    size_t range_size = 0;
    unsigned managed = 0;
    bool ok = false;
};

static PtrInfo query_ptr(uint64_t p) {
    PtrInfo info;
    auto fn = driver().ptr_attrs;
    if (fn == nullptr) return info;
    CUpointer_attribute attrs[6] = {CU_POINTER_ATTRIBUTE_MEMORY_TYPE,
                                    CU_POINTER_ATTRIBUTE_DEVICE_ORDINAL,
                                    CU_POINTER_ATTRIBUTE_DEVICE_POINTER,
                                    CU_POINTER_ATTRIBUTE_RANGE_START_ADDR,
                                    CU_POINTER_ATTRIBUTE_RANGE_SIZE,
                                    CU_POINTER_ATTRIBUTE_IS_MANAGED};
    CUdeviceptr dptr = 0, rlo = 0;
    void* data[6] = {&info.mem_type, &info.ordinal, &dptr, &rlo, &info.range_size, &info.managed};
    CUresult r = fn(6, attrs, data, static_cast<CUdeviceptr>(p));
    if (r != CUDA_SUCCESS) {
        // Some attributes are not defined for every kind of memory; retry with the
        // three that always are.
        info = PtrInfo();
        CUpointer_attribute a3[3] = {CU_POINTER_ATTRIBUTE_MEMORY_TYPE,
                                     CU_POINTER_ATTRIBUTE_DEVICE_ORDINAL,
                                     CU_POINTER_ATTRIBUTE_DEVICE_POINTER};
        void* d3[3] = {&info.mem_type, &info.ordinal, &dptr};
        if (fn(3, a3, d3, static_cast<CUdeviceptr>(p)) != CUDA_SUCCESS) return info;
        rlo = 0;
        info.range_size = 0;
    }
    cudaGetLastError();
    info.dev_ptr = static_cast<uint64_t>(dptr);
    info.range_lo = static_cast<uint64_t>(rlo);
    info.ok = true;
    return info;
}

bool discover_range(gfd_ctx* ctx, uint64_t p, uint64_t n, int kind) {
    PtrInfo a = query_ptr(p);
    if (!a.ok) return false;
    if (kind == 0) {
        // pinned host memory mapped at the same address on the device (UVA)
        if (a.mem_type != CU_MEMORYTYPE_HOST || a.dev_ptr != p) return false;
        Range r{p, p + n, false, false, -1};
        if (a.range_size > 0 && a.range_lo <= p && p - a.range_lo <= a.range_size &&
            n <= a.range_size - (p - a.range_lo)) {
            r.lo = a.range_lo;
            r.hi = a.range_lo + a.range_size;
        } else if (n > 1) {
            PtrInfo b = query_ptr(p + n - 1);
            if (!b.ok || b.mem_type != CU_MEMORYTYPE_HOST || b.dev_ptr != p + n - 1) return false;
        }
        ctx->host_ranges.add(r);
        return true;
    }
    // device memory of this context's GPU (or managed memory)
    const bool dev_ok = (a.mem_type == CU_MEMORYTYPE_DEVICE && a.ordinal == ctx->device) ||
                        a.managed != 0;
    if (!dev_ok) return false;
    if (a.range_size == 0 || a.range_lo > p || p - a.range_lo > a.range_size ||
        n > a.range_size - (p - a.range_lo))
        return false;
    ctx->dev_ranges.add(Range{a.range_lo, a.range_lo + a.range_size, false, false, -1});
    return true;
}

// Ranges this library pinned itself (gfd_pool_alloc / gfd_pool_register) are trusted
// until gfd_pool_free / gfd_pool_unregister.  Ranges learnt from the driver are asked
// again on every check: the caller may have freed that memory and been handed the same
// addresses for a smaller allocation since.  Callers check once per distinct range per
// call (they remember the last range that matched), so this costs one driver lookup
// per range switch.
bool check_host(gfd_ctx* ctx, uint64_t p, uint64_t n) {
    if (p + n < p) return false;
    const Range* r = ctx->host_ranges.find(p, n);
    if (r != nullptr && (r->owned || r->registered)) return true;
    return discover_range(ctx, p, n, 0) && ctx->host_ranges.contains(p, n);
}

bool check_dev(gfd_ctx* ctx, uint64_t p, uint64_t n) {
    if (p + n < p) return false;
    return discover_range(ctx, p, n, 1) && ctx->dev_ranges.contains(p, n);
}

// [p, p + n) is pageable host memory: the driver knows no allocation at either end (not
// pinned, device or managed memory) and every page of the range is mapped in this process
// (pages_mapped).  On success *page_lo / *page_hi are the page span that was checked.
static bool pageable_host(uint64_t p, uint64_t n, uint64_t* page_lo, uint64_t* page_hi) {
    if (n == 0 || p + n < p) return false;
    const PtrInfo a = query_ptr(p);
    if (a.ok && a.mem_type != 0) return false;  // pinned (but not validated above), device or managed
    const PtrInfo b = query_ptr(p + n - 1);
    if (b.ok && b.mem_type != 0) return false;
    return pages_mapped(p, n, page_lo, page_hi);
}

// [p, p + n) inside one device allocation of a GPU this context can write to: its own,
// or a peer reachable over NVLink / PCIe peer access (an IPC mapping or peer-enabled
// memory).  Asked of the driver on every call and not cached: the range is not this
// GPU's memory, so it must never validate an ordinary call.
static bool check_peer_dev(gfd_ctx* ctx, uint64_t p, uint64_t n) {
    if (p + n < p) return false;
    const PtrInfo a = query_ptr(p);
    if (!a.ok || a.mem_type != CU_MEMORYTYPE_DEVICE) return false;
    if (a.range_size == 0 || a.range_lo > p || p - a.range_lo > a.range_size ||
        n > a.range_size - (p - a.range_lo))
        return false;
    if (a.ordinal == ctx->device) return true;
    int can = 0;
    if (cudaDeviceCanAccessPeer(&can, ctx->device, a.ordinal) != cudaSuccess || can == 0) {
        cudaGetLastError();
        return false;
    }
    // map the peer's allocations into this context (per-context state, idempotent), then
    // require that this context may write the range: a store the context cannot make
    // would fault the kernel, so anything the driver does not confirm is refused
    const cudaError_t pe = cudaDeviceEnablePeerAccess(a.ordinal, 0);
    if (pe != cudaSuccess && pe != cudaErrorPeerAccessAlreadyEnabled) {
        cudaGetLastError();
        return false;
    }
    cudaGetLastError();
    auto fn = driver().ptr_attrs;
    if (fn == nullptr) return false;
    CUpointer_attribute attr = CU_POINTER_ATTRIBUTE_ACCESS_FLAGS;
    unsigned long long access = 0;
    void* data = &access;
    if (fn(1, &attr, &data, static_cast<CUdeviceptr>(p)) != CUDA_SUCCESS) return false;
    return access == CU_POINTER_ATTRIBUTE_ACCESS_FLAG_READWRITE;
}

std::vector<Range> live_host_ranges(gfd_ctx* ctx) {
    std::vector<Range> out;
    for (const Range& r : ctx->host_ranges.snapshot()) {
        bool live = r.owned || r.registered;
        if (!live) {
            const PtrInfo a = query_ptr(r.lo);
            live = a.ok && a.mem_type == CU_MEMORYTYPE_HOST && a.dev_ptr == r.lo &&
                   ((a.range_size > 0 && a.range_lo == r.lo && a.range_size == r.hi - r.lo) ||
                    (a.range_size == 0 && r.hi - r.lo > 0 && [&] {
                        const PtrInfo b = query_ptr(r.hi - 1);
                        return b.ok && b.mem_type == CU_MEMORYTYPE_HOST && b.dev_ptr == r.hi - 1;
                    }()));
        }
        if (live) out.push_back(r);
        else ctx->host_ranges.remove(r.lo, nullptr);
    }
    return out;
}

// ---------------------------------------------------------------------------
// Host-built pull tables
// ---------------------------------------------------------------------------
static int ensure_slot(gfd_ctx* ctx, StageSlot& s, size_t rows, size_t ctas) {
    if (s.cta_first == nullptr) {
        cudaError_t e = cudaHostAlloc(reinterpret_cast<void**>(&s.cta_first), kMaxPullGrid * sizeof(uint32_t),
                                      cudaHostAllocMapped | cudaHostAllocPortable);
        if (e != cudaSuccess) {
            s.cta_first = nullptr;
            return cuda_error(ctx, e, "cudaHostAlloc(staging first-row table)");
        }
    }
    if (s.capacity < rows) {
        // the old table is released with the context, not here: freeing pinned memory
        // waits for the whole device, which may be running kernels that wait for a ring
        // drain this thread is about to issue
        if (s.rows) ctx->retired_host.push_back(s.rows);
        s.rows = nullptr;
        const size_t cap = std::max<size_t>(std::max<size_t>(rows, 2 * s.capacity), 4096);  // geometric
        cudaError_t e = cudaHostAlloc(reinterpret_cast<void**>(&s.rows), cap * sizeof(PullRow),
                                      cudaHostAllocMapped | cudaHostAllocPortable);
        if (e != cudaSuccess) {
            s.capacity = 0;
            return cuda_error(ctx, e, "cudaHostAlloc(staging rows)");
        }
        s.capacity = cap;
    }
    (void)ctas;
    return GFD_OK;
}

struct HostTable {
    uint32_t n_rows = 0;
    uint32_t n_misc = 0;
    uint64_t total = 0;
    uint64_t bytes = 0;
    uint64_t n_ce = 0;
};

// Walks the caller's entries once: validation, run merging, stream offsets.  Stream
// rows are written straight into `rows` (pinned staging), misc rows to ctx->host_misc,
// copy-engine runs to ctx->ce_runs.
// d2h: sources are device memory and destinations pinned host memory (scatter).
static int build_rows(gfd_ctx* ctx, const gfd_sg_entry* e, int64_t n, bool validate, bool d2h,
                      uint32_t flags, PullRow* rows, HostTable* t) {
    ctx->host_misc.clear();
    ctx->ce_runs.clear();
    ctx->pageable_runs.clear();
    const bool force_ce = (flags & GFD_GATHER_FORCE_CE) != 0;
    const bool auto_ce = (flags & GFD_GATHER_AUTO_CE) != 0;
    const bool pageable_ok = !d2h && (flags & GFD_GATHER_PAGEABLE) != 0;
    uint64_t bytes = 0;
    TableBuilder tb(rows, &ctx->host_misc);
    uint64_t slo = 1, shi = 1, dlo = 1, dhi = 1;  // last matched ranges (empty)
    uint64_t plo = 1, phi = 1;                     // last page span checked as pageable
    for (int64_t i = 0; i < n; ++i) {
        const uint64_t src = reinterpret_cast<uint64_t>(e[i].src);
        const uint64_t dst = e[i].dst;
        const uint64_t size = e[i].size;
        if (size == 0) continue;
        bool pageable = false;
        // most entries of a call share one pool and one destination buffer: test the
        // ranges of the previous entry before searching the registry
        if (validate && !(src >= slo && size <= shi - slo && src - slo <= shi - slo - size)) {
            if (pageable_ok && src >= plo && size <= phi - plo && src - plo <= phi - plo - size) {
                pageable = true;
            } else {
                bool ok = d2h ? check_dev(ctx, src, size) : check_host(ctx, src, size);
                if (!ok && pageable_ok) ok = pageable = pageable_host(src, size, &plo, &phi);
                if (!ok)
                    return set_error(ctx, GFD_ERR_INVALID, "entry %lld: src [0x%llx, +%llu) is not %s", (long long)i,
                                     (unsigned long long)src, (unsigned long long)size,
                                     d2h ? "inside one device allocation of this GPU"
                                     : pageable_ok ? "in pinned, device-mapped host memory or mapped pageable memory"
                                                   : "in pinned, device-mapped host memory");
                if (!pageable) {
                    const Range* r = d2h ? ctx->dev_ranges.find(src, size) : ctx->host_ranges.find(src, size);
                    slo = r->lo;
                    shi = r->hi;
                }
            }
        }
        if (validate && !(dst >= dlo && size <= dhi - dlo && dst - dlo <= dhi - dlo - size)) {
            const bool ok = d2h ? check_host(ctx, dst, size) : check_dev(ctx, dst, size);
            if (!ok)
                return set_error(ctx, GFD_ERR_INVALID, "entry %lld: dst [0x%llx, +%llu) is not %s", (long long)i,
                                 (unsigned long long)dst, (unsigned long long)size,
                                 d2h ? "in pinned, device-mapped host memory"
                                     : "inside one device allocation of this GPU");
            const Range* r = d2h ? ctx->host_ranges.find(dst, size) : ctx->dev_ranges.find(dst, size);
            dlo = r->lo;
            dhi = r->hi;
        }
        bytes += size;
        if (force_ce || pageable) {
            std::vector<gfd_sg_entry>& runs = pageable ? ctx->pageable_runs : ctx->ce_runs;
            if (!runs.empty()) {
                gfd_sg_entry& last = runs.back();
                if (reinterpret_cast<uint64_t>(last.src) + last.size == src &&
                    last.dst + last.size == dst) {
                    last.size += size;
                    continue;
                }
            }
            runs.push_back(gfd_sg_entry{dst, reinterpret_cast<const void*>(src), size});
            continue;
        }
        tb.add(src, dst, size);
    }
    // evenly strided layouts: a few 2D copy-engine copies beat the SM pull for large rows
    // (2048 x 16..64 KiB at 2x stride: 51.2-54.4 GB/s against 49.3-50.8) and for small
    // calls, where one copy call costs less than a kernel launch and its completion word
    // (16 / 64 x 4 KiB: 5.0 / 14.8 GB/s against 3.9 / 12.0)
    if (!force_ce && !auto_ce && !d2h && (flags & (GFD_GATHER_FORCE_PULL | GFD_GATHER_BULK_STAGE)) == 0 &&
        ctx->host_misc.empty() &&
        tb.n_rows() >= 2) {
        std::vector<CeCopy>& g = ctx->ce_copies;
        g.clear();
        group_strided(rows, tb.n_rows(), &g);
        const bool small = tb.total() <= kStridedCeSmallCall;
        bool strided = g.size() <= kStridedCeGroups;
        for (const CeCopy& c : g) strided = strided && c.height >= 2 && (small || c.width >= kStridedCeMinRow);
        // Splitting the other evenly strided calls (shorter rows) between the copy engines
        // and the pull, both at once, measured slower at every share tried (10-50%)
        if (strided)
            tb.remove_rows([&](const PullRow& row) {
                ctx->ce_runs.push_back(gfd_sg_entry{row.dst, reinterpret_cast<const void*>(row.src), row.len});
                return true;
            });
    }
    if (auto_ce && !force_ce && ctx->ce_threshold != ~0ull) {
        // move long rows to the copy engine and re-pack the stream
        tb.remove_rows([&](const PullRow& row) {
            if (row.len < ctx->ce_threshold) return false;
            ctx->ce_runs.push_back(gfd_sg_entry{row.dst, reinterpret_cast<const void*>(row.src), row.len});
            return true;
        });
    }
    const uint32_t nr = tb.n_rows();
    const uint64_t total = tb.total();
    t->n_rows = nr;
    t->n_misc = static_cast<uint32_t>(ctx->host_misc.size());
    t->total = total;
    t->bytes = bytes;
    t->n_ce = ctx->ce_runs.size() + ctx->pageable_runs.size();
    return GFD_OK;
}

bool wait_flag(volatile uint64_t* flag, uint64_t value, uint64_t timeout_ns, cudaStream_t st,
               cudaError_t* err) {
    *err = cudaSuccess;
    const uint64_t t0 = now_ns();
    uint32_t spins = 0;
    for (;;) {
        if (__atomic_load_n(flag, __ATOMIC_ACQUIRE) >= value) return true;
        if ((++spins & 0xfff) == 0) {
            cudaError_t q = cudaStreamQuery(st);
            if (q != cudaSuccess && q != cudaErrorNotReady) {
                *err = q;
                return false;
            }
            if (q == cudaSuccess) {
                // Stream idle: the word must be visible now (allow in-flight posted
                // writes a moment); otherwise the kernel did not run to completion.
                const uint64_t t1 = now_ns();
                while (now_ns() - t1 < 1000000ull)
                    if (__atomic_load_n(flag, __ATOMIC_ACQUIRE) >= value) return true;
                *err = cudaErrorLaunchFailure;
                return false;
            }
            if (now_ns() - t0 > timeout_ns) return false;
        }
        cpu_relax();
    }
}

}  // namespace gfdb

using namespace gfdb;

namespace {

int ensure_device_scratch(gfd_ctx* ctx, size_t rows) {
    if (ctx->d_capacity >= rows && ctx->d_rows != nullptr) return GFD_OK;
    // outgrown buffers are released with the context: cudaFree waits for the whole
    // device, which may be running kernels that wait for this library's ring drains
    // (earlier launches may also still be reading them)
    for (void* p : {static_cast<void*>(ctx->d_rows), static_cast<void*>(ctx->d_misc), static_cast<void*>(ctx->d_tiles)})
        if (p) ctx->retired_dev.push_back(p);
    ctx->d_rows = nullptr;
    ctx->d_misc = nullptr;
    ctx->d_tiles = nullptr;
    const size_t cap = std::max<size_t>(std::max<size_t>(rows, 2 * ctx->d_capacity), 4096);  // geometric
    cudaError_t e = cudaMalloc(&ctx->d_rows, cap * sizeof(PullRow));
    if (e == cudaSuccess) e = cudaMalloc(&ctx->d_misc, cap * sizeof(PullRow));
    if (e == cudaSuccess) e = cudaMalloc(&ctx->d_tiles, plan_tile_slots(cap) * sizeof(TileTotals));
    if (e != cudaSuccess) {
        ctx->d_capacity = 0;
        return set_error(ctx, GFD_ERR_NOMEM, "cudaMalloc(device row table, %zu rows): %s", cap,
                         cudaGetErrorString(e));
    }
    ctx->d_capacity = cap;
    return GFD_OK;
}

// Issues copy-engine copies for ctx->ce_runs and ctx->pageable_runs, ordered after the
// work recorded in ctx->join_event (the caller's stream before this call's pull launch)
// and joined back into the caller's stream by join_ce.  Evenly strided pinned runs become one 2D copy
// each (group_strided); a pageable run is always a 1D copy of its own bytes (a 2D copy
// would span the gaps between rows, which need not be mapped).  The copies are spread
// over the three copy-engine streams, a large 2D copy split by rows when there are fewer
// copies than streams.
int issue_ce(gfd_ctx* ctx, bool d2h) {
    const size_t nr = ctx->ce_runs.size() + ctx->pageable_runs.size();
    if (nr == 0) return GFD_OK;
    std::vector<PullRow>& runs = ctx->ce_rows;
    runs.clear();
    for (const gfd_sg_entry& r : ctx->ce_runs)
        runs.push_back(PullRow{reinterpret_cast<uint64_t>(r.src), r.dst, r.size, 0});
    std::vector<CeCopy>& cp = ctx->ce_copies;
    cp.clear();
    group_strided(runs.data(), runs.size(), &cp);
    for (const gfd_sg_entry& r : ctx->pageable_runs)
        cp.push_back(CeCopy{r.dst, reinterpret_cast<uint64_t>(r.src), r.size, 1, r.size, r.size});
    if (cp.size() < 3) {
        std::vector<CeCopy> split;
        for (const CeCopy& c : cp) {
            const uint64_t parts = c.height >= 3 && c.width * c.height >= (1ull << 20) ? 3 : 1;
            uint64_t row = 0;
            for (uint64_t k = 0; k < parts; ++k) {
                const uint64_t h = c.height / parts + (k < c.height % parts ? 1 : 0);
                split.push_back(CeCopy{c.dst + row * c.dpitch, c.src + row * c.spitch, c.width, h, c.dpitch, c.spitch});
                row += h;
            }
        }
        cp.swap(split);
    }
    const size_t n = cp.size();
    const cudaMemcpyKind kind = d2h ? cudaMemcpyDeviceToHost : cudaMemcpyHostToDevice;
    cudaError_t e = cudaSuccess;
    const int nch = n < 3 ? static_cast<int>(n) : 3;
    const size_t per = (n + nch - 1) / nch;
    int rc = GFD_OK;
    for (int c = 0; c < nch && rc == GFD_OK; ++c) {
        cudaStream_t cs = ctx->ce_streams[c];
        e = cudaStreamWaitEvent(cs, ctx->join_event, 0);
        if (e != cudaSuccess) return cuda_error(ctx, e, "cudaStreamWaitEvent");
        const size_t b = c * per, end = std::min(n, b + per);
        for (size_t i = b; i < end; ++i) {
            const CeCopy& x = cp[i];
            if (x.height == 1)
                e = cudaMemcpyAsync(reinterpret_cast<void*>(x.dst), reinterpret_cast<const void*>(x.src), x.width, kind, cs);
            else
                e = cudaMemcpy2DAsync(reinterpret_cast<void*>(x.dst), x.dpitch, reinterpret_cast<const void*>(x.src),
                                      x.spitch, x.width, x.height, kind, cs);
            if (e != cudaSuccess) {
                rc = cuda_error(ctx, e, "copy-engine copy");
                break;
            }
            ctx->st_ce++;
        }
        // the stream's event is recorded even after a failed copy, so join_ce still orders
        // later work after the copies that were issued
        e = cudaEventRecord(ctx->ce_events[c], cs);
        if (e != cudaSuccess) return cuda_error(ctx, e, "CE join");
        ctx->ce_pending = c + 1;
    }
    return rc;
}

// Orders later work on `st` after the copies of the last issue_ce (called after the pull
// kernel of the same call is launched, so the two run at the same time).
int join_ce(gfd_ctx* ctx, cudaStream_t st) {
    for (int c = 0; c < ctx->ce_pending; ++c) {
        const cudaError_t e = cudaStreamWaitEvent(st, ctx->ce_events[c], 0);
        if (e != cudaSuccess) {
            ctx->ce_pending = 0;
            return cuda_error(ctx, e, "CE join");
        }
    }
    ctx->ce_pending = 0;
    return GFD_OK;
}

// Shared body of gfd_gather / gfd_gather_sync.  On return *flag/*value identify the
// completion word of the pull launch (flag null when no pull kernel was needed).
// drain (ring drains): completion work for the last CTA of the launch, which then runs
// even when there is nothing to move; bytes_ctr: device counter of the bytes moved.
int gather_locked(gfd_ctx* ctx, const gfd_sg_entry* entries, int64_t n, cudaStream_t st,
                  uint32_t flags, bool d2h, volatile uint64_t** flag_out, uint64_t* value_out,
                  const RingDrain* drain = nullptr, const RingTables* tables = nullptr,
                  unsigned long long* bytes_ctr = nullptr) {
    *flag_out = nullptr;
    *value_out = 0;
    if (n < 0 || (n > 0 && entries == nullptr))
        return set_error(ctx, GFD_ERR_INVALID, "gather: bad entry array (n=%lld)", (long long)n);
    if (n > 0x7fffffffll)
        return set_error(ctx, GFD_ERR_INVALID, "gather: at most 2^31-1 entries per call");
    if ((flags & GFD_GATHER_PAGEABLE) != 0 && (flags & GFD_GATHER_TRUSTED) != 0 && !d2h)
        return set_error(ctx, GFD_ERR_INVALID,
                         "gather: GFD_GATHER_PAGEABLE needs the source check that GFD_GATHER_TRUSTED skips");
    if (n == 0 && drain == nullptr) return GFD_OK;

    const int slot_idx = ctx->next_slot;
    ctx->next_slot = (ctx->next_slot + 1) % gfd_ctx::kSlots;
    StageSlot& slot = ctx->slots[slot_idx];
    if (slot.issued != 0) {
        cudaError_t e;
        if (!wait_flag(slot.flag, slot.issued, ctx->timeout_ns, slot.stream, &e))
            return e != cudaSuccess ? cuda_error(ctx, e, "waiting for staging slot")
                                    : set_error(ctx, GFD_ERR_TIMEOUT,
                                                "staging slot still in use after timeout");
    }
    int rc = ensure_slot(ctx, slot, static_cast<size_t>(n), 0);
    if (rc != GFD_OK) return rc;

    HostTable t;
    const uint64_t t_prep = now_ns();
    rc = build_rows(ctx, entries, n, (flags & GFD_GATHER_TRUSTED) == 0, d2h, flags, slot.rows, &t);
    const uint64_t t_launch = now_ns();
    ctx->st_prep_ns += t_launch - t_prep;
    if (rc != GFD_OK) {
        ctx->st_rejected++;
        return rc;
    }

    // Copy-engine copies of this call wait only for the work before it on st: the pull is
    // launched first, then the copies are issued, and st joins them last, so the two run
    // at the same time (the copies' host-side issue does not delay the pull's launch).
    const bool have_ce = !ctx->ce_runs.empty() || !ctx->pageable_runs.empty();
    if (have_ce) {
        const cudaError_t e = cudaEventRecord(ctx->join_event, st);
        if (e != cudaSuccess) return cuda_error(ctx, e, "cudaEventRecord");
    }
    if (t.n_rows > 0 || t.n_misc > 0 || drain != nullptr) {
        PullArgs a;
        std::memset(&a, 0, sizeof(a));
        if (drain != nullptr) {
            a.drain = *drain;
            a.drain.tables = nullptr;
            if (drain->n_tiles > 0 || drain->n_lists > 0) {
                if (slot.tables == nullptr) {
                    cudaError_t e = cudaHostAlloc(reinterpret_cast<void**>(&slot.tables), sizeof(RingTables),
                                                  cudaHostAllocMapped | cudaHostAllocPortable);
                    if (e != cudaSuccess) {
                        slot.tables = nullptr;
                        return cuda_error(ctx, e, "cudaHostAlloc(drain tables)");
                    }
                }
                std::memcpy(slot.tables->tile_id, tables->tile_id, drain->n_tiles * sizeof(uint16_t));
                std::memcpy(slot.tables->tile_count, tables->tile_count, drain->n_tiles * sizeof(uint32_t));
                std::memcpy(slot.tables->list_id, tables->list_id, drain->n_lists * sizeof(uint16_t));
                a.drain.tables = slot.tables;
            }
        }
        a.bytes_ctr = bytes_ctr;
        if (t.n_rows + t.n_misc <= static_cast<uint32_t>(kInlineRows)) {
            // small request: the whole table travels in the kernel parameters
            std::memcpy(a.rows_inline, slot.rows, t.n_rows * sizeof(PullRow));
            if (t.n_misc > 0)
                std::memcpy(a.rows_inline + t.n_rows, ctx->host_misc.data(), t.n_misc * sizeof(PullRow));
            a.rows = nullptr;
            a.misc = nullptr;
        } else {
            // misc rows follow the stream rows in the staging slot
            if (t.n_misc > 0)
                std::memcpy(slot.rows + t.n_rows, ctx->host_misc.data(), t.n_misc * sizeof(PullRow));
            a.rows = slot.rows;
            a.misc = slot.rows + t.n_rows;
        }
        a.geo.total = t.total;
        a.geo.n_rows = t.n_rows;
        a.geo.n_misc = t.n_misc;
        int grid = pull_grid_for(t.total, ctx->num_sms);
        uint64_t per = (t.total + grid - 1) / grid;
        per = (per + kPiece - 1) / kPiece * kPiece;
        if (per == 0) per = kPiece;
        a.geo.per_cta = per;
        int active = static_cast<int>((t.total + per - 1) / per);
        int misc_grid = static_cast<int>(std::min<uint64_t>((t.n_misc + kPullWarps - 1) / kPullWarps,
                                                            static_cast<uint64_t>(2 * ctx->num_sms)));
        grid = std::max(1, std::max(active, misc_grid));
        if (grid > kMaxPullGrid) grid = kMaxPullGrid;
        uint32_t* first = grid <= kInlineFirst ? a.cta_first_inline : slot.cta_first;
        partition_ctas(slot.rows, t.n_rows, per, grid, first);
        a.cta_first = grid <= kInlineFirst ? nullptr : slot.cta_first;
        a.done_ctr = ctx->d_done_ctr + slot_idx;
        a.done_flag = slot.flag;
        a.done_value = ++ctx->seq;
        a.sys_fence = d2h ? 1u : 0u;
        cudaError_t e = launch_pull(a, grid, st, (flags & GFD_GATHER_BULK_STAGE) != 0 && !d2h);
        if (e != cudaSuccess) return cuda_error(ctx, e, "pull kernel launch");
        slot.issued = a.done_value;
        slot.stream = st;
        *flag_out = slot.flag;
        *value_out = a.done_value;
        ctx->st_pulls++;
    }
    if (have_ce) {
        rc = issue_ce(ctx, d2h);
        const int jrc = join_ce(ctx, st);
        if (rc != GFD_OK) return rc;
        if (jrc != GFD_OK) return jrc;
    }
    ctx->st_launch_ns += now_ns() - t_launch;
    ctx->st_calls++;
    ctx->st_entries += static_cast<uint64_t>(n);
    ctx->st_bytes += t.bytes;
    return GFD_OK;
}

}  // namespace

namespace gfdb {

int reserve_drain_slots(gfd_ctx* ctx, size_t rows) {
    for (StageSlot& slot : ctx->slots) {
        int rc = ensure_slot(ctx, slot, rows, 0);
        if (rc != GFD_OK) return rc;
        if (slot.tables == nullptr) {
            cudaError_t e = cudaHostAlloc(reinterpret_cast<void**>(&slot.tables), sizeof(RingTables),
                                          cudaHostAllocMapped | cudaHostAllocPortable);
            if (e != cudaSuccess) {
                slot.tables = nullptr;
                return cuda_error(ctx, e, "cudaHostAlloc(drain tables)");
            }
        }
    }
    return GFD_OK;
}

int gather_drain(gfd_ctx* ctx, const gfd_sg_entry* entries, int64_t n, cudaStream_t st, const RingDrain& drain,
                 const RingTables& tables, unsigned long long* bytes_ctr) {
    volatile uint64_t* flag;
    uint64_t value;
    // always the SM pull: the drain's completion runs in the pull kernel's last CTA, and
    // copy-engine copies would add a launch and a join per drain
    return gather_locked(ctx, entries, n, st, GFD_GATHER_TRUSTED | GFD_GATHER_FORCE_PULL, false, &flag, &value,
                         &drain, &tables, bytes_ctr);
}

}  // namespace gfdb

namespace {

int async_call(gfd_ctx* ctx, const gfd_sg_entry* entries, int64_t n, void* stream, uint32_t flags, bool d2h) {
    if (!ctx) return GFD_ERR_INVALID;
    std::lock_guard<std::mutex> lk(ctx->mu);
    CtxScope scope(ctx->cu_ctx);
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
    volatile uint64_t* flag;
    uint64_t value;
    return gather_locked(ctx, entries, n, st, flags, d2h, &flag, &value);
}

int sync_call(gfd_ctx* ctx, const gfd_sg_entry* entries, int64_t n, uint32_t flags, double* elapsed_us,
              bool d2h) {
    if (!ctx) return GFD_ERR_INVALID;
    const uint64_t t0 = now_ns();
    std::lock_guard<std::mutex> lk(ctx->mu);
    CtxScope scope(ctx->cu_ctx);
    volatile uint64_t* flag;
    uint64_t value;
    int rc = gather_locked(ctx, entries, n, ctx->stream, flags, d2h, &flag, &value);
    if (rc != GFD_OK) return rc;
    const uint64_t t_wait = now_ns();
    struct WaitTimer {
        gfd_ctx* c;
        uint64_t t;
        ~WaitTimer() { c->st_wait_ns += now_ns() - t; }
    } wt{ctx, t_wait};
    if (!ctx->ce_runs.empty() || !ctx->pageable_runs.empty() || flag == nullptr) {
        cudaError_t e = cudaStreamSynchronize(ctx->stream);
        if (e != cudaSuccess) return cuda_error(ctx, e, "cudaStreamSynchronize");
    } else {
        // the completion word is raised after every CTA's stores are visible (system
        // scope for a scatter into host memory)
        cudaError_t e;
        if (!wait_flag(flag, value, ctx->timeout_ns, ctx->stream, &e))
            return e != cudaSuccess ? cuda_error(ctx, e, d2h ? "scatter" : "gather")
                                    : set_error(ctx, GFD_ERR_TIMEOUT, "%s did not complete in time",
                                                d2h ? "scatter" : "gather");
    }
    if (elapsed_us) *elapsed_us = (now_ns() - t0) / 1000.0;
    return GFD_OK;
}

}  // namespace

// ===========================================================================
// C ABI
// ===========================================================================
extern "C" {

int gfd_ctx_create(int device, gfd_ctx** out) {
    if (out == nullptr) return GFD_ERR_INVALID;
    *out = nullptr;
    int count = 0;
    cudaError_t e = cudaGetDeviceCount(&count);
    if (e != cudaSuccess || device < 0 || device >= count) {
        cudaGetLastError();
        return GFD_ERR_CUDA;
    }
    gfd_ctx* ctx = new (std::nothrow) gfd_ctx();
    if (ctx == nullptr) return GFD_ERR_NOMEM;
    ctx->device = device;
    // Run in the context current on this thread if it belongs to `device` (a driver
    // API context such as one from cuCtxCreate, as the reference's programs use),
    // otherwise in the device's primary context.
    const Driver& drv = driver();
    if (!drv.ok) {
        delete ctx;
        return GFD_ERR_CUDA;
    }
    CUcontext cur = nullptr;
    drv.ctx_get_current(&cur);
    int cur_dev = -1;
    if (cur != nullptr && cudaGetDevice(&cur_dev) == cudaSuccess && cur_dev == device) {
        ctx->cu_ctx = cur;
    } else {
        CUdevice dev = 0;
        if (drv.device_get(&dev, device) != CUDA_SUCCESS || drv.primary_retain(&ctx->cu_ctx, dev) != CUDA_SUCCESS) {
            cudaGetLastError();
            delete ctx;
            return GFD_ERR_CUDA;
        }
        ctx->primary_retained = true;
    }
    cudaGetLastError();
    {
    CtxScope scope(ctx->cu_ctx);
    cudaDeviceGetAttribute(&ctx->num_sms, cudaDevAttrMultiProcessorCount, device);
    int lo = 0, hi = 0;
    cudaDeviceGetStreamPriorityRange(&lo, &hi);
    e = cudaStreamCreateWithPriority(&ctx->stream, cudaStreamNonBlocking, hi);
    for (int i = 0; e == cudaSuccess && i < 3; ++i) {
        e = cudaStreamCreateWithPriority(&ctx->ce_streams[i], cudaStreamNonBlocking, hi);
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ctx->ce_events[i], cudaEventDisableTiming);
    }
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ctx->join_event, cudaEventDisableTiming);
    if (e == cudaSuccess)
        e = cudaHostAlloc(reinterpret_cast<void**>(&ctx->flags_host), 64 * gfd_ctx::kSlots,
                          cudaHostAllocMapped | cudaHostAllocPortable);
    if (e == cudaSuccess) e = cudaMalloc(&ctx->d_done_ctr, 64 * sizeof(uint32_t));
    if (e == cudaSuccess) e = cudaMemsetAsync(ctx->d_done_ctr, 0, 64 * sizeof(uint32_t), ctx->stream);
    if (e == cudaSuccess) e = cudaMalloc(&ctx->d_hdr, sizeof(PlanHeader));
    if (e == cudaSuccess) e = cudaMemsetAsync(ctx->d_hdr, 0, sizeof(PlanHeader), ctx->stream);  // list fields at rest
    if (e == cudaSuccess) e = cudaMalloc(&ctx->d_cta_first, kMaxPullGrid * sizeof(uint32_t));
    if (e == cudaSuccess) e = preload_gather_kernels();
    if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
    cudaGetLastError();
    }  // scope: the context is popped before a failed create is torn down
    if (e != cudaSuccess) {
        gfd_ctx_destroy(ctx);
        return GFD_ERR_CUDA;
    }
    std::memset(ctx->flags_host, 0, 64 * gfd_ctx::kSlots);
    for (int i = 0; i < gfd_ctx::kSlots; ++i)
        ctx->slots[i].flag = reinterpret_cast<volatile uint64_t*>(
            reinterpret_cast<char*>(ctx->flags_host) + 64 * i);
    *out = ctx;
    return GFD_OK;
}

int gfd_ctx_destroy(gfd_ctx* ctx) {
    if (ctx == nullptr) return GFD_OK;
    {
    CtxScope scope(ctx->cu_ctx);
    if (ctx->stream) cudaStreamSynchronize(ctx->stream);
    for (int i = 0; i < 3; ++i) {
        if (ctx->ce_streams[i]) {
            cudaStreamSynchronize(ctx->ce_streams[i]);
            cudaStreamDestroy(ctx->ce_streams[i]);
        }
        if (ctx->ce_events[i]) cudaEventDestroy(ctx->ce_events[i]);
    }
    if (ctx->join_event) cudaEventDestroy(ctx->join_event);
    if (ctx->stream) cudaStreamDestroy(ctx->stream);
    for (auto& s : ctx->slots) {
        if (s.rows) cudaFreeHost(s.rows);
        if (s.cta_first) cudaFreeHost(s.cta_first);
        if (s.tables) cudaFreeHost(s.tables);
    }
    for (void* p : ctx->retired_host) cudaFreeHost(p);
    for (void* p : ctx->retired_dev) cudaFree(p);
    if (ctx->flags_host) cudaFreeHost(ctx->flags_host);
    if (ctx->d_done_ctr) cudaFree(ctx->d_done_ctr);
    if (ctx->d_rows) cudaFree(ctx->d_rows);
    if (ctx->d_misc) cudaFree(ctx->d_misc);
    if (ctx->d_cta_first) cudaFree(ctx->d_cta_first);
    if (ctx->d_hdr) cudaFree(ctx->d_hdr);
    if (ctx->d_tiles) cudaFree(ctx->d_tiles);
    if (ctx->d_sel) cudaFree(ctx->d_sel);
    for (const Range& r : ctx->host_ranges.snapshot()) {
        if (r.registered) cudaHostUnregister(reinterpret_cast<void*>(r.lo));
        if (r.owned) munmap(reinterpret_cast<void*>(r.lo), r.hi - r.lo);
    }
    cudaGetLastError();
    }
    if (ctx->primary_retained) {
        CUdevice dev = 0;
        if (driver().device_get(&dev, ctx->device) == CUDA_SUCCESS) driver().primary_release(dev);
    }
    delete ctx;
    return GFD_OK;
}

int gfd_ctx_device(const gfd_ctx* ctx) { return ctx ? ctx->device : -1; }

const char* gfd_last_error(const gfd_ctx* ctx) {
    return ctx ? ctx->last_error.c_str() : "null context";
}

int gfd_set_timeout_ns(gfd_ctx* ctx, uint64_t ns) {
    if (!ctx || ns == 0) return GFD_ERR_INVALID;
    ctx->timeout_ns = ns;
    return GFD_OK;
}

int gfd_set_ce_threshold(gfd_ctx* ctx, uint64_t bytes) {
    if (!ctx) return GFD_ERR_INVALID;
    ctx->ce_threshold = bytes == 0 ? ~0ull : bytes;
    return GFD_OK;
}

int gfd_get_stats(const gfd_ctx* ctx, gfd_stats* out) {
    if (!ctx || !out) return GFD_ERR_INVALID;
    out->calls = ctx->st_calls.load();
    out->entries = ctx->st_entries.load();
    out->bytes = ctx->st_bytes.load();
    out->pull_launches = ctx->st_pulls.load();
    out->ce_copies = ctx->st_ce.load();
    out->rejected = ctx->st_rejected.load();
    out->prep_ns = ctx->st_prep_ns.load();
    out->launch_ns = ctx->st_launch_ns.load();
    out->wait_ns = ctx->st_wait_ns.load();
    return GFD_OK;
}

static int gpu_numa_node(int device) {
    char bus[32] = {0};
    if (cudaDeviceGetPCIBusId(bus, sizeof(bus), device) != cudaSuccess) return -1;
    for (char* p = bus; *p; ++p)
        if (*p >= 'A' && *p <= 'F') *p = static_cast<char>(*p - 'A' + 'a');
    char path[128];
    snprintf(path, sizeof(path), "/sys/bus/pci/devices/%s/numa_node", bus);
    FILE* f = fopen(path, "r");
    if (!f) return -1;
    int node = -1;
    if (fscanf(f, "%d", &node) != 1) node = -1;
    fclose(f);
    return node;
}

int gfd_pool_alloc(gfd_ctx* ctx, size_t bytes, int numa_node, void** out_host) {
    if (!ctx || !out_host || bytes == 0) return GFD_ERR_INVALID;
    std::lock_guard<std::mutex> lk(ctx->mu);
    CtxScope scope(ctx->cu_ctx);
    *out_host = nullptr;
    // An explicit node must be honoured; the GPU's own node (numa_node < 0) is a
    // preference: a host that reports none, or cannot bind to it, gets an unbound pool.
    MappedPool m;
    if (numa_node >= 0) {
        if (map_numa_pool(bytes, numa_node, &m) != 0)
            return set_error(ctx, m.err == ENOMEM ? GFD_ERR_NOMEM : GFD_ERR_INVALID,
                             "gfd_pool_alloc: %zu bytes on NUMA node %d: %s", bytes, numa_node, strerror(m.err));
    } else {
        const int gpu_node = gpu_numa_node(ctx->device);
        if (map_numa_pool(bytes, gpu_node, &m) != 0 && (gpu_node < 0 || map_numa_pool(bytes, -1, &m) != 0))
            return set_error(ctx, GFD_ERR_NOMEM, "gfd_pool_alloc: mmap(%zu): %s", bytes, strerror(m.err));
    }
    void* p = m.ptr;
    const size_t len = m.len;
    cudaError_t e = cudaHostRegister(p, len, cudaHostRegisterMapped | cudaHostRegisterPortable);
    if (e != cudaSuccess) {
        unmap_numa_pool(p, len);
        cudaGetLastError();
        return cuda_error(ctx, e, "cudaHostRegister(pool)");
    }
    void* dp = nullptr;
    if (cudaHostGetDevicePointer(&dp, p, 0) != cudaSuccess || dp != p) {
        cudaHostUnregister(p);
        unmap_numa_pool(p, len);
        cudaGetLastError();
        return set_error(ctx, GFD_ERR_UNSUPPORTED, "pool is not mapped at its host address (no UVA)");
    }
    ctx->host_ranges.add(Range{reinterpret_cast<uint64_t>(p), reinterpret_cast<uint64_t>(p) + len,
                               true, true, m.node});
    *out_host = p;
    return GFD_OK;
}

int gfd_pool_numa_node(gfd_ctx* ctx, const void* host, int* node) {
    if (!ctx || !host || !node) return GFD_ERR_INVALID;
    std::lock_guard<std::mutex> lk(ctx->mu);
    const Range* r = ctx->host_ranges.find(reinterpret_cast<uint64_t>(host), 1);
    if (r == nullptr || !r->owned)
        return set_error(ctx, GFD_ERR_INVALID, "gfd_pool_numa_node: not inside a pool from gfd_pool_alloc");
    *node = r->numa;
    return GFD_OK;
}

int gfd_pool_free(gfd_ctx* ctx, void* host) {
    if (!ctx || !host) return GFD_ERR_INVALID;
    std::lock_guard<std::mutex> lk(ctx->mu);
    CtxScope scope(ctx->cu_ctx);
    Range r;
    if (!ctx->host_ranges.remove(reinterpret_cast<uint64_t>(host), &r) || !r.owned)
        return set_error(ctx, GFD_ERR_INVALID, "gfd_pool_free: not a pool from gfd_pool_alloc");
    cudaStreamSynchronize(ctx->stream);
    cudaHostUnregister(host);
    munmap(host, r.hi - r.lo);
    cudaGetLastError();
    return GFD_OK;
}

int gfd_pool_register(gfd_ctx* ctx, void* host, size_t bytes) {
    if (!ctx || !host || bytes == 0) return GFD_ERR_INVALID;
    std::lock_guard<std::mutex> lk(ctx->mu);
    CtxScope scope(ctx->cu_ctx);
    cudaError_t e =
        cudaHostRegister(host, bytes, cudaHostRegisterMapped | cudaHostRegisterPortable);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return cuda_error(ctx, e, "cudaHostRegister");
    }
    void* dp = nullptr;
    if (cudaHostGetDevicePointer(&dp, host, 0) != cudaSuccess || dp != host) {
        cudaHostUnregister(host);
        cudaGetLastError();
        return set_error(ctx, GFD_ERR_UNSUPPORTED, "registered memory is not mapped at its host address");
    }
    const uint64_t lo = reinterpret_cast<uint64_t>(host);
    ctx->host_ranges.add(Range{lo, lo + bytes, false, true, -1});
    return GFD_OK;
}

int gfd_pool_unregister(gfd_ctx* ctx, void* host) {
    if (!ctx || !host) return GFD_ERR_INVALID;
    std::lock_guard<std::mutex> lk(ctx->mu);
    CtxScope scope(ctx->cu_ctx);
    Range r;
    if (!ctx->host_ranges.remove(reinterpret_cast<uint64_t>(host), &r) || !r.registered || r.owned)
        return set_error(ctx, GFD_ERR_INVALID, "gfd_pool_unregister: not a registered pool");
    cudaStreamSynchronize(ctx->stream);
    cudaHostUnregister(host);
    cudaGetLastError();
    return GFD_OK;
}

int gfd_gather(gfd_ctx* ctx, const gfd_sg_entry* entries, int64_t n, void* stream, uint32_t flags) {
    return async_call(ctx, entries, n, stream, flags, false);
}

int gfd_gather_sync(gfd_ctx* ctx, const gfd_sg_entry* entries, int64_t n, uint32_t flags,
                    double* elapsed_us) {
    return sync_call(ctx, entries, n, flags, elapsed_us, false);
}

int gfd_scatter(gfd_ctx* ctx, const gfd_sg_entry* entries, int64_t n, void* stream, uint32_t flags) {
    return async_call(ctx, entries, n, stream, flags, true);
}

int gfd_scatter_sync(gfd_ctx* ctx, const gfd_sg_entry* entries, int64_t n, uint32_t flags,
                     double* elapsed_us) {
    return sync_call(ctx, entries, n, flags, elapsed_us, true);
}

int gfd_gather_device(gfd_ctx* ctx, const gfd_sg_entry* d_entries, int64_t n, void* dst_base,
                      size_t dst_bytes, void* stream, uint32_t flags) {
    if (!ctx) return GFD_ERR_INVALID;
    if ((flags & ~static_cast<uint32_t>(GFD_GATHER_PEER_DST)) != 0)
        return set_error(ctx, GFD_ERR_INVALID, "gather_device: unknown flags 0x%x", flags);
    std::lock_guard<std::mutex> lk(ctx->mu);
    CtxScope scope(ctx->cu_ctx);
    if (n < 0 || (n > 0 && d_entries == nullptr) || n > 0x7fffffffll)
        return set_error(ctx, GFD_ERR_INVALID, "gather_device: bad entry array");
    if (reinterpret_cast<uint64_t>(d_entries) & 7u)
        return set_error(ctx, GFD_ERR_INVALID, "gather_device: entry array is not 8-byte aligned");
    if (n == 0) return GFD_OK;
    const uint64_t dlo = reinterpret_cast<uint64_t>(dst_base);
    if ((flags & GFD_GATHER_PEER_DST) != 0 ? !check_peer_dev(ctx, dlo, dst_bytes) : !check_dev(ctx, dlo, dst_bytes))
        return set_error(ctx, GFD_ERR_INVALID,
                         (flags & GFD_GATHER_PEER_DST) != 0
                             ? "gather_device: dst window is not inside one allocation of this GPU or a reachable peer"
                             : "gather_device: dst window is not inside one device allocation");
    if (!check_dev(ctx, reinterpret_cast<uint64_t>(d_entries), static_cast<uint64_t>(n) * sizeof(gfd_sg_entry)))
        return set_error(ctx, GFD_ERR_INVALID, "gather_device: entry array is not in device memory");
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
    // sources may lie in any host range this context knows and the driver still confirms
    std::vector<Range> hr = live_host_ranges(ctx);
    if (static_cast<uint64_t>(n) <= kListMax && hr.size() <= static_cast<size_t>(kListRanges)) {
        // short list: one launch, no plan
        ListArgs la;
        std::memset(&la, 0, sizeof(la));
        la.entries = d_entries;
        la.n = static_cast<uint32_t>(n);
        for (const Range& r : hr) {
            la.src_lo[la.n_src] = r.lo;
            la.src_hi[la.n_src] = r.hi;
            la.n_src++;
        }
        la.dst_lo = dlo;
        la.dst_hi = dlo + dst_bytes;
        la.hdr = ctx->d_hdr;
        cudaError_t e = launch_list_pull(la, ctx->num_sms, st);
        if (e != cudaSuccess) return cuda_error(ctx, e, "list pull kernel launch");
        ctx->last_device_stream = st;
        ctx->st_pulls++;
        ctx->st_calls++;
        ctx->st_entries += static_cast<uint64_t>(n);
        return GFD_OK;
    }
    int rc = ensure_device_scratch(ctx, static_cast<size_t>(n));
    if (rc != GFD_OK) return rc;

    PlanArgs p;
    std::memset(&p, 0, sizeof(p));
    p.entries = d_entries;
    p.n = static_cast<uint64_t>(n);
    for (const Range& r : hr) {
        if (p.src_ok.n == kMaxCheckRanges) break;
        p.src_ok.lo[p.src_ok.n] = r.lo;
        p.src_ok.hi[p.src_ok.n] = r.hi;
        p.src_ok.n++;
    }
    p.dst_ok.lo[0] = dlo;
    p.dst_ok.hi[0] = dlo + dst_bytes;
    p.dst_ok.n = 1;
    p.rows = ctx->d_rows;
    p.misc = ctx->d_misc;
    p.cta_first = ctx->d_cta_first;
    const int grid = std::min(2 * ctx->num_sms, kMaxPullGrid);
    p.grid = static_cast<uint32_t>(grid);
    p.hdr = ctx->d_hdr;
    p.tiles = ctx->d_tiles;
    cudaError_t e = launch_plan(p, st);
    if (e != cudaSuccess) return cuda_error(ctx, e, "plan kernel launch");
    ctx->last_device_stream = st;

    PullArgs a;
    std::memset(&a, 0, sizeof(a));
    a.rows = ctx->d_rows;
    a.misc = ctx->d_misc;
    a.cta_first = ctx->d_cta_first;
    a.hdr = ctx->d_hdr;
    a.done_ctr = nullptr;
    e = launch_pull(a, grid, st, false, true);
    if (e != cudaSuccess) return cuda_error(ctx, e, "pull kernel launch");
    ctx->st_pulls++;
    ctx->st_calls++;
    ctx->st_entries += static_cast<uint64_t>(n);
    return GFD_OK;
}

int gfd_gather_device_status(gfd_ctx* ctx, int64_t* first_bad_entry) {
    if (!ctx) return GFD_ERR_INVALID;
    std::lock_guard<std::mutex> lk(ctx->mu);
    CtxScope scope(ctx->cu_ctx);
    cudaError_t e = cudaStreamSynchronize(ctx->last_device_stream ? ctx->last_device_stream : ctx->stream);
    if (e != cudaSuccess) return cuda_error(ctx, e, "cudaStreamSynchronize");
    PlanHeader h;
    e = cudaMemcpy(&h, ctx->d_hdr, sizeof(h), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return cuda_error(ctx, e, "reading plan header");
    if (first_bad_entry) *first_bad_entry = h.bad_entry == ~0ull ? -1 : static_cast<int64_t>(h.bad_entry);
    if (h.status != GFD_OK)
        return set_error(ctx, GFD_ERR_INVALID, "gather_device: entry %lld rejected by validation",
                         (long long)h.bad_entry);
    return GFD_OK;
}

}  // extern "C"
