#pragma once
// Internal declarations shared by the libgfd_b200 translation units.

#include <cuda.h>
#include <cuda_runtime.h>
#include <atomic>
#include <cstdint>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "gfd_b200.h"
#include "table.h"

namespace gfdb {

// Pull work table (rows, run merging): see table.h.
// Values the pull kernel needs; either passed by value (host-built tables) or read
// from device memory (GPU-built tables, see PlanHeader).
constexpr uint64_t kLensFromStarts = 1;  // PullGeometry::flags: row len = next start - start

struct PullGeometry {
    uint64_t total;      // aligned stream bytes
    uint64_t per_cta;    // stream bytes per CTA (multiple of kPiece except the tail)
    uint64_t flags;      // kLensFromStarts: stream rows' len fields are not set
    uint32_t n_rows;
    uint32_t n_misc;
};

struct PlanHeader {
    PullGeometry geo;
    uint64_t bad_entry;  // first rejected entry index, or ~0
    uint32_t status;     // GFD_OK / GFD_ERR_INVALID
    uint32_t list_done;  // list_pull_kernel: CTAs finished in the current launch (0 between launches)
    unsigned long long list_nbad;  // list_pull_kernel: ~(first rejected entry), 0 = none (0 between launches)
};

// Short device-resident entry lists skip the plan: one kernel where each warp takes whole
// entries, validates them against these ranges and copies them (no run merging, which
// short lists gain little from).  Zero-initialised PlanHeader list fields are its
// between-launch state, so the static scratch of the allocation-free entry point works.
constexpr int kListRanges = 8;        // source ranges a short-list launch carries
constexpr uint32_t kListMax = 512;    // entries up to which a device list takes this kernel
struct ListArgs {
    const gfd_sg_entry* entries;
    uint32_t n;
    uint32_t n_src;
    uint64_t src_lo[kListRanges];
    uint64_t src_hi[kListRanges];
    uint64_t dst_lo, dst_hi;
    PlanHeader* hdr;  // status and first rejected entry, as the plan path reports them
};

constexpr int kPullThreads = 256;           // threads per pull CTA
constexpr int kPullWarps = kPullThreads / 32;
constexpr int kPullUnroll = 8;              // 16-byte loads in flight per thread
constexpr uint64_t kPiece = 512ull * kPullUnroll;  // bytes one warp moves per step
constexpr int kRowWindow = 256;             // rows staged in shared memory at a time

// Default path: a host->device call whose rows form at most this many evenly strided
// groups, each row at least kStridedCeMinRow long or the whole call at most
// kStridedCeSmallCall bytes, goes to the copy engines as 2D copies.
constexpr size_t kStridedCeGroups = 3;
constexpr uint64_t kStridedCeMinRow = 16384;
constexpr uint64_t kStridedCeSmallCall = 256 * 1024;

constexpr int kMaxPullGrid = 512;  // CTAs of one pull launch (first-row table inline)

// Small requests travel entirely in the kernel parameters (rows and per-CTA first rows),
// so the kernel does not start with a round trip to host memory for its table.  The
// structure stays under 1 KiB: larger parameter blocks roughly double the host-side
// launch cost on this platform.
constexpr int kInlineFirst = 64;  // CTAs whose first row can travel inline
constexpr int kInlineRows = 16;   // stream + misc rows that can travel inline

// Completion work of a ring drain (GPU-queued submit), done by the last CTA of the drain's
// pull kernel once every byte has landed: per-tile token counts, per-list completion,
// then read_idx / done_idx and their device-memory copies.  Built by the host-driven
// drain (gfd_ring_poll) from the descriptors it copied out of the ring.  The header
// travels in the kernel parameters;
// the per-tile / per-list tables (RingTables) in pinned host memory, one per staging
// slot, until the launch has completed.
constexpr int kEpiTiles = 1024;  // gfd::MAX_TILES
constexpr int kEpiLists = 512;   // gfd::MAX_SG_LISTS
struct RingTables {
    uint16_t tile_id[kEpiTiles];
    uint32_t tile_count[kEpiTiles];
    uint16_t list_id[kEpiLists];
};
struct RingDrain {
    volatile uint64_t* read_idx;         // DescriptorQueue::read_idx; null: not a ring drain
    volatile uint64_t* done_idx;         // DescriptorQueue::done_idx
    volatile uint64_t* mirror_read;      // QueueMirror::read_idx (may be null)
    volatile uint64_t* mirror_done;      // QueueMirror::done_idx (may be null)
    uint64_t* tile_done;                 // per-tile cumulative token counts (may be null)
    uint64_t* list_done;                 // d_list_done (may be null)
    volatile uint64_t* lists_completed;  // SGTaskQueue::lists_completed (may be null)
    const RingTables* tables;            // set by the launcher (staging slot)
    uint64_t end;                        // slots below this are drained
    uint32_t n_tiles;                    // entries used in tile_id / tile_count
    uint32_t n_lists;                    // entries used in list_id
    uint32_t lists_landed;               // lists whose last descriptor is in this drain
    uint32_t _pad;
};

struct PullArgs {
    const PullRow* rows;        // stream rows, device-visible; null: rows_inline[0, n_rows)
    const uint32_t* cta_first;  // first row of each CTA (device-visible), or null:
                                // then cta_first_inline is used
    const PullRow* misc;        // misc rows; null: rows_inline[n_rows, n_rows + n_misc)
    const PlanHeader* hdr;      // non-null: read geometry from here (GPU-built table)
    PullGeometry geo;           // used when hdr == null
    uint32_t* done_ctr;         // device counter for last-CTA detection (may be null)
    volatile uint64_t* done_flag;  // host-mapped word set to done_value at the end
    uint64_t done_value;
    unsigned long long* bytes_ctr;  // optional device byte counter
    uint32_t sys_fence;             // destinations are host memory: system-scope fence per CTA
                                    // before the completion count (device -> host scatter)
    RingDrain drain;                // ring drain completion run by the last CTA (read_idx null: none)
    uint32_t cta_first_inline[kInlineFirst];
    PullRow rows_inline[kInlineRows];
};
static_assert(sizeof(PullArgs) <= 1024, "pull kernel parameters stay within 1 KiB");

// Source pools / destination windows the GPU plan validates against.
constexpr int kMaxCheckRanges = 32;
struct RangeTable {
    uint64_t lo[kMaxCheckRanges];
    uint64_t hi[kMaxCheckRanges];
    uint32_t n;
};

// Per-tile totals of a multi-CTA plan (also used for the scanned carries).
struct TileTotals {
    unsigned long long bytes;  // stream bytes
    unsigned long long bad;    // first rejected entry, or ~0
    uint32_t heads;            // rows started
    uint32_t misc;             // misaligned rows
};

struct PlanArgs {
    const gfd_sg_entry* entries;  // entry list, device-visible
    uint64_t n;
    RangeTable src_ok;       // allowed source ranges (pinned host pools)
    RangeTable dst_ok;       // allowed destination ranges (device)
    PullRow* rows;           // out
    PullRow* misc;           // out
    uint32_t* cta_first;     // out [grid]
    uint32_t grid;           // pull grid size the table is built for
    PlanHeader* hdr;         // out
    TileTotals* tiles;       // scratch of plan_tile_slots(n) entries for lists longer than
                             // one tile (null: single-CTA plan)
};

// ---------------------------------------------------------------------------
// Launchers (gather.cu)
// ---------------------------------------------------------------------------
// bulk: the cp.async.bulk mover (host -> device only; GFD_GATHER_BULK_STAGE)
// after_plan: launched right behind launch_plan on the same stream (programmatic
// dependent launch: the CTAs become resident while the plan runs)
cudaError_t launch_pull(const PullArgs& a, int grid, cudaStream_t st, bool bulk = false, bool after_plan = false);
cudaError_t launch_list_pull(const ListArgs& a, int num_sms, cudaStream_t st);
// A ring drain (context.cpp): host-validated entries gathered on `st` through a staging
// slot, with `drain` completed by the pull kernel's last CTA (`tables` copied into the
// slot).  The caller holds ctx->mu.
int gather_drain(gfd_ctx* ctx, const gfd_sg_entry* entries, int64_t n, cudaStream_t st, const RingDrain& drain,
                 const RingTables& tables, unsigned long long* bytes_ctr);
// Sizes every staging slot for drains of `rows` entries (and their tables) up front, so
// a host-driven ring drain never allocates pinned memory.  The caller holds ctx->mu.
int reserve_drain_slots(gfd_ctx* ctx, size_t rows);
cudaError_t preload_gather_kernels();  // forces module loading (see gather.cu)
cudaError_t launch_plan(const PlanArgs& a, cudaStream_t st);
size_t plan_tile_slots(uint64_t n);  // TileTotals a plan of n entries needs (PlanArgs::tiles)
int pull_grid_for(uint64_t total_bytes, int num_sms);

// ---------------------------------------------------------------------------
// Host range registry (context.cpp)
// ---------------------------------------------------------------------------
struct Range {
    uint64_t lo, hi;  // [lo, hi)
    bool owned;       // allocated by this library (gfd_pool_alloc)
    bool registered;  // pinned by gfd_pool_register (needs unregister)
    int numa;
};

class RangeSet {
public:
    // Returns true if [p, p + n) lies in one known range.
    bool contains(uint64_t p, uint64_t n) const;
    // The range holding [p, p + n), or null.
    const Range* find(uint64_t p, uint64_t n) const;
    void add(const Range& r);
    bool remove(uint64_t lo, Range* out);
    std::vector<Range> snapshot() const;

private:
    std::vector<Range> v_;  // sorted by lo, non-overlapping
};

// Staging slot for host-built tables (pinned, device-mapped host memory).
struct StageSlot {
    PullRow* rows = nullptr;         // capacity rows (stream rows then misc rows)
    uint32_t* cta_first = nullptr;   // capacity_cta
    size_t capacity = 0;
    size_t capacity_cta = 0;
    RingTables* tables = nullptr;    // ring drain tables (pinned, allocated on first use)
    volatile uint64_t* flag = nullptr;  // completion word written by the pull kernel
    uint64_t issued = 0;                // last done_value issued on this slot
    cudaStream_t stream = nullptr;      // stream of that launch
};

}  // namespace gfdb

struct gfd_ctx {
    int device = 0;
    CUcontext cu_ctx = nullptr;     // the CUDA context every call of this gfd_ctx runs in
    bool primary_retained = false;  // cu_ctx is the device's primary context, retained here
    int num_sms = 0;
    cudaStream_t stream = nullptr;       // high priority, non-blocking
    cudaStream_t ce_streams[3] = {};
    cudaEvent_t ce_events[3] = {};
    cudaEvent_t join_event = nullptr;
    uint64_t timeout_ns = 10ull * 1000 * 1000 * 1000;
    uint64_t ce_threshold = ~0ull;
    int ce_pending = 0;  // copy-engine streams whose copies st has not joined yet

    std::mutex mu;            // serialises calls on this context
    std::string last_error;

    gfdb::RangeSet host_ranges;  // pinned, device-mapped host memory
    gfdb::RangeSet dev_ranges;   // device allocations on `device`

    // staging ring for host-built tables
    static constexpr int kSlots = 4;
    gfdb::StageSlot slots[kSlots];
    uint64_t* flags_host = nullptr;   // kSlots completion words (pinned)
    int next_slot = 0;
    uint64_t seq = 0;

    // device scratch: done counters + GPU-built tables
    uint32_t* d_done_ctr = nullptr;   // kSlots + 1 counters
    gfdb::PullRow* d_rows = nullptr;
    gfdb::PullRow* d_misc = nullptr;
    uint32_t* d_cta_first = nullptr;
    gfdb::PlanHeader* d_hdr = nullptr;
    size_t d_capacity = 0;
    cudaStream_t last_device_stream = nullptr;  // stream of the last gfd_gather_device
    gfdb::TileTotals* d_tiles = nullptr;        // multi-CTA plan scratch (plan_tile_slots(d_capacity))
    uint16_t* d_sel = nullptr;                  // routing scratch: top-k expert ids per token
    size_t d_sel_capacity = 0;

    std::vector<void*> retired_host;       // outgrown staging tables (pinned), freed with the context
    std::vector<void*> retired_dev;        // outgrown device scratch, freed with the context
    std::vector<gfdb::PullRow> host_rows;  // scratch for building tables
    std::vector<gfdb::PullRow> host_misc;
    std::vector<gfd_sg_entry> ce_runs;
    std::vector<gfd_sg_entry> pageable_runs;  // runs from pageable sources (GFD_GATHER_PAGEABLE)
    std::vector<gfdb::PullRow> ce_rows;   // ce_runs as rows, then grouped into ce_copies
    std::vector<gfdb::CeCopy> ce_copies;

    std::atomic<uint64_t> st_calls{0}, st_entries{0}, st_bytes{0}, st_pulls{0}, st_ce{0},
        st_rejected{0}, st_prep_ns{0}, st_launch_ns{0}, st_wait_ns{0};
};

namespace gfdb {

// Driver entry points (resolved once through cudaGetDriverEntryPoint; the runtime is
// linked statically and libcuda is never linked directly).
struct Driver {
    CUresult (*ctx_get_current)(CUcontext*) = nullptr;
    CUresult (*ctx_set_current)(CUcontext) = nullptr;
    CUresult (*ctx_push)(CUcontext) = nullptr;
    CUresult (*ctx_pop)(CUcontext*) = nullptr;
    CUresult (*device_get)(CUdevice*, int) = nullptr;
    CUresult (*primary_retain)(CUcontext*, CUdevice) = nullptr;
    CUresult (*primary_release)(CUdevice) = nullptr;
    CUresult (*ptr_attrs)(unsigned int, CUpointer_attribute*, void**, CUdeviceptr) = nullptr;
    CUresult (*ctx_get_id)(CUcontext, unsigned long long*) = nullptr;  // may be null (older drivers)
    bool ok = false;
};
const Driver& driver();

// Makes `c` the calling thread's current context for the scope (no-op when it already
// is).  Every entry point of a gfd_ctx runs inside one, so the library uses the
// context its gfd_ctx was created in even when the caller has another one current.
class CtxScope {
public:
    explicit CtxScope(CUcontext c);
    ~CtxScope();
    CtxScope(const CtxScope&) = delete;
    CtxScope& operator=(const CtxScope&) = delete;

private:
    bool pushed_ = false;
};

int set_error(gfd_ctx* ctx, int code, const char* fmt, ...);
int cuda_error(gfd_ctx* ctx, cudaError_t e, const char* what);

// Classify [p, p+n) through the driver (cuPointerGetAttributes) and cache the
// allocation's range.  kind: 0 host pinned (device-mapped), 1 device memory of ctx.
bool discover_range(gfd_ctx* ctx, uint64_t p, uint64_t n, int kind);
bool check_host(gfd_ctx* ctx, uint64_t p, uint64_t n);
bool check_dev(gfd_ctx* ctx, uint64_t p, uint64_t n);
// The context's host ranges that are still live allocations (stale ones are dropped).
std::vector<Range> live_host_ranges(gfd_ctx* ctx);

// Builds rows for a host entry array; returns GFD_OK or GFD_ERR_INVALID.
int build_host_table(gfd_ctx* ctx, const gfd_sg_entry* e, int64_t n, bool validate,
                     uint64_t ce_threshold, PullGeometry* geo, uint64_t* bytes);

// Waits (bounded) for a host-mapped word to reach `value`.
bool wait_flag(volatile uint64_t* flag, uint64_t value, uint64_t timeout_ns, cudaStream_t st,
               cudaError_t* err);

uint64_t now_ns();

}  // namespace gfdb
