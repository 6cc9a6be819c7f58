/*
 * gfd_b200.h -- C ABI of the B200-native scattered host->device gather library.
 *
 * Plain C types only (pointers, sizes, integer status codes), so any FFI can bind
 * it: ctypes, cgo, JNI, N-API.  The C++ drop-in API in include/gfd/ (CpuPollingThread,
 * WarpSpecSession, SGWarpSpecSession, device primitives) is implemented on top of
 * these entry points.
 *
 * Data path: sm_100a kernels read the scattered tokens directly out of pinned,
 * device-mapped host memory over PCIe (16-byte vector loads, one warp per >= 512 B
 * span) and store them to HBM; evenly strided layouts may go to the copy engines as 2D
 * copies instead (see GFD_GATHER_DEFAULT).  No host core copies payload bytes (the one
 * exception is opt-in: under GFD_GATHER_PAGEABLE the CUDA driver stages pageable sources).
 *
 * Error behaviour: every entry point returns GFD_OK (0) or a GFD_ERR_* code and
 * never throws; gfd_last_error() gives a one-line reason for the last failure on
 * that context.  Entries are validated before any kernel reads them: a source
 * outside pinned host memory (outside mapped host memory under GFD_GATHER_PAGEABLE),
 * a destination outside device memory of the context's
 * GPU, or a range running past its allocation is rejected with GFD_ERR_INVALID and
 * nothing is copied.
 */
#ifndef GFD_B200_H
#define GFD_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GFD_B200_ABI_VERSION 1

enum {
    GFD_OK = 0,
    GFD_ERR_INVALID = 1,      /* bad argument or entry rejected by validation      */
    GFD_ERR_TIMEOUT = 2,      /* a bounded wait (host or device) expired           */
    GFD_ERR_CUDA = 3,         /* CUDA runtime / driver call failed                 */
    GFD_ERR_NOMEM = 4,        /* host or device allocation failed                  */
    GFD_ERR_UNSUPPORTED = 5,  /* feature unavailable on this device / build        */
    GFD_ERR_STATE = 6         /* call not valid in the object's current state      */
};

/* One scatter-gather entry.  Same layout as gfd::SGEntry
 * (reference include/gfd/copy_engine.h:29-33): dst device pointer, src host
 * pointer, size in bytes; 24 bytes. */
typedef struct gfd_sg_entry {
    uint64_t dst;
    const void* src;
    size_t size;
} gfd_sg_entry;

/* gfd_gather* flags */
#define GFD_GATHER_DEFAULT 0u      /* SM pull, except host->device calls that reduce to at most
                                      three evenly strided groups of rows >= 16 KiB (or of any
                                      length when the call is <= 256 KiB): those go to the copy
                                      engines as 2D copies, which measured faster             */
#define GFD_GATHER_FORCE_CE 1u     /* copy engine (one copy per merged run or strided group)  */
#define GFD_GATHER_AUTO_CE 2u      /* copy engine only for runs >= the context's CE threshold */
#define GFD_GATHER_TRUSTED 4u      /* skip host-side range validation (caller guarantees)   */
#define GFD_GATHER_FORCE_PULL 8u   /* SM pull for every entry, never the copy engine        */
#define GFD_GATHER_PEER_DST 32u    /* gfd_gather_device only: the destination window may lie
                                      in another GPU's memory that this context reaches (peer
                                      access enabled, or a CUDA IPC mapping): the pull reads
                                      over this GPU's host link and stores over NVLink, so a
                                      GPU with a faster host link can fetch rows for a peer   */
#define GFD_GATHER_BULK_STAGE 16u  /* SM pull whose warps move 4 KiB pieces with cp.async.bulk
                                      (host memory -> shared memory -> HBM) instead of 16-byte
                                      loads and stores; implies FORCE_PULL unless FORCE_CE or
                                      AUTO_CE is set; host -> device only (scatter ignores it).
                                      Measured at the same rate as the default pull: the
                                      link's 128-byte read requests bound both             */
#define GFD_GATHER_PAGEABLE 64u    /* gfd_gather / gfd_gather_sync only: a source outside
                                      pinned memory is accepted when every page it covers is
                                      mapped host memory (malloc, mmap, stack) that the driver
                                      does not know as device or managed memory.  A kernel
                                      cannot read such pages, so their runs go to the copy
                                      engine (cudaMemcpyAsync from pageable memory, which the
                                      CUDA driver stages through its own pinned buffers);
                                      pinned entries of the same call still take the SM pull.
                                      Unmapped pages are rejected with GFD_ERR_INVALID before
                                      anything is copied.  Not with GFD_GATHER_TRUSTED
                                      (refused: the source check is what finds pageable
                                      runs).  CpuPollingThread::submit_direct
                                      sets it: the reference's CPU gather reads any host
                                      memory (src/direct_submit.cpp:68-142)                 */

typedef struct gfd_ctx gfd_ctx;
typedef struct gfd_ring gfd_ring;

typedef struct gfd_stats {
    uint64_t calls;           /* gather calls accepted                 */
    uint64_t entries;         /* entries moved                         */
    uint64_t bytes;           /* payload bytes moved                   */
    uint64_t pull_launches;   /* SM-pull kernel launches               */
    uint64_t ce_copies;       /* copy-engine copies issued             */
    uint64_t rejected;        /* calls rejected by validation          */
    uint64_t prep_ns;         /* host time validating entries / building row tables */
    uint64_t launch_ns;       /* host time issuing kernels and copies               */
    uint64_t wait_ns;         /* host time waiting for completion (sync calls)      */
} gfd_stats;

/* ---- context (one per GPU; thread-safe) ------------------------------------
 * Replaces the per-GPU CUDA context + copy-engine setup of the reference
 * (CpuPollingThread::init_copy_engine, src/cpu_polling.cpp:141;
 *  CopyEngineManager::init, src/copy_engine.cpp:13-46).                      */
int gfd_ctx_create(int device, gfd_ctx** out);
int gfd_ctx_destroy(gfd_ctx* ctx);
int gfd_ctx_device(const gfd_ctx* ctx);
const char* gfd_last_error(const gfd_ctx* ctx);
/* Bound for host-side waits of this context (default 10 s). */
int gfd_set_timeout_ns(gfd_ctx* ctx, uint64_t ns);
/* Runs at least this long go to the copy engine under GFD_GATHER_AUTO_CE. */
int gfd_set_ce_threshold(gfd_ctx* ctx, uint64_t bytes);
int gfd_get_stats(const gfd_ctx* ctx, gfd_stats* out);

/* ---- host pools --------------------------------------------------------------
 * Pinned, device-mapped host memory bound to a NUMA node (numa_node < 0: the GPU's
 * own node).  Replaces the reference's pinned pools and hugepage staging
 * (include/gfd/staging_pool.h:29-189; examples/05_multi_gpu_benchmark.cu:217-231).
 * Memory obtained from cudaMallocHost / cudaHostAlloc elsewhere is accepted without
 * registration; gfd_pool_register pins caller-owned (malloc/mmap) memory.        */
int gfd_pool_alloc(gfd_ctx* ctx, size_t bytes, int numa_node, void** out_host);
int gfd_pool_free(gfd_ctx* ctx, void* host);
int gfd_pool_register(gfd_ctx* ctx, void* host, size_t bytes);
int gfd_pool_unregister(gfd_ctx* ctx, void* host);
/* NUMA node that a pool from gfd_pool_alloc is bound to (-1: not bound; any address
 * inside the pool).  An explicit numa_node that the host cannot bind makes
 * gfd_pool_alloc fail with GFD_ERR_INVALID; the GPU's own node (numa_node < 0) is used
 * when the host reports one and binds, else the pool stays unbound.  The reference
 * places pools with set_mempolicy(MPOL_BIND) around cudaMallocHost
 * (examples/05_multi_gpu_benchmark.cu:217-231) and does not report the node.       */
int gfd_pool_numa_node(gfd_ctx* ctx, const void* host, int* node);

/* ---- direct submit -------------------------------------------------------------
 * Gather n entries (host array; copied before return) into device memory.
 * gfd_gather is asynchronous on `stream` (NULL: the context's stream); the entry
 * array may be reused as soon as the call returns.  gfd_gather_sync waits for the
 * bytes to land and reports the host wall-clock latency in microseconds.
 * Replaces CpuPollingThread::submit_direct (reference src/direct_submit.cpp:28-164)
 * and its CPU gather + CE DMA data path (src/parallel_gather.cpp:10-116,
 * src/copy_engine.cpp:89-177).                                                   */
int gfd_gather(gfd_ctx* ctx, const gfd_sg_entry* entries, int64_t n, void* stream, uint32_t flags);
int gfd_gather_sync(gfd_ctx* ctx, const gfd_sg_entry* entries, int64_t n, uint32_t flags,
                    double* elapsed_us);
/* ---- device -> host scatter (reverse path) ------------------------------------
 * The reverse of gfd_gather: entries {dst, src, size} with dst in pinned,
 * device-mapped host memory and src in device memory of the context's GPU (KV-cache
 * offload, spilling activations).  Same kernel, validation, run merging, flags and
 * staging as gfd_gather; each CTA fences at system scope before the completion word,
 * so the bytes are visible to the CPU when gfd_scatter_sync returns (gfd_scatter:
 * when `stream` is synchronised).  No counterpart exists in the reference; it is the
 * future work its architecture notes name (docs/Architecture.md:993).            */
int gfd_scatter(gfd_ctx* ctx, const gfd_sg_entry* entries, int64_t n, void* stream, uint32_t flags);
int gfd_scatter_sync(gfd_ctx* ctx, const gfd_sg_entry* entries, int64_t n, uint32_t flags,
                     double* elapsed_us);

/* Same as gfd_gather, for an entry array already resident in device memory (e.g. written by a
 * routing kernel).  The GPU validates every entry against the context's pools and
 * the window [dst_base, dst_base + dst_bytes), merges contiguous runs (warp ballot +
 * prefix scan) and pulls them.  `status` (may be NULL) receives GFD_OK or
 * GFD_ERR_INVALID after the stream reaches the call; rejected entries are skipped.
 * flags: 0, or GFD_GATHER_PEER_DST (the window is one allocation of a peer GPU that this
 * context can access; the entry array stays in this GPU's memory). */
int gfd_gather_device(gfd_ctx* ctx, const gfd_sg_entry* d_entries, int64_t n, void* dst_base,
                      size_t dst_bytes, void* stream, uint32_t flags);
/* Status of the most recent gfd_gather_device on this context (synchronises). */
int gfd_gather_device_status(gfd_ctx* ctx, int64_t* first_bad_entry);

/* ---- allocation-free device gather --------------------------------------------
 * No counterpart in the reference.  For callers that may not allocate device memory
 * themselves: operator plugins inside an engine that owns all device memory through
 * its own pooling allocator, and latency-critical serving paths where cudaMalloc /
 * cudaFree (which can synchronise the device or fail under a memory budget) must not
 * run.  Same work as gfd_gather_device, without a gfd_ctx and without allocating:
 * its scratch is a fixed device array of about 258 KiB per GPU, held until exit.
 *   - at most GFD_NOALLOC_MAX_ENTRIES entries per call (more: GFD_ERR_INVALID and a
 *     message on stderr); n == 0 is a no-op;
 *   - src_base/src_bytes: a pinned, device-mapped host window holding every source;
 *     dst_base/dst_bytes: a device window holding every destination; entries outside
 *     them are skipped and reported through status_out; each window (and the entry
 *     list) must lie inside one allocation -- one mapping, for cuMemMap'd memory --
 *     or the call returns GFD_ERR_INVALID;
 *   - status_out (NULL or 2 x int64 in device or pinned host memory) receives
 *     {GFD_OK or GFD_ERR_INVALID, first rejected entry or -1} when `stream` reaches
 *     the call;
 *   - runs in the calling thread's current CUDA context; the first call in each
 *     context resolves the scratch array's address (cudaGetSymbolAddress) and keeps it
 *     under the context's driver ID, so a context destroyed and replaced by another
 *     (even one given the same handle) resolves afresh -- make the first call in each
 *     context before any stream capture;
 *   - every call on a GPU shares the one scratch array: calls that overlap on the GPU
 *     race and must be ordered by the caller (same stream, or events).            */
#define GFD_NOALLOC_MAX_ENTRIES 4096
int gfd_gather_device_noalloc(const gfd_sg_entry* d_entries, int64_t n, const void* src_base,
                              size_t src_bytes, void* dst_base, size_t dst_bytes, void* stream,
                              int64_t* status_out);

/* ---- MoE routing front end -----------------------------------------------------
 * Routes `tokens` tokens over `experts` experts from fp32 router logits (device,
 * row-major [tokens x experts]) and gathers the selected rows into per-expert
 * contiguous segments of dst_base, all stream-ordered on the GPU with no host round
 * trip.  Each token picks its k highest logits (ties: lower expert id first; NaN
 * ranks below every number).  The destination holds tokens*k rows of row_bytes:
 * expert 0's rows first, then expert 1's, ..., each expert's rows in ascending token
 * order -- the order of the reference's per-expert SG lists
 * (examples/09_sg_warp_spec.cu:246-276).  Row of token t comes from the pinned host
 * address d_token_src[t] (device array).  Outputs (device): d_counts[e] rows routed to
 * e, d_offsets[e] first row of e's segment, d_entries (tokens*k) the gather list.
 * experts <= 1024, k <= 32.  GFD_MOE_ROUTE_ONLY: route and write the list, skip the
 * gather.  The gather itself is gfd_gather_device (status via
 * gfd_gather_device_status).                                                      */
#define GFD_MOE_ROUTE_ONLY 1u
int gfd_moe_route_gather(gfd_ctx* ctx, const float* d_logits, int64_t tokens, int experts, int k,
                         const uint64_t* d_token_src, size_t row_bytes, void* dst_base,
                         size_t dst_bytes, uint32_t* d_counts, uint32_t* d_offsets,
                         gfd_sg_entry* d_entries, void* stream, uint32_t flags);

/* ---- GPU-queued submit: descriptor ring consumer ------------------------------
 * Attaches to a gfd::DescriptorQueue written by GPU producers (device.cuh /
 * device_primitives.cuh / sg protocol).  Between gfd_ring_start and gfd_ring_stop a
 * device-resident kernel (the ring agent: one front CTA + `movers` mover CTAs) polls
 * the commit markers, copies committed runs out, clears the markers, advances read_idx,
 * validates and run-merges the descriptors, pulls the bytes and publishes done_idx (and,
 * when attached, per-tile counters or per-list completion).  No host core reads a
 * descriptor or a payload byte.  Replaces the reference's CPU poller + batch processor
 * (src/cpu_polling.cpp:337-436, src/batch_processor.cpp:69-831).
 * `tiled` is a gfd::TiledQueue* whose .base is `queue` (or NULL); `sg` is a
 * gfd::SGTaskQueue* for per-list signalling (or NULL).                          */
int gfd_ring_create(gfd_ctx* ctx, void* queue, void* tiled, void* sg, gfd_ring** out);
int gfd_ring_destroy(gfd_ring* ring);
/* Launches the agent (in resident mode: returns once all its CTAs run, GFD_ERR_TIMEOUT
 * if they cannot become resident within 2 s, so kernels launched afterwards find it on
 * the GPU).  By default the agent leaves after `linger_ns` with nothing committed
 * (cudaDeviceSynchronize and cudaFree wait for every kernel of the context) and a
 * service thread relaunches it when the next commit marker appears; that thread reads
 * no descriptor or payload, only answers range queries (below) and watches one marker
 * while the agent is away.
 * Sources must be pinned, device-mapped host memory and destinations device memory of
 * the context's GPU: the agent checks every descriptor against ranges it has cached
 * and asks the host once about a range it has not seen (rejected descriptors are
 * skipped, counted and their run still completes). */
int gfd_ring_start(gfd_ring* ring);
/* Stops the agent after it has drained every slot committed so far.  Once stopped (and
 * in gfd_ring_destroy) the ring no longer reads the queue, so the caller may free it. */
int gfd_ring_stop(gfd_ring* ring);
/* Without gfd_ring_start: one drain pass from the calling thread (the descriptors are
 * read and validated on the host; one pull kernel per committed run); *launched = number
 * of drains launched.  While the ring runs it does nothing (the agent consumes). */
int gfd_ring_poll(gfd_ring* ring, int* launched);
/* Waits until done_idx >= target (bounded by the context timeout). */
int gfd_ring_wait(gfd_ring* ring, uint64_t target);
int gfd_ring_counters(const gfd_ring* ring, uint64_t* consumed, uint64_t* drains,
                      uint64_t* bytes);
/* Agent settings, before gfd_ring_start (the environment variables GFD_RING_MOVERS,
 * GFD_RING_LINGER_NS and GFD_RING_RESIDENT set the same at gfd_ring_create):
 * movers: mover CTAs (1..32, 0: 8); linger_ns: idle time before the agent leaves
 * (default 20 us); resident != 0: the agent stays until gfd_ring_stop (bounded by the
 * context timeout when idle) -- for producer kernels that occupy every SM and wait on
 * done_idx; the application then synchronises with streams or events, because
 * cudaDeviceSynchronize waits for the agent too, and loads its kernels before the ring
 * starts (cudaFuncGetAttributes, or CUDA_MODULE_LOADING=EAGER): with lazy loading, the
 * first launch of a kernel waits for the kernels already running, the agent included.
 * No counterpart in the reference, whose consumer is a host thread.                  */
int gfd_ring_configure(gfd_ring* ring, uint32_t movers, uint64_t linger_ns, int resident);
/* Declares a window the agent may trust without asking (pinned host memory as a source,
 * device memory as a destination); bytes == 0: the whole allocation holding ptr.
 * CpuPollingThread::start declares its constructor's gpu_base / cpu_base this way.    */
int gfd_ring_allow(gfd_ring* ring, const void* ptr, size_t bytes);
/* What the agent did so far. */
typedef struct gfd_ring_agent_stats_t {
    uint64_t launches;      /* agent launches (start + relaunches after idle exits)        */
    uint64_t queries;       /* range queries the agent asked the host                      */
    uint64_t rejected;      /* descriptors rejected by validation                          */
    uint64_t timeouts;      /* bounded waits of the agent that gave up                     */
    uint64_t idle_exits;    /* launches that ended after linger_ns / the idle bound         */
    uint64_t stop_exits;    /* launches that ended on gfd_ring_stop                        */
    uint64_t error_exits;   /* launches that ended on a wait that gave up                  */
    uint64_t resident;      /* 1 if the ring is configured resident                        */
    /* last launch, nanoseconds after its front CTA started (0: did not happen):           */
    uint64_t last_first_batch_ns;  /* first batch published                                 */
    uint64_t last_done_ns;         /* last batch completed (done_idx published)            */
    uint64_t last_exit_ns;         /* launch ended                                          */
} gfd_ring_agent_stats_t;
int gfd_ring_agent_stats(const gfd_ring* ring, gfd_ring_agent_stats_t* out);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif /* GFD_B200_H */
