// MoE gather through SGWarpSpecSession with lists submitted on the GPU: the reference's
// dynamic-submission pattern (examples/09_sg_warp_spec.cu:244-294: a submitter warp turns
// routing decisions into one SG list per expert while the transfer and compute warps of
// the same kernel consume them), fed by this library's routing kernels
// (gfd_moe_route_gather with GFD_MOE_ROUTE_ONLY writes the per-expert entry list, counts
// and offsets).  Built as libgfd_moe_sg.so, a client of libgfd_b200.so.
//
// Kernel shape: every CTA runs the SG framework (producer warps pull each list's
// rows from pinned host memory, the compute warp runs the functor); CTA 0 has one
// more warp, the submitter, which walks the experts in ascending order, waits (bounded)
// for pool and ring space, writes the expert's entries into the pool (the session's
// device pool: SG_FLAG_DEVICE_ENTRIES lists) and commits the list.  When every list has completed it raises sq->terminate, which ends the
// framework warps.  32,768 entries pass through the 16,384-entry pool in waves.

#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>

#include "gfd/sg_device_primitives.cuh"
#include "gfd/sg_warp_spec.cuh"
#include "gfd/warp_spec_session.h"
#include "gfd_b200.h"

namespace {

struct NoCompute {
    __device__ void operator()(const gfd::sg_warp_spec::SGListView&) const {}
};

struct Routed {
    const gfd_sg_entry* entries;  // per-expert contiguous, experts ascending
    const uint32_t* counts;       // rows per expert
    const uint32_t* offsets;      // first row of each expert
    uint32_t experts;
    uint32_t rows_per_list;       // split an expert's rows into lists of at most this many (0: one list)
};

__global__ void __launch_bounds__(GFD_SG_WARP_SPEC_MAX_THREADS)
    moe_sg_kernel(gfd::DescriptorQueue* dq, gfd::SGTaskQueue* sq, NoCompute fn, Routed rt, uint32_t framework_warps) {
    const uint32_t warp = threadIdx.x >> 5;
    if (warp < framework_warps) {
        gfd::sg_warp_spec::_sg_transfer_warp_loop(dq, sq, fn, framework_warps);
        return;
    }
    if (blockIdx.x != 0 || warp != framework_warps) return;

    // ---- submitter warp (CTA 0) ----
    // Each expert's lists go out in batches of up to kBatchRows rows: one pool
    // reservation and one slot reservation per batch, the entries and headers written,
    // then one fence and the markers (SGSubmitter::publish), so the fence's PCIe round
    // trips are paid once per batch.  Batches stay within one expert: lists of the same
    // batch start together and end together, and larger batches (tried across experts)
    // made the consumers' in-order releases arrive in bursts.
    const uint32_t lane = threadIdx.x & 31;
    const gfd::sg::SGSubmitter sub(sq);
    constexpr uint32_t kBatchRows = gfd::MAX_SG_POOL_ENTRIES / 8;
    uint64_t lists = 0;
    uint32_t batch = 0;
    for (uint32_t e = 0; e < rt.experts; ++e) {
        const uint32_t rows = rt.counts[e];
        // one list per expert unless asked otherwise, but never more than half the pool
        uint32_t per = rt.rows_per_list ? rt.rows_per_list : rows;
        if (per > gfd::MAX_SG_POOL_ENTRIES / 2) per = gfd::MAX_SG_POOL_ENTRIES / 2;
        const uint32_t batch_lists = per >= kBatchRows ? 1u : kBatchRows / per;
        for (uint32_t first = 0; first < rows; ++batch) {
            uint32_t n = 0, batch_rows = 0;
            while (n < batch_lists && first + batch_rows < rows) {
                const uint32_t c = rows - first - batch_rows < per ? rows - first - batch_rows : per;
                batch_rows += c;
                ++n;
            }
            if (!sub.wait_entry_space(batch_rows) || !sub.wait_list_space(n) ||
                (batch % 8 == 0 && __shfl_sync(0xffffffffu, sq->wait_timeouts, 0) != 0)) {
                e = rt.experts;  // a wait gave up (here or in a consumer): the pass has failed
                break;
            }
            const uint64_t po = sub.alloc_entries(batch_rows);
            const uint64_t ls = sub.alloc_list(n);
            const uint32_t off = rt.offsets[e] + first;
            // With the session's mirror the lists are device-entry lists: entries and
            // headers go to device memory and commit with device fences, so nothing of a
            // list crosses PCIe (posted writes to host memory and system fences wait behind
            // the payload reads once the link is saturated, which held back the first lists
            // of a pass by ~200 us).  Without it the pool in host memory is used.
            // Lane l writes 8-byte word l of each 256-byte group of the batch (a
            // DeviceSGEntry is three words: src, dst, size | tag << 32), so every store
            // instruction covers whole 128-byte lines, and each lane loads kWords words of
            // the routed list before storing any of them (one load per store made the loop
            // wait a memory latency per word).
            gfd::DeviceSGEntry* const dpool = sub.device_pool();
            {
                constexpr uint32_t kWords = 8;
                const uint64_t* in = reinterpret_cast<const uint64_t*>(rt.entries + off);  // dst, src, size
                uint64_t* pool = reinterpret_cast<uint64_t*>(dpool != nullptr ? dpool : sq->entries);
                const uint32_t nw = 3u * batch_rows;
                for (uint32_t w0 = 0; w0 < nw; w0 += 32u * kWords) {
                    uint64_t v[kWords];
#pragma unroll
                    for (uint32_t u = 0; u < kWords; ++u) {
                        const uint32_t w = w0 + u * 32u + lane;
                        const uint32_t i = w / 3u, f = w - 3u * i;
                        v[u] = w < nw ? in[3u * i + (f == 0 ? 1u : f == 1 ? 0u : 2u)] : 0ull;
                    }
#pragma unroll
                    for (uint32_t u = 0; u < kWords; ++u) {
                        const uint32_t w = w0 + u * 32u + lane;
                        if (w >= nw) break;
                        const uint32_t i = w / 3u, f = w - 3u * i;
                        const uint64_t x = f == 2 ? (v[u] & 0xffffffffull) | (static_cast<uint64_t>(e) << 32) : v[u];
                        pool[((po + i) % gfd::MAX_SG_POOL_ENTRIES) * 3u + f] = x;
                    }
                }
            }
            uint32_t done = 0;
            for (uint32_t j = 0; j < n; ++j) {
                const uint32_t c = batch_rows - done < per ? batch_rows - done : per;
                // list ids: the expert when it is one list, else a running number (entries
                // keep the expert in their tag)
                const uint32_t id = rt.rows_per_list ? static_cast<uint32_t>((lists + j) % gfd::MAX_SG_LISTS) : e;
                if (dpool != nullptr) sub.write_header_device(ls + j, po + done, c, id, gfd::SG_FLAG_NONE);
                else sub.write_header(ls + j, static_cast<uint32_t>(po + done), c, id, gfd::SG_FLAG_NONE);
                done += c;
            }
            if (dpool != nullptr) sub.publish_device(ls, n);
            else sub.publish(ls, n);
            lists += n;
            first += batch_rows;
        }
    }
    gfd::sg::sg_wait_list_done(sq, lists);
    __syncwarp();
    if (lane == 0) {
        __threadfence_system();
        sq->terminate = 1;
        if (sq->poll_mirror != nullptr) sq->poll_mirror->terminate = 1u;
        __threadfence_system();
    }
}

}  // namespace

struct gfd_moe_sg {
    gfd::SGWarpSpecSession* session = nullptr;
    gfd::SGWarpSpecSession::LaunchParams params{};
    bool prepared = false;
    cudaStream_t stream = nullptr;
};

extern "C" {

// producer_warps: pulling warps per CTA (0: the default); wait_timeout_ms: bound on every
// in-kernel wait (0: the default); num_blocks: CTAs of the SG kernel (0: one per SM).
int gfd_moe_sg_create(int producer_warps, uint64_t wait_timeout_ms, int num_blocks, gfd_moe_sg** out) {
    if (out == nullptr || num_blocks < 0) return GFD_ERR_INVALID;
    *out = nullptr;
    gfd::SGWarpSpecConfig cfg;
    cfg.num_compute_warps = 1;
    cfg.producer_warps = producer_warps;
    cfg.wait_timeout_ms = wait_timeout_ms;
    cfg.num_blocks = num_blocks;
    auto* m = new gfd_moe_sg;
    m->session = new gfd::SGWarpSpecSession(cfg);
    if (!m->session->ok()) {
        delete m->session;
        delete m;
        return GFD_ERR_CUDA;
    }
    *out = m;
    return GFD_OK;
}

// Resets the session's queues for the next pass (host work and small synchronous
// memsets: keep it outside a timed region).  The previous pass must be synchronised.
int gfd_moe_sg_prepare(gfd_moe_sg* m) {
    if (m == nullptr) return GFD_ERR_INVALID;
    m->session->reset();
    m->params = m->session->get_launch_params();
    m->prepared = true;
    return GFD_OK;
}

// Launches one prepared pass on `stream` over the lists of `experts` experts (device
// arrays written by gfd_moe_route_gather with GFD_MOE_ROUTE_ONLY, on the same stream).
// `stream` is a CUDA stream as given (NULL: the legacy default stream); pass the routing
// call the same non-NULL stream, since a NULL stream there means the context's stream.
// rows_per_list: split each expert's rows into lists of at most this many (0: one list
// per expert, the reference's shape).
int gfd_moe_sg_run(gfd_moe_sg* m, const gfd_sg_entry* d_entries, const uint32_t* d_counts, const uint32_t* d_offsets,
                   uint32_t experts, uint32_t rows_per_list, void* stream) {
    if (m == nullptr || !m->prepared || d_entries == nullptr || d_counts == nullptr || d_offsets == nullptr ||
        experts == 0 || experts > static_cast<uint32_t>(gfd::MAX_SG_LISTS) ||
        rows_per_list > static_cast<uint32_t>(gfd::MAX_SG_POOL_ENTRIES))
        return GFD_ERR_INVALID;
    const uint32_t fw = m->params.block.x / 32;
    const uint32_t threads = (fw + 1) * 32;
    if (threads > GFD_SG_WARP_SPEC_MAX_THREADS) return GFD_ERR_INVALID;
    m->prepared = false;
    m->stream = static_cast<cudaStream_t>(stream);
    moe_sg_kernel<<<m->params.grid, threads, 0, m->stream>>>(m->params.dq, m->params.sq, NoCompute{},
                                                             Routed{d_entries, d_counts, d_offsets, experts, rows_per_list}, fw);
    if (cudaPeekAtLastError() != cudaSuccess) return GFD_ERR_CUDA;
    m->session->get_poller()->start();
    return GFD_OK;
}

// Waits for the pass; reports in-kernel waits that gave up and the payload bytes moved.
int gfd_moe_sg_sync(gfd_moe_sg* m, uint64_t* timeouts, uint64_t* bytes) {
    if (m == nullptr) return GFD_ERR_INVALID;
    const cudaError_t e = cudaStreamSynchronize(m->stream);
    m->session->synchronize();
    const auto st = m->session->get_stats();
    const uint64_t to = m->session->timeouts();
    if (timeouts) *timeouts = to;
    if (bytes) *bytes = st.bytes_transferred;
    if (e != cudaSuccess) return GFD_ERR_CUDA;
    return to == 0 ? GFD_OK : GFD_ERR_TIMEOUT;
}

void gfd_moe_sg_destroy(gfd_moe_sg* m) {
    if (m == nullptr) return;
    delete m->session;
    delete m;
}

}  // extern "C"
