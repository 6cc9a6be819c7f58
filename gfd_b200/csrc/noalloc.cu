// gfd_gather_device_noalloc: the device-resident-entry gather (plan + pull, the same
// kernels as gfd_gather_device) with its scratch in a fixed, file-scope device array
// instead of memory obtained from cudaMalloc.
//
// Who needs it: code that is not allowed to allocate device memory on its own --
// operator plugins hosted by an inference engine or framework that owns every byte
// of device memory through its own pooling allocator, and latency-critical serving
// paths where cudaMalloc / cudaFree (which can synchronise the whole device and can
// fail under the host's memory budget) must not appear.  Such callers hand in their
// inputs (the entry list in device memory, the source and destination windows) and
// outputs (the destination bytes, an optional status word); this entry point calls
// no cudaMalloc, cudaFree or other allocating routine, and needs no gfd_ctx.
//
// Limits and sharing:
//   * at most GFD_NOALLOC_MAX_ENTRIES entries per call (rows for the stream part and
//     the unaligned part, the per-CTA first-row table and the header all live in the
//     array g_noalloc_scratch below, about 258 KiB, held by every GPU that loads the
//     library until the process exits);
//   * every call on a GPU uses the same array, which keeps the previous call's
//     contents; calls whose kernels overlap on that GPU (different streams without
//     ordering between them) race on it and must be ordered by the caller;
//   * nothing needs clearing between calls: the plan kernel writes the header, every
//     row it produces and every CTA's first-row index before the pull kernel reads
//     them.
// Set-up: the first call in each CUDA context (the device's primary context, or a
// context created with the driver API) resolves the array's device address with
// cudaGetSymbolAddress in that context (the array's name in host code is only a
// host-side stand-in, never a device address) and caches it under the context's
// driver ID (cuCtxGetId), which is never reused within a process -- a handle value
// can be, after a context is destroyed and another created, with the module loaded
// at a different address; make that first call before any stream capture.  Without
// cuCtxGetId (drivers before CUDA 12.0) the address is resolved on every call.
// Windows: the source window must lie inside one pinned host allocation, and the
// destination window, the entry list and the status words inside one device
// allocation each (one mapping, for memory mapped with cuMemMap); a window that
// spans several is refused with GFD_ERR_INVALID.

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <mutex>

#include "gfd/log.h"
#include "internal.h"

namespace gfdb {
namespace {

constexpr size_t kNoAllocRows = GFD_NOALLOC_MAX_ENTRIES;
constexpr size_t kRowsOff = 0;
constexpr size_t kMiscOff = kRowsOff + kNoAllocRows * sizeof(PullRow);
constexpr size_t kCtaOff = kMiscOff + kNoAllocRows * sizeof(PullRow);
constexpr size_t kHdrOff = (kCtaOff + kMaxPullGrid * sizeof(uint32_t) + 255) / 256 * 256;
constexpr size_t kScratchBytes = kHdrOff + 256;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

// The array's device address belongs to the CUDA context the module is loaded in, so
// the resolved address is cached per context (the primary context of a device, or a
// context the caller created with the driver API), keyed by the context's driver ID.
constexpr int kMaxContexts = 64;
struct ContextSlot {
    unsigned long long id = 0;         // cuCtxGetId of the context
    unsigned char* scratch = nullptr;  // device address of g_noalloc_scratch in it
    int num_sms = 0;
};

// ID of the calling thread's current context; false when there is none or the driver
// cannot tell (then nothing is cached).
bool current_ctx_id(unsigned long long* id) {
    const Driver& drv = driver();
    CUcontext cur = nullptr;
    if (drv.ctx_get_id == nullptr || drv.ctx_get_current(&cur) != CUDA_SUCCESS || cur == nullptr) return false;
    return drv.ctx_get_id(cur, id) == CUDA_SUCCESS;
}
ContextSlot g_ctx_slots[kMaxContexts];
int g_ctx_count = 0;
std::mutex g_ctx_mu;

// Copies the plan header's verdict to the caller's status words.
__global__ void noalloc_status_kernel(const PlanHeader* hdr, int64_t* out) {
    if (threadIdx.x == 0 && blockIdx.x == 0) {
        out[0] = static_cast<int64_t>(hdr->status);
        out[1] = hdr->bad_entry == ~0ull ? -1 : static_cast<int64_t>(hdr->bad_entry);
    }
}

struct PtrAttrs {
    unsigned mem_type = 0, managed = 0;
    int ordinal = -1;
    CUdeviceptr dptr = 0, lo = 0;
    size_t size = 0;
};

bool query(uint64_t p, PtrAttrs* r) {
    auto fn = driver().ptr_attrs;
    if (fn == nullptr) return false;
    CUpointer_attribute a[6] = {CU_POINTER_ATTRIBUTE_MEMORY_TYPE, CU_POINTER_ATTRIBUTE_DEVICE_ORDINAL,
                                CU_POINTER_ATTRIBUTE_DEVICE_POINTER, CU_POINTER_ATTRIBUTE_RANGE_START_ADDR,
                                CU_POINTER_ATTRIBUTE_RANGE_SIZE, CU_POINTER_ATTRIBUTE_IS_MANAGED};
    void* d[6] = {&r->mem_type, &r->ordinal, &r->dptr, &r->lo, &r->size, &r->managed};
    if (fn(6, a, d, static_cast<CUdeviceptr>(p)) == CUDA_SUCCESS) return true;
    *r = PtrAttrs();  // range attributes unsupported for this memory: the basic three
    void* d3[3] = {&r->mem_type, &r->ordinal, &r->dptr};
    const bool ok = fn(3, a, d3, static_cast<CUdeviceptr>(p)) == CUDA_SUCCESS;
    cudaGetLastError();
    return ok;
}

// true if [p, p+n) lies inside one allocation of the wanted kind:
// host == true: pinned host memory mapped at the same address on the device;
// host == false: device memory of `device` (or managed memory).
bool window_ok(uint64_t p, uint64_t n, bool host, int device) {
    if (n == 0 || p + n < p) return false;
    PtrAttrs a;
    if (!query(p, &a)) return false;
    if (host) {
        if (a.mem_type != CU_MEMORYTYPE_HOST || a.dptr != p) return false;
        if (a.size == 0) {  // no range information: both ends must be mapped host memory
            PtrAttrs b;
            return query(p + n - 1, &b) && b.mem_type == CU_MEMORYTYPE_HOST && b.dptr == p + n - 1;
        }
    } else if (!((a.mem_type == CU_MEMORYTYPE_DEVICE && a.ordinal == device) || a.managed)) {
        return false;
    }
    return a.size > 0 && a.lo <= p && p - a.lo <= a.size && n <= a.size - (p - a.lo);
}

}  // namespace
}  // namespace gfdb

extern "C" int gfd_gather_device_noalloc(const gfd_sg_entry* d_entries, int64_t n, const void* src_base,
                                         size_t src_bytes, void* dst_base, size_t dst_bytes, void* stream,
                                         int64_t* status_out) {
    using namespace gfdb;
    if (n < 0 || (n > 0 && d_entries == nullptr)) return GFD_ERR_INVALID;
    if (reinterpret_cast<uint64_t>(d_entries) & 7u) {
        std::fprintf(stderr, "gfd_gather_device_noalloc: entry array is not 8-byte aligned\n");
        return GFD_ERR_INVALID;
    }
    if (n > static_cast<int64_t>(GFD_NOALLOC_MAX_ENTRIES)) {
        GFD_LOG_ERROR("gfd_gather_device_noalloc: %lld entries exceed GFD_NOALLOC_MAX_ENTRIES (%d)\n",
                      (long long)n, GFD_NOALLOC_MAX_ENTRIES);
        return GFD_ERR_INVALID;
    }
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0) {
        cudaGetLastError();
        return GFD_ERR_CUDA;
    }
    const Driver& drv = driver();
    if (!drv.ok) return GFD_ERR_CUDA;
    unsigned char* scratch = nullptr;
    int num_sms = 0;
    {
        std::lock_guard<std::mutex> lk(g_ctx_mu);
        unsigned long long id = 0;
        if (current_ctx_id(&id))
            for (int i = 0; i < g_ctx_count; ++i)
                if (g_ctx_slots[i].id == id) {
                    scratch = g_ctx_slots[i].scratch;
                    num_sms = g_ctx_slots[i].num_sms;
                }
        if (scratch == nullptr) {
            // set-up, once per context: resolve the array's device address (this also
            // makes the device's primary context current when none was), load the kernels
            void* ptr = nullptr;
            cudaError_t err = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
            if (err == cudaSuccess) err = cudaDeviceGetAttribute(&num_sms, cudaDevAttrMultiProcessorCount, dev);
            cudaFuncAttributes fa;
            if (err == cudaSuccess) err = cudaFuncGetAttributes(&fa, noalloc_status_kernel);
            if (err == cudaSuccess) err = preload_gather_kernels();
            if (err != cudaSuccess || ptr == nullptr) {
                cudaGetLastError();
                GFD_LOG_ERROR("gfd_gather_device_noalloc: scratch set-up failed: %s\n", cudaGetErrorString(err));
                return GFD_ERR_CUDA;
            }
            // the set-up may have made the primary context current: cache under its ID
            if (current_ctx_id(&id) && g_ctx_count < kMaxContexts) {
                g_ctx_slots[g_ctx_count].id = id;
                g_ctx_slots[g_ctx_count].scratch = static_cast<unsigned char*>(ptr);
                g_ctx_slots[g_ctx_count].num_sms = num_sms;
                ++g_ctx_count;
            }
            scratch = static_cast<unsigned char*>(ptr);
        }
    }
    if (n == 0) return GFD_OK;
    const uint64_t slo = reinterpret_cast<uint64_t>(src_base);
    const uint64_t dlo = reinterpret_cast<uint64_t>(dst_base);
    if (!window_ok(slo, src_bytes, true, dev) || !window_ok(dlo, dst_bytes, false, dev) ||
        !window_ok(reinterpret_cast<uint64_t>(d_entries), static_cast<uint64_t>(n) * sizeof(gfd_sg_entry), false,
                   dev))
        return GFD_ERR_INVALID;
    if (status_out != nullptr) {
        const uint64_t sp = reinterpret_cast<uint64_t>(status_out);
        if (!window_ok(sp, 2 * sizeof(int64_t), false, dev) && !window_ok(sp, 2 * sizeof(int64_t), true, dev))
            return GFD_ERR_INVALID;
    }

    cudaStream_t st = static_cast<cudaStream_t>(stream);
    unsigned char* s = scratch;
    PullRow* rows = reinterpret_cast<PullRow*>(s + kRowsOff);
    PullRow* misc = reinterpret_cast<PullRow*>(s + kMiscOff);
    uint32_t* cta_first = reinterpret_cast<uint32_t*>(s + kCtaOff);
    PlanHeader* hdr = reinterpret_cast<PlanHeader*>(s + kHdrOff);
    const int grid = num_sms * 2 < kMaxPullGrid ? num_sms * 2 : kMaxPullGrid;

    if (static_cast<uint64_t>(n) <= kListMax) {
        // short list: one launch, no plan (the header's list fields start zeroed with the
        // static scratch and every launch leaves them so)
        ListArgs la;
        memset(&la, 0, sizeof(la));
        la.entries = d_entries;
        la.n = static_cast<uint32_t>(n);
        la.n_src = 1;
        la.src_lo[0] = slo;
        la.src_hi[0] = slo + src_bytes;
        la.dst_lo = dlo;
        la.dst_hi = dlo + dst_bytes;
        la.hdr = hdr;
        if (launch_list_pull(la, num_sms, st) != cudaSuccess) return GFD_ERR_CUDA;
        if (status_out != nullptr) {
            noalloc_status_kernel<<<1, 32, 0, st>>>(hdr, status_out);
            if (cudaGetLastError() != cudaSuccess) return GFD_ERR_CUDA;
        }
        return GFD_OK;
    }

    PlanArgs p;
    memset(&p, 0, sizeof(p));
    p.entries = d_entries;
    p.n = static_cast<uint64_t>(n);
    p.src_ok.lo[0] = slo;
    p.src_ok.hi[0] = slo + src_bytes;
    p.src_ok.n = 1;
    p.dst_ok.lo[0] = dlo;
    p.dst_ok.hi[0] = dlo + dst_bytes;
    p.dst_ok.n = 1;
    p.rows = rows;
    p.misc = misc;
    p.cta_first = cta_first;
    p.grid = static_cast<uint32_t>(grid);
    p.hdr = hdr;
    cudaError_t e = launch_plan(p, st);
    if (e != cudaSuccess) return GFD_ERR_CUDA;

    PullArgs a;
    memset(&a, 0, sizeof(a));
    a.rows = rows;
    a.misc = misc;
    a.cta_first = cta_first;
    a.hdr = hdr;
    e = launch_pull(a, grid, st);
    if (e != cudaSuccess) return GFD_ERR_CUDA;
    if (status_out != nullptr) {
        noalloc_status_kernel<<<1, 32, 0, st>>>(hdr, status_out);
        if (cudaGetLastError() != cudaSuccess) return GFD_ERR_CUDA;
    }
    return GFD_OK;
}
