#pragma once
// Copy-engine path and the scatter-gather entry type.
//
// Source-compatible with the reference interface include/gfd/copy_engine.h:10-100:
// GFD_CU_CHECK, MAX_CE_CHANNELS, MAX_SG_ENTRIES_PER_BATCH, SGEntry (24 bytes) and
// CopyEngineManager with the same methods.  In this library the copy engine is not
// the main data path (SM-pull kernels are); CopyEngineManager spreads copies over up to
// three high-priority streams in contiguous per-stream ranges as the reference does
// (src/copy_engine.cpp:89-153), merging entries that continue each other and issuing
// evenly strided runs as single 2D copies.

#include <cuda.h>
#include <cstdint>
#include <cstdio>

namespace gfd {

#define GFD_CU_CHECK(call)                                                              \
    do {                                                                                \
        CUresult gfd_cu_err_ = (call);                                                  \
        if (gfd_cu_err_ != CUDA_SUCCESS) {                                              \
            fprintf(stderr, "CUDA driver error at %s:%d: code %d\n", __FILE__, __LINE__, \
                    static_cast<int>(gfd_cu_err_));                                     \
            return gfd_cu_err_;                                                         \
        }                                                                               \
    } while (0)

constexpr int MAX_CE_CHANNELS = 3;
constexpr int MAX_SG_ENTRIES_PER_BATCH = 8192;

// One (src, dst, size) triple; identical layout to gfd_sg_entry in gfd_b200.h.
struct SGEntry {
    CUdeviceptr dst;   // device destination
    const void* src;   // host source (pinned)
    size_t size;       // bytes
};

static_assert(sizeof(SGEntry) == 24, "SGEntry is 24 bytes");

class CopyEngineManager {
public:
    CopyEngineManager();
    ~CopyEngineManager();
    CopyEngineManager(const CopyEngineManager&) = delete;
    CopyEngineManager& operator=(const CopyEngineManager&) = delete;

    // Creates the channel streams on the device of `ctx` (or the current device when
    // ctx is null).  num_channels 0 means MAX_CE_CHANNELS.
    CUresult init(CUcontext ctx, int num_channels = 0);
    void shutdown();

    // Kept for source compatibility; the runtime API keeps the context current.
    CUresult pin_context();
    void unpin_context();

    // Enqueues the copies (asynchronous): one per merged run or strided group of runs.
    CUresult submit_scatter_gather(const SGEntry* entries, int count);
    // Blocks until every channel used since the last wait has drained.
    CUresult wait_completion();
    CUresult submit_and_wait(const SGEntry* entries, int count);
    CUresult record_event_on_last_stream(CUevent event);
    // `stream` waits (on the GPU) for all channels used since the last wait.
    CUresult make_stream_wait_on_all(CUstream stream);

    uint64_t get_total_submissions() const { return total_submissions_; }
    uint64_t get_total_entries() const { return total_entries_; }
    double get_total_bytes() const { return total_bytes_; }
    bool is_initialized() const { return initialized_; }

private:
    int device_ = -1;
    CUstream streams_[MAX_CE_CHANNELS] = {};
    CUevent events_[MAX_CE_CHANNELS] = {};
    int channels_ = MAX_CE_CHANNELS;
    int next_ = 0;
    uint32_t dirty_ = 0;
    bool initialized_ = false;
    uint64_t total_submissions_ = 0;
    uint64_t total_entries_ = 0;
    double total_bytes_ = 0;
};

}  // namespace gfd
