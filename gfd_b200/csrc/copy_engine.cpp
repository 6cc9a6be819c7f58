// gfd::CopyEngineManager (include/gfd/copy_engine.h): copies over up to three
// high-priority streams -- entries that continue each other merged into one copy, runs
// that advance by constant pitches issued as one 2D copy, the rest one cudaMemcpyAsync
// each.  Copies are split into contiguous per-stream ranges (a few go one per stream),
// each used stream records an event, and wait_completion blocks on the events of every
// stream used since the last wait -- the channel semantics of the reference
// src/copy_engine.cpp:13-218, written on the runtime API (streams and events are the
// same objects).

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <vector>

#include "gfd/copy_engine.h"
#include "gfd/log.h"
#include "table.h"

namespace gfd {
namespace {
CUresult to_cu(cudaError_t e) {
    if (e == cudaSuccess) return CUDA_SUCCESS;
    GFD_LOG_ERROR("copy engine: %s\n", cudaGetErrorString(e));
    return CUDA_ERROR_UNKNOWN;
}
}  // namespace

CopyEngineManager::CopyEngineManager() = default;
CopyEngineManager::~CopyEngineManager() { shutdown(); }

CUresult CopyEngineManager::init(CUcontext ctx, int num_channels) {
    (void)ctx;  // the runtime API uses the context current on this thread
    if (initialized_) return CUDA_SUCCESS;
    if (num_channels > 0 && num_channels <= MAX_CE_CHANNELS) channels_ = num_channels;
    if (cudaGetDevice(&device_) != cudaSuccess) return CUDA_ERROR_INVALID_CONTEXT;
    int lo = 0, hi = 0;
    cudaDeviceGetStreamPriorityRange(&lo, &hi);
    for (int i = 0; i < channels_; ++i) {
        cudaStream_t s;
        cudaEvent_t ev;
        cudaError_t e = cudaStreamCreateWithPriority(&s, cudaStreamNonBlocking, hi);
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ev, cudaEventDisableTiming);
        if (e != cudaSuccess) {
            shutdown();
            return to_cu(e);
        }
        streams_[i] = s;
        events_[i] = ev;
    }
    initialized_ = true;
    return CUDA_SUCCESS;
}

void CopyEngineManager::shutdown() {
    for (int i = 0; i < MAX_CE_CHANNELS; ++i) {
        if (streams_[i]) {
            cudaStreamSynchronize(streams_[i]);
            cudaStreamDestroy(streams_[i]);
            streams_[i] = nullptr;
        }
        if (events_[i]) {
            cudaEventDestroy(events_[i]);
            events_[i] = nullptr;
        }
    }
    initialized_ = false;
    dirty_ = 0;
}

CUresult CopyEngineManager::pin_context() { return initialized_ ? CUDA_SUCCESS : CUDA_ERROR_NOT_INITIALIZED; }
void CopyEngineManager::unpin_context() {}

CUresult CopyEngineManager::submit_scatter_gather(const SGEntry* entries, int count) {
    if (!initialized_ || count <= 0) return CUDA_SUCCESS;
    // entries that continue each other become one run; runs that advance by constant
    // pitches become one 2D copy (the same bytes land as with one copy per entry)
    std::vector<gfdb::PullRow> runs;
    runs.reserve(static_cast<size_t>(count));
    for (int i = 0; i < count; ++i) {
        total_bytes_ += static_cast<double>(entries[i].size);
        gfdb::append_run(&runs, reinterpret_cast<uint64_t>(entries[i].src), entries[i].dst, entries[i].size);
    }
    std::vector<gfdb::CeCopy> copies;
    gfdb::group_strided(runs.data(), runs.size(), &copies);
    const int nc = static_cast<int>(copies.size());
    auto issue = [&](int ch, const gfdb::CeCopy& c) -> cudaError_t {
        if (c.height == 1)
            return cudaMemcpyAsync(reinterpret_cast<void*>(c.dst), reinterpret_cast<const void*>(c.src), c.width,
                                   cudaMemcpyHostToDevice, streams_[ch]);
        return cudaMemcpy2DAsync(reinterpret_cast<void*>(c.dst), c.dpitch, reinterpret_cast<const void*>(c.src),
                                 c.spitch, c.width, c.height, cudaMemcpyHostToDevice, streams_[ch]);
    };
    uint32_t used = 0;
    if (nc <= channels_) {
        for (int i = 0; i < nc; ++i) {
            const int ch = next_;
            next_ = (next_ + 1) % channels_;
            used |= 1u << ch;
            cudaError_t e = issue(ch, copies[i]);
            if (e != cudaSuccess) return to_cu(e);
        }
    } else {
        const int per = (nc + channels_ - 1) / channels_;
        for (int ch = 0; ch < channels_; ++ch) {
            const int b = ch * per;
            const int end = b + per < nc ? b + per : nc;
            if (b >= nc) break;
            used |= 1u << ch;
            for (int i = b; i < end; ++i) {
                cudaError_t e = issue(ch, copies[i]);
                if (e != cudaSuccess) return to_cu(e);
            }
        }
        next_ = 0;
    }
    dirty_ |= used;
    for (uint32_t m = used; m; m &= m - 1) {
        const int ch = __builtin_ctz(m);
        cudaError_t e = cudaEventRecord(events_[ch], streams_[ch]);
        if (e != cudaSuccess) return to_cu(e);
    }
    ++total_submissions_;
    total_entries_ += static_cast<uint64_t>(count);
    return CUDA_SUCCESS;
}

CUresult CopyEngineManager::wait_completion() {
    if (!initialized_) return CUDA_SUCCESS;
    for (uint32_t m = dirty_; m; m &= m - 1) {
        cudaError_t e = cudaEventSynchronize(events_[__builtin_ctz(m)]);
        if (e != cudaSuccess) return to_cu(e);
    }
    dirty_ = 0;
    return CUDA_SUCCESS;
}

CUresult CopyEngineManager::submit_and_wait(const SGEntry* entries, int count) {
    CUresult r = submit_scatter_gather(entries, count);
    return r == CUDA_SUCCESS ? wait_completion() : r;
}

CUresult CopyEngineManager::record_event_on_last_stream(CUevent event) {
    if (!initialized_) return CUDA_SUCCESS;
    const int last = (next_ + channels_ - 1) % channels_;
    return to_cu(cudaEventRecord(event, streams_[last]));
}

CUresult CopyEngineManager::make_stream_wait_on_all(CUstream stream) {
    if (!initialized_) return CUDA_SUCCESS;
    for (uint32_t m = dirty_; m; m &= m - 1) {
        const int ch = __builtin_ctz(m);
        cudaError_t e = cudaEventRecord(events_[ch], streams_[ch]);
        if (e == cudaSuccess) e = cudaStreamWaitEvent(stream, events_[ch], 0);
        if (e != cudaSuccess) return to_cu(e);
    }
    return CUDA_SUCCESS;
}

}  // namespace gfd
