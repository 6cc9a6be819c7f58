#pragma once
// StagingPool: source-compatible shim for the reference's hugepage staging pool
// (include/gfd/staging_pool.h:29-189).
//
// The reference gathers scattered tokens on CPU cores into pinned staging buffers
// before a DMA.  Here the GPU reads the tokens in place, so no staging memory is
// needed: init() allocates nothing and records the requested geometry, and
// acquire_buffers() reports that no set is available (callers fall through to the
// direct path).  The interface is kept so existing programs compile and link.

#include <cstddef>
#include <mutex>

namespace gfd {

class StagingPool {
public:
    static constexpr int MAX_BUFFER_SETS = 8;
    static constexpr int BUFS_PER_SET = 5;
    static constexpr size_t MAX_BUF_SIZE = 128ull * 1024 * 1024;

    static StagingPool& instance() {
        static StagingPool pool;
        return pool;
    }

    bool init(int num_gpus, size_t buf_size, int numa_node = 0) {
        std::lock_guard<std::mutex> lk(mu_);
        (void)numa_node;
        num_sets_ = num_gpus > MAX_BUFFER_SETS ? MAX_BUFFER_SETS : num_gpus;
        buf_size_ = buf_size;
        initialized_ = true;
        return true;
    }

    int acquire_buffers(size_t, int = 0) { return -1; }

    void get_buffers(int, char* out_bufs[BUFS_PER_SET], size_t& out_size, bool& out_hugepage) {
        for (int b = 0; b < BUFS_PER_SET; ++b) out_bufs[b] = nullptr;
        out_size = 0;
        out_hugepage = false;
    }

    void release_buffers(int) {}

    bool is_initialized() const { return initialized_; }
    size_t buffer_size() const { return buf_size_; }

    void shutdown() {
        std::lock_guard<std::mutex> lk(mu_);
        initialized_ = false;
    }

private:
    StagingPool() = default;
    StagingPool(const StagingPool&) = delete;
    StagingPool& operator=(const StagingPool&) = delete;

    std::mutex mu_;
    bool initialized_ = false;
    int num_sets_ = 0;
    size_t buf_size_ = 0;
};

}  // namespace gfd
