#pragma once
// Host memory for source pools: an anonymous mapping rounded to 2 MiB, advised for
// transparent huge pages, bound to one NUMA node and touched once so every page is
// placed there before the GPU driver pins it.  Plain C++ (no CUDA) so the CPU tests
// compile it on its own (tests/topology_probe.cpp).  Replaces the reference's NUMA
// placement of pinned pools: set_mempolicy(MPOL_BIND) around cudaMallocHost
// (examples/05_multi_gpu_benchmark.cu:217-231) and the staging pool's mbind
// (include/gfd/staging_pool.h:29-189).

#include <sys/mman.h>
#include <sys/syscall.h>
#include <unistd.h>

#include <cerrno>
#include <cstddef>
#include <cstdint>

namespace gfdb {

constexpr size_t kPoolHugePage = 2ull << 20;
constexpr int kMpolBind = 2;            // MPOL_BIND
constexpr unsigned kMpolFNode = 1u;     // MPOL_F_NODE
constexpr unsigned kMpolFAddr = 2u;     // MPOL_F_ADDR
constexpr int kMaxPoolNode = 63;        // one 64-bit node mask

struct MappedPool {
    void* ptr = nullptr;
    size_t len = 0;   // mapping length (bytes rounded up to 2 MiB)
    int node = -1;    // node the pages are bound to, -1: not bound
    int err = 0;      // errno of a failed mmap or mbind
};

// node >= 0: bind to that node; a node the host does not have fails the bind and the
// mapping is released (out->err = errno).  node < 0: no binding (first-touch policy).
// Returns 0 on success, -1 on failure.
inline int map_numa_pool(size_t bytes, int node, MappedPool* out) {
    *out = MappedPool();
    if (bytes == 0) return -1;
    const size_t len = (bytes + kPoolHugePage - 1) / kPoolHugePage * kPoolHugePage;
    void* p = mmap(nullptr, len, PROT_READ | PROT_WRITE, MAP_PRIVATE | MAP_ANONYMOUS, -1, 0);
    if (p == MAP_FAILED) {
        out->err = errno;
        return -1;
    }
    madvise(p, len, MADV_HUGEPAGE);
    if (node >= 0) {
        if (node > kMaxPoolNode) {
            munmap(p, len);
            out->err = EINVAL;
            return -1;
        }
        const unsigned long mask = 1ul << node;
        if (syscall(SYS_mbind, p, len, kMpolBind, &mask, static_cast<unsigned long>(kMaxPoolNode + 2), 0u) != 0) {
            out->err = errno;
            munmap(p, len);
            return -1;
        }
    }
    // first touch: every page is placed now (on the bound node), not on the GPU's first read
    for (size_t off = 0; off < len; off += 4096) static_cast<volatile char*>(p)[off] = 0;
    out->ptr = p;
    out->len = len;
    out->node = node;
    return 0;
}

inline void unmap_numa_pool(void* p, size_t len) {
    if (p != nullptr) munmap(p, len);
}

// NUMA node holding the page at p (the page must be present), or -1.
inline int page_numa_node(const void* p) {
    int node = -1;
    if (syscall(SYS_get_mempolicy, &node, nullptr, 0ul, const_cast<void*>(p), kMpolFNode | kMpolFAddr) != 0)
        return -1;
    return node;
}

}  // namespace gfdb
