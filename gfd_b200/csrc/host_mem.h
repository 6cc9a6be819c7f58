#pragma once
// Host-memory checks of the direct-submit path that need no GPU.

#include <sys/mman.h>
#include <unistd.h>

#include <cstdint>
#include <vector>

namespace gfdb {

// Every page of [p, p + n) is mapped in this process: mincore fails with ENOMEM when the
// page span has a hole.  Sources that only the copy engine can read (pageable memory,
// GFD_GATHER_PAGEABLE) are checked this way before anything is copied, so an unmapped
// range is rejected instead of faulting the driver's staging copy.  On success *page_lo /
// *page_hi are the checked page span.
inline bool pages_mapped(uint64_t p, uint64_t n, uint64_t* page_lo, uint64_t* page_hi) {
    if (n == 0 || p + n < p) return false;
    static const uint64_t page = static_cast<uint64_t>(sysconf(_SC_PAGESIZE));
    const uint64_t lo = p / page * page;
    if (p + n > ~0ull - page) return false;
    const uint64_t hi = (p + n + page - 1) / page * page;
    std::vector<unsigned char> vec((hi - lo) / page);
    if (mincore(reinterpret_cast<void*>(lo), hi - lo, vec.data()) != 0) return false;
    *page_lo = lo;
    *page_hi = hi;
    return true;
}

}  // namespace gfdb
