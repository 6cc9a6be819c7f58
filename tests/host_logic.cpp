// CPU test harness for the host-side table logic of libgfd_b200 (gfd_b200/csrc/table.h):
// C entry points over TableBuilder and partition_ctas, built with g++ by
// tests/test_host_logic.py.  No CUDA involved.
#include <cstdint>
#include <vector>

#include "table.h"

extern "C" {

// Builds the table of n entries (src, dst, size arrays).  rows: room for n rows;
// misc: room for n rows.  Returns the aligned stream bytes; *n_rows / *n_misc get the
// counts.
uint64_t gfdt_build(const uint64_t* src, const uint64_t* dst, const uint64_t* size, int n, gfdb::PullRow* rows,
                    uint32_t* n_rows, gfdb::PullRow* misc, uint32_t* n_misc) {
    std::vector<gfdb::PullRow> m;
    gfdb::TableBuilder tb(rows, &m);
    for (int i = 0; i < n; ++i) tb.add(src[i], dst[i], size[i]);
    *n_rows = tb.n_rows();
    *n_misc = static_cast<uint32_t>(m.size());
    for (size_t i = 0; i < m.size(); ++i) misc[i] = m[i];
    return tb.total();
}

// Same, then removes rows of at least `threshold` bytes (the copy-engine split).
uint64_t gfdt_build_split(const uint64_t* src, const uint64_t* dst, const uint64_t* size, int n, uint64_t threshold,
                          gfdb::PullRow* rows, uint32_t* n_rows, gfdb::PullRow* misc, uint32_t* n_misc,
                          gfdb::PullRow* taken, uint32_t* n_taken) {
    std::vector<gfdb::PullRow> m;
    gfdb::TableBuilder tb(rows, &m);
    for (int i = 0; i < n; ++i) tb.add(src[i], dst[i], size[i]);
    uint32_t k = 0;
    tb.remove_rows([&](const gfdb::PullRow& r) {
        if (r.len < threshold) return false;
        taken[k++] = r;
        return true;
    });
    *n_taken = k;
    *n_rows = tb.n_rows();
    *n_misc = static_cast<uint32_t>(m.size());
    for (size_t i = 0; i < m.size(); ++i) misc[i] = m[i];
    return tb.total();
}

// Groups (src, dst, len) runs into copy-engine copies; returns the number written to out.
size_t gfdt_group(const gfdb::PullRow* runs, size_t n, gfdb::CeCopy* out) {
    std::vector<gfdb::CeCopy> v;
    gfdb::group_strided(runs, n, &v);
    for (size_t i = 0; i < v.size(); ++i) out[i] = v[i];
    return v.size();
}

void gfdt_partition(const gfdb::PullRow* rows, uint32_t n_rows, uint64_t per, int grid, uint32_t* first) {
    gfdb::partition_ctas(rows, n_rows, per, grid, first);
}

}  // extern "C"
