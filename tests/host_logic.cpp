// CPU test harness for the host-side logic of libgfd_b200: the pull tables
// (gfd_b200/csrc/table.h: TableBuilder, partition_ctas, append_run, group_strided) and the ring drain
// (gfd_b200/csrc/drain.h: committed_run, BatchGate, DrainAccounting) and the page check of
// pageable sources (gfd_b200/csrc/host_mem.h), as C entry points built with g++ by
// tests/test_host_logic.py.  No CUDA involved.
#include <cstdint>
#include <vector>

#include "drain.h"
#include "host_mem.h"
#include "table.h"

extern "C" {

// gfdb::pages_mapped: 1 when every page of [p, p + n) is mapped, with the page span.
int gfdt_pages_mapped(uint64_t p, uint64_t n, uint64_t* lo, uint64_t* hi) { return gfdb::pages_mapped(p, n, lo, hi); }

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

// The copy-engine plan of CopyEngineManager: continuing entries merged, then grouped.
size_t gfdt_ce_plan(const uint64_t* src, const uint64_t* dst, const uint64_t* size, size_t n, gfdb::CeCopy* out) {
    std::vector<gfdb::PullRow> runs;
    for (size_t i = 0; i < n; ++i) gfdb::append_run(&runs, src[i], dst[i], size[i]);
    std::vector<gfdb::CeCopy> v;
    gfdb::group_strided(runs.data(), runs.size(), &v);
    for (size_t i = 0; i < v.size(); ++i) out[i] = v[i];
    return v.size();
}

uint32_t gfdt_committed_run(const void* queue, uint64_t next, uint32_t max_n, int* urgent) {
    bool u = false;
    const uint32_t n = gfdb::committed_run(static_cast<const gfd::DescriptorQueue*>(queue), next, max_n, &u);
    *urgent = u ? 1 : 0;
    return n;
}

void* gfdt_gate_new(uint64_t quiet_ns) { return new gfdb::BatchGate(quiet_ns); }
int gfdt_gate_ready(void* g, uint32_t n, int urgent, int force, uint64_t now_ns) {
    return static_cast<gfdb::BatchGate*>(g)->ready(n, urgent != 0, force != 0, now_ns) ? 1 : 0;
}
void gfdt_gate_free(void* g) { delete static_cast<gfdb::BatchGate*>(g); }

// Accounts n descriptors (flags, user_data); outputs as DrainAccounting leaves them.
void gfdt_account(int tiled, int sg, const uint32_t* flags, const uint64_t* user, int n, uint16_t* tile_id,
                  uint32_t* tile_count, uint32_t* n_tiles, uint16_t* list_id, uint32_t max_lists, uint32_t* n_lists,
                  uint32_t* landed) {
    std::vector<uint32_t> counts(gfd::MAX_TILES, 0);
    gfdb::DrainAccounting a(tiled != 0, sg != 0, counts.data(), tile_id, tile_count, list_id, max_lists);
    for (int i = 0; i < n; ++i) a.add(flags[i], user[i]);
    a.finish();
    *n_tiles = a.n_tiles();
    *n_lists = a.n_lists();
    *landed = a.lists_landed();
    for (uint32_t c : counts)
        if (c != 0) *n_tiles = 0xffffffffu;  // scratch must come back zeroed
}

void gfdt_partition(const gfdb::PullRow* rows, uint32_t n_rows, uint64_t per, int grid, uint32_t* first) {
    gfdb::partition_ctas(rows, n_rows, per, grid, first);
}

}  // extern "C"
