// CPU test harness for host-side helpers with no GPU in the loop, as C entry points
// built with g++ by tests/test_topology.py:
//   * cpulist parsing and topology discovery over a sysfs tree (include/gfd/pcie_topology.h,
//     discover_topology_in), with the exclusive-core split the multi-GPU programs use;
//   * sg_compat::linear_to_sg_entries (include/gfd/sg_task_queue.h);
//   * NUMA-bound pool memory (gfd_b200/csrc/numa_pool.h): bind, first touch, page placement.
// cuda_runtime.h is only included (pcie_topology.h's live discover_topology calls
// cudaDeviceGetPCIBusId); nothing here calls the CUDA runtime, so nothing links it.
#include <cstdint>
#include <string>
#include <vector>

#include "gfd/pcie_topology.h"
#include "gfd/sg_task_queue.h"
#include "numa_pool.h"

extern "C" {

// Parses a cpulist; writes up to cap [lo, hi] pairs, returns the number of ranges.
int probe_parse_list(const char* s, int* out, int cap) {
    auto v = gfd::topo_detail::parse_list(s);
    for (int i = 0; i < static_cast<int>(v.size()) && i < cap; ++i) {
        out[2 * i] = v[i].first;
        out[2 * i + 1] = v[i].second;
    }
    return static_cast<int>(v.size());
}

// Topology of n GPUs from the tree at `root`; bus_ids: n NUL-separated ids (an empty id:
// unknown).  Per GPU g, out[8 g ..] = numa_node, cpu_start, cpu_end, ht_offset,
// num_physical_cores, exclusive base, exclusive count, pcie_bus.  head[0..3] =
// total_numa_nodes, cpus_per_numa, physical_cores_per_numa, gpus on node 0.
void probe_topology(const char* root, const char* bus_ids, int n, int* head, int* out) {
    std::vector<std::string> ids;
    const char* p = bus_ids;
    for (int g = 0; g < n; ++g) {
        ids.emplace_back(p);
        p += ids.back().size() + 1;
    }
    const gfd::TopologyConfig t = gfd::discover_topology_in(root, ids);
    head[0] = t.total_numa_nodes;
    head[1] = t.cpus_per_numa;
    head[2] = t.physical_cores_per_numa;
    head[3] = t.gpus_per_numa.empty() ? 0 : t.gpus_per_numa[0];
    for (int g = 0; g < n; ++g) {
        const gfd::GpuTopology& gt = t.gpus[g];
        int base = 0, count = 0, stride = 0;
        t.get_exclusive_cores(g, base, count, stride);
        int* o = out + 8 * g;
        o[0] = gt.numa_node;
        o[1] = gt.cpu_start;
        o[2] = gt.cpu_end;
        o[3] = gt.ht_offset;
        o[4] = gt.num_physical_cores;
        o[5] = base;
        o[6] = count;
        o[7] = gt.pcie_bus;
    }
}

// linear_to_sg_entries into `out` (count DeviceSGEntry records of 24 bytes).
void probe_linear_to_sg(void* out, uint64_t cpu_base, uint64_t gpu_base, uint32_t token_size, uint32_t start_idx,
                        uint32_t count, uint32_t tag) {
    gfd::sg_compat::linear_to_sg_entries(static_cast<gfd::DeviceSGEntry*>(out), reinterpret_cast<const void*>(cpu_base),
                                         reinterpret_cast<void*>(gpu_base), token_size, start_idx, count, tag);
}

// Maps `bytes` bound to `node` (-1: unbound); returns 0 and the mapping, or -1 and errno.
int probe_map_pool(uint64_t bytes, int node, void** ptr, uint64_t* len, int* bound, int* err) {
    gfdb::MappedPool m;
    const int rc = gfdb::map_numa_pool(bytes, node, &m);
    *ptr = m.ptr;
    *len = m.len;
    *bound = m.node;
    *err = m.err;
    return rc;
}

int probe_page_node(const void* p) { return gfdb::page_numa_node(p); }

void probe_unmap_pool(void* p, uint64_t len) { gfdb::unmap_numa_pool(p, len); }

}  // extern "C"
