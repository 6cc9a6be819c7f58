#pragma once
// Host topology discovery: which NUMA node each GPU hangs off and which host cores
// belong to it.  Same types and functions as the reference interface
// include/gfd/pcie_topology.h:20-174 (GpuTopology, TopologyConfig with
// recommended_ce_channels / get_exclusive_cores, discover_topology,
// print_topology).  This version parses /sys cpulists in general form ("0-15",
// "0-31,64-95", "3", ...) instead of assuming one "a-b,c-d" pattern, and maps a GPU
// whose PCI device reports no node (-1, e.g. in a VM) to node 0.  Used to place
// NUMA-local pinned pools and to pin host threads in multi-GPU runs.

#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include "gfd/log.h"

namespace gfd {

struct GpuTopology {
    int gpu_id;
    int numa_node;
    int pcie_bus;
    int cpu_start;
    int cpu_end;
    int ht_offset;
    int num_physical_cores;
};

struct TopologyConfig {
    int num_gpus = 0;
    int total_numa_nodes = 1;
    int cpus_per_numa = 0;
    int physical_cores_per_numa = 0;
    std::vector<GpuTopology> gpus;
    std::vector<int> gpus_per_numa;

    int recommended_ce_channels(int active_gpus_on_same_numa) const {
        return active_gpus_on_same_numa <= 2 ? 3 : (active_gpus_on_same_numa <= 4 ? 2 : 1);
    }

    // Splits the physical cores of a GPU's NUMA node evenly among the GPUs on it.
    void get_exclusive_cores(int gpu_id, int& out_base_cpu, int& out_num_cores,
                             int& out_stride) const {
        const GpuTopology& g = gpus[gpu_id];
        const int share_n = gpus_per_numa[g.numa_node] > 0 ? gpus_per_numa[g.numa_node] : 1;
        const int per = physical_cores_per_numa / share_n > 0 ? physical_cores_per_numa / share_n : 1;
        int rank = 0;
        for (int i = 0; i < gpu_id; ++i) rank += gpus[i].numa_node == g.numa_node;
        out_stride = 1;
        out_base_cpu = g.cpu_start + rank * per;
        out_num_cores = per;
        if (out_base_cpu + out_num_cores - 1 > g.cpu_end) out_num_cores = g.cpu_end - out_base_cpu + 1;
        if (out_num_cores < 1) {
            out_base_cpu = g.cpu_start;
            out_num_cores = 1;
        }
    }
};

namespace topo_detail {

inline std::string read_line(const char* path) {
    std::string s;
    if (FILE* f = fopen(path, "r")) {
        char buf[4096];
        if (fgets(buf, sizeof(buf), f)) s = buf;
        fclose(f);
    }
    while (!s.empty() && (s.back() == '\n' || s.back() == ' ')) s.pop_back();
    return s;
}

// "0-3,8,10-11" -> list of [lo, hi] ranges
inline std::vector<std::pair<int, int>> parse_list(const std::string& s) {
    std::vector<std::pair<int, int>> out;
    size_t i = 0;
    while (i < s.size()) {
        size_t j = s.find(',', i);
        if (j == std::string::npos) j = s.size();
        std::string part = s.substr(i, j - i);
        if (!part.empty()) {
            size_t d = part.find('-');
            int a = atoi(part.c_str());
            int b = d == std::string::npos ? a : atoi(part.c_str() + d + 1);
            out.emplace_back(a, b);
        }
        i = j + 1;
    }
    return out;
}

}  // namespace topo_detail

// Topology from a sysfs tree: `sysfs` is the tree's root ("/sys" on a live system) and
// bus_ids[g] the PCI bus id of GPU g ("0000:1B:00.0"; empty when unknown).  Split from
// discover_topology so the parsing can be checked against a fake tree.
static inline TopologyConfig discover_topology_in(const std::string& sysfs, const std::vector<std::string>& bus_ids) {
    using namespace topo_detail;
    TopologyConfig t;
    const int num_gpus = static_cast<int>(bus_ids.size());
    t.num_gpus = num_gpus;
    t.gpus.resize(num_gpus);
    auto nodes = parse_list(read_line((sysfs + "/devices/system/node/online").c_str()));
    int max_node = 0;
    for (auto& r : nodes) max_node = r.second > max_node ? r.second : max_node;
    t.total_numa_nodes = max_node + 1;

    std::vector<std::vector<std::pair<int, int>>> cpus(t.total_numa_nodes);
    for (int n = 0; n < t.total_numa_nodes; ++n)
        cpus[n] = parse_list(read_line((sysfs + "/devices/system/node/node" + std::to_string(n) + "/cpulist").c_str()));
    auto first_range = [&](int n) -> std::pair<int, int> {
        if (n < (int)cpus.size() && !cpus[n].empty()) return cpus[n][0];
        return {0, 0};
    };
    auto count_cpus = [&](int n) {
        int c = 0;
        if (n < (int)cpus.size())
            for (auto& r : cpus[n]) c += r.second - r.first + 1;
        return c;
    };
    const std::pair<int, int> r0 = first_range(0);
    t.physical_cores_per_numa = r0.second - r0.first + 1;
    t.cpus_per_numa = count_cpus(0) > 0 ? count_cpus(0) : t.physical_cores_per_numa;

    for (int g = 0; g < num_gpus; ++g) {
        GpuTopology& gt = t.gpus[g];
        gt.gpu_id = g;
        gt.pcie_bus = g;
        int node = -1;
        std::string bus = bus_ids[g];
        if (!bus.empty()) {
            for (char& c : bus)
                if (c >= 'A' && c <= 'F') c = static_cast<char>(c - 'A' + 'a');
            std::string v = read_line((sysfs + "/bus/pci/devices/" + bus + "/numa_node").c_str());
            if (!v.empty()) node = atoi(v.c_str());
            unsigned dom = 0, b = 0;
            if (sscanf(bus.c_str(), "%x:%x", &dom, &b) == 2) gt.pcie_bus = static_cast<int>(b);
        }
        if (node < 0 || node >= t.total_numa_nodes) node = 0;
        gt.numa_node = node;
        const std::pair<int, int> r = first_range(node);
        gt.cpu_start = r.first;
        gt.cpu_end = r.second;
        gt.num_physical_cores = r.second - r.first + 1;
        gt.ht_offset = (node < (int)cpus.size() && cpus[node].size() > 1)
                           ? cpus[node][1].first - r.first
                           : 0;
    }
    t.gpus_per_numa.assign(t.total_numa_nodes, 0);
    for (int g = 0; g < num_gpus; ++g) t.gpus_per_numa[t.gpus[g].numa_node]++;
    return t;
}

static inline TopologyConfig discover_topology(int num_gpus) {
    std::vector<std::string> bus_ids(num_gpus > 0 ? num_gpus : 0);
    for (int g = 0; g < num_gpus; ++g) {
        char bus[32] = {0};
        if (cudaDeviceGetPCIBusId(bus, sizeof(bus), g) == cudaSuccess) bus_ids[g] = bus;
        else cudaGetLastError();
    }
    return discover_topology_in("/sys", bus_ids);
}

static inline void print_topology(const TopologyConfig& t) {
    GFD_LOG_INFO("Topology: %d GPUs, %d NUMA nodes, %d physical cores per node\n", t.num_gpus,
                 t.total_numa_nodes, t.physical_cores_per_numa);
    for (int g = 0; g < t.num_gpus; ++g) {
        int base, n, stride;
        t.get_exclusive_cores(g, base, n, stride);
        GFD_LOG_INFO("  GPU %d: NUMA %d, cores %d-%d\n", g, t.gpus[g].numa_node, base, base + n - 1);
    }
}

}  // namespace gfd
