// SGWarpSpecSession + GFD_SG_WARP_SPEC_KERNEL: host-submitted lists (reference
// test/test_sg_e2e.cu pattern), many lists beyond the entry pool (backpressure while
// the kernel consumes), scattered sources and destinations, and GPU-submitted lists
// from a submitter warp in the same CTA (reference test/test_sg_gpu_submit.cu
// pattern, 4 lists x 8 x 4 KiB).
#include <gfd/gfd.h>
#include <gfd/sg_warp_spec.cuh>

#include <algorithm>
#include <cmath>
#include <thread>

#include "common.h"

// per list: count entries and sum the first float of each landed entry
struct ListCheck {
    unsigned long long* seen;  // [MAX_SG_LISTS]
    float* first_sum;          // [MAX_SG_LISTS]
    __device__ void operator()(gfd::sg_warp_spec::SGListView v) {
        float s = 0.f;
        for (uint32_t i = v.lane_id; i < v.count; i += 32) s += *v.dst_ptr<float>(i);
        for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        if (v.lane_id == 0) {
            atomicAdd(&seen[v.list_id], (unsigned long long)v.count);
            atomicAdd(&first_sum[v.list_id], s);
        }
    }
};

GFD_SG_WARP_SPEC_KERNEL(sg_kernel, ListCheck);

// framework warps + one submitter warp in the same CTA
__global__ void sg_gpu_submit_kernel(gfd::DescriptorQueue* dq, gfd::SGTaskQueue* sq, ListCheck fn, const char* cpu,
                                     char* gpu, int per_list, int lists, uint32_t entry_size, uint32_t framework_warps) {
    const uint32_t warp = threadIdx.x >> 5;
    if (warp < framework_warps) {
        gfd::sg_warp_spec::_sg_transfer_warp_loop(dq, sq, fn, framework_warps);
        return;
    }
    for (int l = 0; l < lists; ++l) {
        gfd::sg::sg_wait_entry_space(sq, per_list);
        const uint64_t off = gfd::sg::sg_alloc_entries(sq, per_list);
        for (int i = threadIdx.x & 31; i < per_list; i += 32) {
            const uint64_t g = (uint64_t)l * per_list + i;
            sq->entries[(off + i) % gfd::MAX_SG_POOL_ENTRIES] =
                gfd::DeviceSGEntry{(uint64_t)cpu + g * entry_size, (uint64_t)gpu + g * entry_size, entry_size, (uint32_t)l};
        }
        __syncwarp();
        gfd::sg::sg_wait_list_space(sq);
        const uint64_t slot = gfd::sg::sg_alloc_list(sq);
        gfd::sg::sg_commit_list(sq, slot, (uint32_t)off, per_list, l, gfd::SG_FLAG_NONE);
    }
    gfd::sg::sg_wait_list_done(sq, lists);
    if ((threadIdx.x & 31) == 0) {
        __threadfence_system();
        sq->terminate = 1;
        __threadfence_system();
    }
}

// Device-entry lists (SG_FLAG_DEVICE_ENTRIES): the submitter warp of CTA 0 writes each
// list's entries into the session's device pool and commits it in device memory
// (SGSubmitter::write_header_device / publish_device); every CTA's framework warps pull
// them, and ListCheck reads the entries back through SGListView (device pool).
__global__ void sg_device_entries_kernel(gfd::DescriptorQueue* dq, gfd::SGTaskQueue* sq, ListCheck fn,
                                         const char* cpu, char* gpu, const uint32_t* perm, int per_list, int lists,
                                         uint32_t entry_size, uint32_t framework_warps) {
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (warp < framework_warps) {
        gfd::sg_warp_spec::_sg_transfer_warp_loop(dq, sq, fn, framework_warps);
        return;
    }
    if (blockIdx.x != 0 || warp != framework_warps) return;
    const gfd::sg::SGSubmitter sub(sq);
    gfd::DeviceSGEntry* pool = sub.device_pool();
    int l = 0;
    for (; pool != nullptr && l < lists; ++l) {
        if (!sub.wait_entry_space(per_list) || !sub.wait_list_space(1)) break;
        const uint64_t po = sub.alloc_entries(per_list);
        const uint64_t ls = sub.alloc_list(1);
        for (int i = lane; i < per_list; i += 32) {
            const uint64_t g = (uint64_t)l * per_list + i;
            pool[(po + i) % gfd::MAX_SG_POOL_ENTRIES] = gfd::DeviceSGEntry{
                (uint64_t)cpu + (uint64_t)perm[g] * entry_size, (uint64_t)gpu + g * entry_size, entry_size, (uint32_t)l};
        }
        sub.write_header_device(ls, po, per_list, l, gfd::SG_FLAG_NONE);
        sub.publish_device(ls, 1);
    }
    gfd::sg::sg_wait_list_done(sq, l);
    if (lane == 0) {
        __threadfence_system();
        sq->terminate = 1;
        if (sq->poll_mirror != nullptr) sq->poll_mirror->terminate = 1u;
        __threadfence_system();
    }
}

struct Fixture {
    unsigned long long* seen;
    float* sums;
    Fixture() {
        CK(cudaMalloc(&seen, gfd::MAX_SG_LISTS * 8));
        CK(cudaMalloc(&sums, gfd::MAX_SG_LISTS * 4));
        CK(cudaMemset(seen, 0, gfd::MAX_SG_LISTS * 8));
        CK(cudaMemset(sums, 0, gfd::MAX_SG_LISTS * 4));
    }
    ~Fixture() {
        cudaFree(seen);
        cudaFree(sums);
    }
    std::vector<unsigned long long> counts() {
        std::vector<unsigned long long> h(gfd::MAX_SG_LISTS);
        CK(cudaMemcpy(h.data(), seen, h.size() * 8, cudaMemcpyDeviceToHost));
        return h;
    }
};

static void e2e_small() {
    // test_sg_e2e: 4 x 4 KiB, float i+1, one block, list submitted before launch
    const int N = 4;
    const size_t T = 4096, total = N * T;
    float* cpu;
    CK(cudaMallocHost(&cpu, total));
    for (size_t i = 0; i < total / 4; ++i) cpu[i] = (float)(i + 1);
    float* gpu;
    CK(cudaMalloc(&gpu, total));
    CK(cudaMemset(gpu, 0, total));
    Fixture fx;
    gfd::SGWarpSpecConfig cfg;
    cfg.num_compute_warps = 1;
    cfg.num_blocks = 1;
    gfd::SGWarpSpecSession s(cfg);
    std::vector<gfd::DeviceSGEntry> e(N);
    for (int i = 0; i < N; ++i) e[i] = {(uint64_t)((char*)cpu + i * T), (uint64_t)((char*)gpu + i * T), (uint32_t)T, 0};
    const uint64_t slot = s.submit_sg_list(e.data(), N, 0, gfd::SG_FLAG_HOST_SUBMITTED);
    s.launch(sg_kernel, ListCheck{fx.seen, fx.sums});
    s.synchronize();
    auto st = s.get_stats();
    const bool data = device_equals(gpu, cpu, total);
    const unsigned long long seen = fx.counts()[0];
    bool ok = slot == 0 && data && seen == N && s.timeouts() == 0 && st.descriptors_processed == N &&
              st.bytes_transferred == total;
    char detail[200];
    snprintf(detail, sizeof(detail), "slot=%llu data=%d seen=%llu timeouts=%llu site=%u desc=%llu bytes=%llu completed=%llu",
             (unsigned long long)slot, (int)data, seen, (unsigned long long)s.timeouts(),
             (unsigned)s.get_sg_queue()->timeout_site, (unsigned long long)st.descriptors_processed,
             (unsigned long long)st.bytes_transferred,
             (unsigned long long)s.get_sg_queue()->lists_completed);
    report("sg_e2e_4x4KiB", ok, detail);
    CK(cudaFree(gpu));
    CK(cudaFreeHost(cpu));
}

static void many_lists_backpressure(int blocks, int compute_warps) {
    // 48 lists x 1024 scattered entries (49152 > 16384-entry pool), submitted while running
    const int L = 48, E = 1024;
    const uint32_t T = 2048;
    const size_t pool_tokens = (size_t)L * E * 2;
    char* cpu;
    CK(cudaMallocHost(&cpu, pool_tokens * T));
    fill_pattern(cpu, pool_tokens * T, 41);
    char* gpu;
    CK(cudaMalloc(&gpu, (size_t)L * E * T));
    CK(cudaMemset(gpu, 0, (size_t)L * E * T));
    Fixture fx;
    gfd::SGWarpSpecConfig cfg;
    cfg.num_compute_warps = compute_warps;
    cfg.num_blocks = blocks;
    gfd::SGWarpSpecSession s(cfg);
    // random permutation of source tokens, destinations reversed within each list
    std::vector<uint32_t> perm(pool_tokens);
    for (size_t i = 0; i < pool_tokens; ++i) perm[i] = (uint32_t)i;
    uint64_t x = 7;
    for (size_t i = pool_tokens - 1; i > 0; --i) {
        x = x * 6364136223846793005ull + 1442695040888963407ull;
        std::swap(perm[i], perm[(x >> 33) % (i + 1)]);
    }
    s.launch(sg_kernel, ListCheck{fx.seen, fx.sums});
    bool submitted = true;
    std::vector<gfd::DeviceSGEntry> e(E);
    for (int l = 0; l < L; ++l) {
        for (int i = 0; i < E; ++i) {
            const size_t g = (size_t)l * E + i;
            const size_t d = (size_t)l * E + (E - 1 - i);
            e[i] = {(uint64_t)(cpu + (size_t)perm[g] * T), (uint64_t)(gpu + d * T), T, (uint32_t)l};
        }
        submitted = submitted && s.submit_sg_list(e.data(), E, l) != UINT64_MAX;
    }
    s.synchronize();
    bool ok = submitted && s.timeouts() == 0;
    std::vector<char> got((size_t)L * E * T);
    CK(cudaMemcpy(got.data(), gpu, got.size(), cudaMemcpyDeviceToHost));
    for (int l = 0; ok && l < L; ++l)
        for (int i = 0; ok && i < E; ++i) {
            const size_t g = (size_t)l * E + i, d = (size_t)l * E + (E - 1 - i);
            ok = memcmp(got.data() + d * T, cpu + (size_t)perm[g] * T, T) == 0;
        }
    auto c = fx.counts();
    for (int l = 0; ok && l < L; ++l) ok = c[l] == (unsigned long long)E;
    char name[64], detail[160];
    snprintf(name, sizeof(name), "sg_48_lists_x1024_blocks%d_cw%d", blocks, compute_warps);
    snprintf(detail, sizeof(detail), "submitted=%d timeouts=%llu completed=%llu released=%llu consumed=%llu",
             (int)submitted, (unsigned long long)s.timeouts(), (unsigned long long)s.get_sg_queue()->lists_completed,
             (unsigned long long)s.get_sg_queue()->lists_released,
             (unsigned long long)s.get_sg_queue()->entry_consumed_idx);
    report(name, ok, detail);
    CK(cudaFree(gpu));
    CK(cudaFreeHost(cpu));
}

static void gpu_submitted() {
    const int per_list = 8, lists = 4;
    const uint32_t T = 4096;
    const size_t total = (size_t)per_list * lists * T;
    float* cpu;
    CK(cudaMallocHost(&cpu, total));
    for (size_t i = 0; i < total / 4; ++i) cpu[i] = (float)(i + 1);
    char* gpu;
    CK(cudaMalloc(&gpu, total));
    CK(cudaMemset(gpu, 0, total));
    Fixture fx;
    gfd::SGWarpSpecConfig cfg;
    cfg.num_compute_warps = 1;
    cfg.num_blocks = 1;
    cfg.producer_warps = 1;
    gfd::SGWarpSpecSession s(cfg);
    gfd::SGTaskQueue* sq = s.get_sg_queue();
    sq->producer_warps = 1;
    sq->wait_limit_ns = 20000000000ull;
    sg_gpu_submit_kernel<<<1, 96>>>(s.get_desc_queue(), sq, ListCheck{fx.seen, fx.sums}, (const char*)cpu, gpu,
                                    per_list, lists, T, 2);
    CK(cudaDeviceSynchronize());
    auto c = fx.counts();
    const bool data = device_equals(gpu, cpu, total);
    bool ok = data && sq->wait_timeouts == 0 && sq->lists_completed == (uint64_t)lists;
    for (int l = 0; ok && l < lists; ++l) ok = c[l] == (unsigned long long)per_list;
    char detail[160];
    snprintf(detail, sizeof(detail), "data=%d timeouts=%u completed=%llu seen0=%llu", (int)data,
             (unsigned)sq->wait_timeouts, (unsigned long long)sq->lists_completed, c[0]);
    report("sg_gpu_submitted_4x8x4KiB", ok, detail);
    CK(cudaFree(gpu));
    CK(cudaFreeHost(cpu));
}

static void gpu_submitted_device_entries(int blocks) {
    // 48 lists x 1024 scattered 2 KiB entries (the pool wraps three times)
    const int L = 48, E = 1024;
    const uint32_t T = 2048;
    const size_t pool_tokens = (size_t)L * E * 2;
    float* cpu;
    CK(cudaMallocHost(&cpu, pool_tokens * T));
    for (size_t i = 0; i < pool_tokens * T / 4; ++i) cpu[i] = (float)(i % 1000003) * 0.25f;
    char* gpu;
    CK(cudaMalloc(&gpu, (size_t)L * E * T));
    CK(cudaMemset(gpu, 0, (size_t)L * E * T));
    std::vector<uint32_t> perm(pool_tokens);
    for (size_t i = 0; i < pool_tokens; ++i) perm[i] = (uint32_t)i;
    uint64_t x = 11;
    for (size_t i = pool_tokens - 1; i > 0; --i) {
        x = x * 6364136223846793005ull + 1442695040888963407ull;
        std::swap(perm[i], perm[(x >> 33) % (i + 1)]);
    }
    uint32_t* d_perm;
    CK(cudaMalloc(&d_perm, (size_t)L * E * 4));
    CK(cudaMemcpy(d_perm, perm.data(), (size_t)L * E * 4, cudaMemcpyHostToDevice));
    Fixture fx;
    gfd::SGWarpSpecConfig cfg;
    cfg.num_compute_warps = 1;
    cfg.num_blocks = blocks;
    gfd::SGWarpSpecSession s(cfg);
    auto lp = s.get_launch_params();
    gfd::SGTaskQueue* sq = lp.sq;
    const bool mirrored = sq->poll_mirror != nullptr;
    const uint32_t fw = lp.block.x / 32;
    sg_device_entries_kernel<<<lp.grid, (fw + 1) * 32>>>(lp.dq, sq, ListCheck{fx.seen, fx.sums}, (const char*)cpu, gpu,
                                                         d_perm, E, L, T, fw);
    s.get_poller()->start();
    CK(cudaDeviceSynchronize());
    s.synchronize();
    bool ok = mirrored && s.timeouts() == 0 && sq->lists_completed == (uint64_t)L;
    std::vector<char> got((size_t)L * E * T);
    CK(cudaMemcpy(got.data(), gpu, got.size(), cudaMemcpyDeviceToHost));
    for (size_t g = 0; ok && g < (size_t)L * E; ++g)
        ok = memcmp(got.data() + g * T, (const char*)cpu + (size_t)perm[g] * T, T) == 0;
    auto c = fx.counts();
    std::vector<float> sums(gfd::MAX_SG_LISTS);
    CK(cudaMemcpy(sums.data(), fx.sums, sums.size() * 4, cudaMemcpyDeviceToHost));
    for (int l = 0; ok && l < L; ++l) {
        double want = 0.0;
        for (int i = 0; i < E; ++i) want += cpu[(size_t)perm[(size_t)l * E + i] * T / 4];
        ok = c[l] == (unsigned long long)E && std::fabs(sums[l] - want) <= 1e-4 * std::fabs(want) + 1.0;
    }
    bool markers_clear = true;
    for (int i = 0; i < gfd::MAX_SG_LISTS; ++i) markers_clear = markers_clear && sq->lists[i].sequence == 0;
    ok = ok && markers_clear;
    char name[64], detail[200];
    snprintf(name, sizeof(name), "sg_device_entries_48x1024_blocks%d", blocks);
    snprintf(detail, sizeof(detail), "mirror=%d timeouts=%llu completed=%llu released=%llu consumed=%llu markers_clear=%d",
             (int)mirrored, (unsigned long long)s.timeouts(), (unsigned long long)sq->lists_completed,
             (unsigned long long)sq->lists_released, (unsigned long long)sq->entry_consumed_idx, (int)markers_clear);
    report(name, ok, detail);
    CK(cudaFree(d_perm));
    CK(cudaFree(gpu));
    CK(cudaFreeHost(cpu));
}

static void invalid_entries_rejected() {
    gfd::SGWarpSpecConfig cfg;
    cfg.num_blocks = 1;
    gfd::SGWarpSpecSession s(cfg);
    std::vector<char> pageable(4096);
    char* gpu;
    CK(cudaMalloc(&gpu, 4096));
    gfd::DeviceSGEntry e{(uint64_t)pageable.data(), (uint64_t)gpu, 4096, 0};
    const bool rejected = s.submit_sg_list(&e, 1, 0) == UINT64_MAX;
    report("sg_rejects_pageable_source", rejected);
    CK(cudaFree(gpu));
}

int main() {
    e2e_small();
    many_lists_backpressure(1, 1);
    many_lists_backpressure(8, 2);
    many_lists_backpressure(0, 4);
    gpu_submitted();
    gpu_submitted_device_entries(1);
    gpu_submitted_device_entries(0);
    invalid_entries_rejected();
    return g_failures ? 1 : 0;
}
