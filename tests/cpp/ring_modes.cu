// Ring consumer per-tile and per-list accounting (reference batch_processor.cpp
// process_batch_tiled / process_batch_sg semantics), driven by hand-written kernels
// that use the device API and bounded waits:
//  tiled: one CTA per tile; warp 0 submits each chunk's descriptors (submit_chunk) and
//         waits until d_tile_chunk_done[tile] reaches the chunk's cumulative count,
//         then every thread sums its landed token.
//  sg:    warp 1 commits SG lists (sg_submit_list); warp 0 converts each committed
//         list into descriptors (user_data = list << 32 | i, FLAG_LAST_IN_TILE on the
//         last one) and waits for d_list_done[list] from the drain's completion.
#include <gfd/device_primitives.cuh>
#include <gfd/gfd.h>
#include <gfd/sg_device_primitives.cuh>

#include "common.h"

__global__ void tiled_kernel(gfd::TiledQueue* tq, const float* cpu, float* gpu, float* sums, int dim, int* failed) {
    const uint32_t tile = blockIdx.x;
    const uint32_t T = tq->scheduler.tokens_per_tile, C = tq->scheduler.tokens_per_chunk;
    const uint32_t K = tq->scheduler.chunks_per_tile, ts = tq->scheduler.token_size;
    if (threadIdx.x < 32) {
        for (uint32_t c = 0; c < K; ++c) {
            const uint64_t base = gfd::device::acquire_chunk_slots(tq, C);
            gfd::device::wait_queue_space(tq, C);
            gfd::device::submit_chunk(tq, base, tile, c, C, T, cpu, gpu, ts);
            if (threadIdx.x == 0 && !gfd::device::wait_chunk_done_until(tq, tile, (uint64_t)(c + 1) * C, 5000000000ull))
                atomicAdd(failed, 1);
            __syncwarp();
        }
    }
    __syncthreads();
    for (uint32_t t = threadIdx.x; t < T; t += blockDim.x) {
        const float* v = gpu + ((size_t)tile * T + t) * dim;
        float s = 0.f;
        for (int d = 0; d < dim; ++d) s += v[d];
        sums[tile * T + t] = s;
    }
}

__global__ void sg_ring_kernel(gfd::DescriptorQueue* dq, gfd::SGTaskQueue* sq, const char* cpu, char* gpu,
                               int lists, int per_list, uint32_t esize, int* failed) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (warp == 1) {  // submitter
        for (int l = 0; l < lists; ++l) {
            __shared__ gfd::DeviceSGEntry staged[64];
            for (int i = lane; i < per_list; i += 32) {
                const uint64_t g = (uint64_t)l * per_list + i;
                staged[i] = gfd::DeviceSGEntry{(uint64_t)cpu + g * 2 * esize, (uint64_t)gpu + g * esize, esize, (uint32_t)l};
            }
            __syncwarp();
            gfd::sg::sg_submit_list(sq, staged, per_list, l);
        }
        return;
    }
    if (warp != 0) return;
    for (int l = 0; l < lists; ++l) {
        // claim and wait for the list (bounded)
        unsigned long long idx = 0;
        if (lane == 0) idx = atomicAdd((unsigned long long*)&sq->list_read_idx, 1ull);
        idx = __shfl_sync(0xffffffffu, idx, 0);
        gfd::SGList* L = &sq->lists[idx % gfd::MAX_SG_LISTS];
        int ok = 1;
        if (lane == 0) {
            const uint64_t t0 = gfd::wait::now();
            while (gfd::wait::load_acquire_sys(&L->sequence) != idx + 1)
                if (gfd::wait::expired(t0, 5000000000ull)) { ok = 0; break; }
        }
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) { if (lane == 0) atomicAdd(failed, 1); return; }
        const uint32_t off = L->pool_offset, count = L->count, id = L->list_id;
        unsigned long long base = 0;
        if (lane == 0) base = atomicAdd((unsigned long long*)&dq->write_idx, (unsigned long long)count);
        base = __shfl_sync(0xffffffffu, base, 0);
        for (uint32_t i = lane; i < count; i += 32) {
            const gfd::DeviceSGEntry e = sq->entries[(off + i) % gfd::MAX_SG_POOL_ENTRIES];
            gfd::Descriptor* d = &dq->entries[(base + i) % gfd::QUEUE_SIZE];
            d->src_addr = e.src_addr;
            d->dst_addr = e.dst_addr;
            d->size = e.size;
            d->user_data = ((uint64_t)id << 32) | i;
            d->flags = (i == count - 1) ? gfd::FLAG_LAST_IN_TILE : gfd::FLAG_NONE;
        }
        __threadfence_system();
        __syncwarp();
        for (uint32_t i = lane; i < count; i += 32) dq->entries[(base + i) % gfd::QUEUE_SIZE].sequence = base + i + 1;
        __threadfence_system();
        __syncwarp();
        if (lane == 0) {
            L->sequence = 0;
            atomicMax((unsigned long long*)&sq->entry_consumed_idx, (unsigned long long)((idx + 1) * count));
        }
        gfd::sg::sg_wait_list_id_done(sq, id);
        if (lane == 0 && sq->d_list_done[id] == 0) atomicAdd(failed, 1);
        __syncwarp();
    }
}

static void tiled_case() {
    const int tiles = 24, T = 64, C = 16, dim = 1024;
    const size_t ts = dim * sizeof(float), total = (size_t)tiles * T * ts;
    float* cpu;
    CK(cudaMallocHost(&cpu, total));
    for (int t = 0; t < tiles * T; ++t)
        for (int d = 0; d < dim; ++d) cpu[(size_t)t * dim + d] = (float)(t % 251) + 0.25f;
    float *gpu, *sums;
    int* failed;
    CK(cudaMalloc(&gpu, total));
    CK(cudaMemset(gpu, 0, total));
    CK(cudaMalloc(&sums, tiles * T * sizeof(float)));
    CK(cudaMalloc(&failed, sizeof(int)));
    CK(cudaMemset(failed, 0, sizeof(int)));
    gfd::TiledQueue* tq;
    CK(cudaHostAlloc(&tq, sizeof(gfd::TiledQueue), cudaHostAllocMapped));
    memset(tq, 0, sizeof(*tq));
    tq->scheduler.total_tiles = tiles;
    tq->scheduler.tokens_per_tile = T;
    tq->scheduler.tokens_per_chunk = C;
    tq->scheduler.chunks_per_tile = T / C;
    tq->scheduler.token_size = (uint32_t)ts;
    CK(cudaMalloc(&tq->d_tile_chunk_done, gfd::MAX_TILES * 8));
    CK(cudaMemset(tq->d_tile_chunk_done, 0, gfd::MAX_TILES * 8));
    gfd::CpuPollingThread poller(&tq->base, gpu, cpu, total);
    poller.set_tiled_queue(tq);
    bool ok = poller.init_copy_engine();
    poller.start();
    tiled_kernel<<<tiles, 128>>>(tq, cpu, gpu, sums, dim, failed);
    CK(cudaDeviceSynchronize());
    poller.stop();
    int f = 0;
    CK(cudaMemcpy(&f, failed, sizeof(int), cudaMemcpyDeviceToHost));
    std::vector<float> hs(tiles * T);
    CK(cudaMemcpy(hs.data(), sums, hs.size() * 4, cudaMemcpyDeviceToHost));
    std::vector<uint64_t> done(tiles);
    CK(cudaMemcpy(done.data(), tq->d_tile_chunk_done, tiles * 8, cudaMemcpyDeviceToHost));
    ok = ok && f == 0 && tq->base.wait_timeouts == 0 && device_equals(gpu, cpu, total);
    for (int t = 0; ok && t < tiles * T; ++t) ok = hs[t] == ((float)(t % 251) + 0.25f) * dim;
    for (int t = 0; ok && t < tiles; ++t) ok = done[t] == (uint64_t)T;
    char detail[128];
    snprintf(detail, sizeof(detail), "failed=%d timeouts=%u done_idx=%llu", f, (unsigned)tq->base.wait_timeouts,
             (unsigned long long)tq->base.done_idx);
    report("ring_tiled_per_tile_counters", ok, detail);
    CK(cudaFree(tq->d_tile_chunk_done));
    CK(cudaFreeHost(tq));
    CK(cudaFree(failed));
    CK(cudaFree(sums));
    CK(cudaFree(gpu));
    CK(cudaFreeHost(cpu));
}

static void sg_case() {
    const int lists = 40, per_list = 48;
    const uint32_t es = 4096;
    const size_t n = (size_t)lists * per_list;
    char* cpu;
    CK(cudaMallocHost(&cpu, 2 * n * es));
    fill_pattern(cpu, 2 * n * es, 77);
    char* gpu;
    CK(cudaMalloc(&gpu, n * es));
    CK(cudaMemset(gpu, 0, n * es));
    int* failed;
    CK(cudaMalloc(&failed, sizeof(int)));
    CK(cudaMemset(failed, 0, sizeof(int)));
    gfd::SGTaskQueue* sq;
    gfd::DescriptorQueue* dq;
    CK(cudaHostAlloc(&sq, sizeof(gfd::SGTaskQueue), cudaHostAllocMapped));
    CK(cudaHostAlloc(&dq, sizeof(gfd::DescriptorQueue), cudaHostAllocMapped));
    memset(sq, 0, sizeof(*sq));
    memset(dq, 0, sizeof(*dq));
    sq->wait_limit_ns = 5000000000ull;
    CK(cudaMalloc(&sq->d_list_done, gfd::MAX_SG_LISTS * 8));
    CK(cudaMemset(sq->d_list_done, 0, gfd::MAX_SG_LISTS * 8));
    gfd::CpuPollingThread poller(dq, nullptr, nullptr, 0);
    poller.set_sg_task_queue(sq);
    bool ok = poller.init_copy_engine();
    poller.start();
    sg_ring_kernel<<<1, 64>>>(dq, sq, cpu, gpu, lists, per_list, es, failed);
    CK(cudaDeviceSynchronize());
    poller.stop();
    int f = 0;
    CK(cudaMemcpy(&f, failed, sizeof(int), cudaMemcpyDeviceToHost));
    std::vector<char> got(n * es);
    CK(cudaMemcpy(got.data(), gpu, got.size(), cudaMemcpyDeviceToHost));
    bool data = true;
    for (size_t g = 0; data && g < n; ++g) data = memcmp(got.data() + g * es, cpu + g * 2 * es, es) == 0;
    ok = ok && f == 0 && data && sq->lists_completed == (uint64_t)lists && sq->wait_timeouts == 0;
    char detail[160];
    snprintf(detail, sizeof(detail), "failed=%d data=%d lists_completed=%llu timeouts=%u", f, (int)data,
             (unsigned long long)sq->lists_completed, (unsigned)sq->wait_timeouts);
    report("ring_sg_per_list_completion", ok, detail);
    CK(cudaFree(sq->d_list_done));
    CK(cudaFreeHost(sq));
    CK(cudaFreeHost(dq));
    CK(cudaFree(failed));
    CK(cudaFree(gpu));
    CK(cudaFreeHost(cpu));
}

int main() {
    tiled_case();
    sg_case();
    return g_failures ? 1 : 0;
}
