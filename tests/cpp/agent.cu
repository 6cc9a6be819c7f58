// The ring agent (device-resident consumer of the descriptor ring) serving producer
// kernels that occupy every SM, as the reference's CPU poller does
// (include/gfd/device.cuh:110-118 waiters under grids as wide as the GPU;
// README "mode 5": submit_tile / wait_chunk_done from one CTA per tile on every SM).
// The agent runs resident (gfd_ring_configure) and is on the GPU before the producer
// kernel is launched; the host synchronises with a stream, as resident mode requires
// (cudaDeviceSynchronize would wait for the agent too), and the producer kernels are
// loaded before the ring starts (with lazy module loading, a kernel's first launch waits
// for the kernels already running -- here the resident agent).
//
//  all_sm_basic    one CTA per SM (all co-resident); every thread writes the descriptor of
//                  its token (write_and_commit), thread 0 then spins on done_idx for the
//                  whole launch's tokens and the CTA sums its landed tokens.
//  all_sm_tiled    one CTA per SM, one tile each; warp 0 acquires, submits and waits for
//                  every chunk of its tile (tile counters), then the CTA sums the tile.
//  relaunch        default mode: 40 rounds of submit kernel + wait kernel +
//                  cudaDeviceSynchronize; the agent leaves after each round and the
//                  service thread brings it back at the next commit.
#include <gfd/device.cuh>
#include <gfd/device_primitives.cuh>
#include <gfd/gfd.h>

#include "common.h"
#include "gfd_b200.h"

constexpr uint64_t kWaitNs = 5000000000ull;  // 5 s

__global__ void all_sm_basic(gfd::DescriptorQueue* q, const char* cpu, char* gpu, int per_cta, uint32_t ts,
                             uint64_t base, float* sums, int* failed) {
    const int n = gridDim.x * per_cta;
    const int tok = blockIdx.x * per_cta + threadIdx.x;
    const bool active = threadIdx.x < per_cta;
    gfd::device::write_and_commit(q, base, tok, active, active ? (uint64_t)(cpu + (size_t)tok * 2 * ts) : 0, gpu, ts,
                                  n);
    __shared__ int ok;
    if (threadIdx.x == 0) ok = gfd::device::wait_for_completion_until(q, base + n, kWaitNs) ? 1 : 0;
    __syncthreads();
    if (!ok) {
        if (threadIdx.x == 0) atomicAdd(failed, 1);
        return;
    }
    if (active) {
        const float* v = reinterpret_cast<const float*>(gpu + (size_t)tok * ts);
        float s = 0.f;
        for (uint32_t d = 0; d < ts / 4; ++d) s += v[d];
        sums[tok] = s;
    }
}

__global__ void all_sm_tiled(gfd::TiledQueue* tq, const float* cpu, float* gpu, float* sums, int dim, int* failed) {
    const uint32_t tile = blockIdx.x;
    const uint32_t T = tq->scheduler.tokens_per_tile, C = tq->scheduler.tokens_per_chunk;
    const uint32_t K = tq->scheduler.chunks_per_tile, ts = tq->scheduler.token_size;
    __shared__ int ok;
    if (threadIdx.x == 0) ok = 1;
    __syncthreads();
    if (threadIdx.x < 32) {
        for (uint32_t c = 0; c < K; ++c) {
            const uint64_t b = gfd::device::acquire_chunk_slots(tq, C);
            gfd::device::wait_queue_space(tq, C);
            gfd::device::submit_chunk(tq, b, tile, c, C, T, cpu, gpu, ts);
            if (threadIdx.x == 0 && !gfd::device::wait_chunk_done_until(tq, tile, (uint64_t)(c + 1) * C, kWaitNs)) ok = 0;
            __syncwarp();
        }
    }
    __syncthreads();
    if (!ok) {
        if (threadIdx.x == 0) atomicAdd(failed, 1);
        return;
    }
    for (uint32_t t = threadIdx.x; t < T; t += blockDim.x) {
        const float* v = gpu + ((size_t)tile * T + t) * dim;
        float s = 0.f;
        for (int d = 0; d < dim; ++d) s += v[d];
        sums[tile * T + t] = s;
    }
}

__global__ void submit_kernel(gfd::DescriptorQueue* q, const char* cpu, char* gpu, int n, uint32_t ts, uint64_t base) {
    const int tid = blockIdx.x * blockDim.x + threadIdx.x;
    const bool active = tid < n;
    gfd::device::write_and_commit(q, base, tid, active, active ? (uint64_t)(cpu + (size_t)tid * 2 * ts) : 0, gpu, ts,
                                  n);
}

__global__ void wait_kernel(gfd::DescriptorQueue* q, uint64_t expected, int* ok) {
    *ok = gfd::device::wait_for_completion_until(q, expected, kWaitNs) ? 1 : 0;
}

static int num_sms() {
    int dev = 0, n = 0;
    CK(cudaGetDevice(&dev));
    CK(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
    return n;
}

static void fill_floats(char* cpu, int tokens, uint32_t ts, size_t stride) {
    for (int t = 0; t < tokens; ++t) {
        float* v = reinterpret_cast<float*>(cpu + (size_t)t * stride);
        for (uint32_t d = 0; d < ts / 4; ++d) v[d] = (float)(t % 89) + 0.5f;
    }
}

static void all_sm_basic_case() {
    const int sms = num_sms(), per_cta = 64;
    const uint32_t ts = 4096;
    const int n = sms * per_cta;
    char* cpu;
    CK(cudaMallocHost(&cpu, (size_t)n * 2 * ts));
    fill_floats(cpu, n, ts, 2 * ts);
    char* gpu;
    float* sums;
    int* failed;
    CK(cudaMalloc(&gpu, (size_t)n * ts));
    CK(cudaMemset(gpu, 0, (size_t)n * ts));
    CK(cudaMalloc(&sums, n * sizeof(float)));
    CK(cudaMalloc(&failed, sizeof(int)));
    CK(cudaMemset(failed, 0, sizeof(int)));
    gfd::DescriptorQueue* q;
    CK(cudaHostAlloc(&q, sizeof(gfd::DescriptorQueue), cudaHostAllocMapped));
    memset(q, 0, sizeof(*q));
    cudaStream_t st;
    CK(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
    CK(cudaDeviceSynchronize());
    bool ok;
    {
        gfd::CpuPollingThread poller(q, gpu, cpu, (size_t)n * 2 * ts);
        ok = poller.init_copy_engine();
        ok = ok && gfd_ring_configure(poller.ring(), 0, 0, 1) == GFD_OK;
        poller.start();
        uint64_t base = 0;
        for (int round = 0; ok && round < 3; ++round) {
            all_sm_basic<<<sms, 256, 0, st>>>(q, cpu, gpu, per_cta, ts, base, sums, failed);
            CK(cudaStreamSynchronize(st));
            base += n;
        }
        poller.stop();
        int f = 0;
        CK(cudaMemcpy(&f, failed, sizeof(int), cudaMemcpyDeviceToHost));
        std::vector<float> hs(n);
        CK(cudaMemcpy(hs.data(), sums, n * sizeof(float), cudaMemcpyDeviceToHost));
        int bad = 0;
        for (int t = 0; t < n; ++t) bad += hs[t] != ((float)(t % 89) + 0.5f) * (ts / 4);
        gfd_ring_agent_stats_t st_ = {};
        gfd_ring_agent_stats(poller.ring(), &st_);
        ok = ok && f == 0 && bad == 0 && q->done_idx == base && q->wait_timeouts == 0 && st_.timeouts == 0;
        char detail[256];
        snprintf(detail, sizeof(detail),
                 "ctas=%d failed=%d bad=%d done_idx=%llu launches=%llu timeouts=%llu exits(idle/stop/err)=%llu/%llu/%llu "
                 "resident=%llu",
                 sms, f, bad, (unsigned long long)q->done_idx, (unsigned long long)st_.launches,
                 (unsigned long long)st_.timeouts, (unsigned long long)st_.idle_exits, (unsigned long long)st_.stop_exits,
                 (unsigned long long)st_.error_exits, (unsigned long long)st_.resident);
        report("agent_all_sm_basic_api", ok, detail);
    }
    CK(cudaStreamDestroy(st));
    CK(cudaFreeHost(q));
    CK(cudaFree(failed));
    CK(cudaFree(sums));
    CK(cudaFree(gpu));
    CK(cudaFreeHost(cpu));
}

static void all_sm_tiled_case() {
    const int tiles = num_sms(), T = 64, C = 16, dim = 1024;
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
    cudaStream_t st;
    CK(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
    CK(cudaDeviceSynchronize());
    {
        gfd::CpuPollingThread poller(&tq->base, gpu, cpu, total);
        poller.set_tiled_queue(tq);
        bool ok = poller.init_copy_engine();
        ok = ok && gfd_ring_configure(poller.ring(), 0, 0, 1) == GFD_OK;
        poller.start();
        all_sm_tiled<<<tiles, 128, 0, st>>>(tq, cpu, gpu, sums, dim, failed);
        CK(cudaStreamSynchronize(st));
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
        gfd_ring_agent_stats_t st_ = {};
        gfd_ring_agent_stats(poller.ring(), &st_);
        char detail[256];
        snprintf(detail, sizeof(detail),
                 "tiles=%d failed=%d timeouts=%u done_idx=%llu launches=%llu exits(idle/stop/err)=%llu/%llu/%llu "
                 "resident=%llu",
                 tiles, f, (unsigned)tq->base.wait_timeouts, (unsigned long long)tq->base.done_idx,
                 (unsigned long long)st_.launches, (unsigned long long)st_.idle_exits, (unsigned long long)st_.stop_exits,
                 (unsigned long long)st_.error_exits, (unsigned long long)st_.resident);
        report("agent_all_sm_tiled_api", ok, detail);
    }
    CK(cudaStreamDestroy(st));
    CK(cudaFree(tq->d_tile_chunk_done));
    CK(cudaFreeHost(tq));
    CK(cudaFree(failed));
    CK(cudaFree(sums));
    CK(cudaFree(gpu));
    CK(cudaFreeHost(cpu));
}

static void relaunch_case() {
    const int n = 512;
    const uint32_t ts = 2048;
    char* cpu;
    CK(cudaMallocHost(&cpu, (size_t)n * 2 * ts));
    fill_pattern(cpu, (size_t)n * 2 * ts, 41);
    char* gpu;
    CK(cudaMalloc(&gpu, (size_t)n * ts));
    int* d_ok;
    CK(cudaMalloc(&d_ok, sizeof(int)));
    gfd::DescriptorQueue* q;
    CK(cudaMallocManaged(&q, sizeof(gfd::DescriptorQueue)));
    memset(q, 0, sizeof(*q));
    bool ok;
    {
        gfd::CpuPollingThread poller(q, gpu, cpu, (size_t)n * 2 * ts);
        ok = poller.init_copy_engine();
        poller.start();
        uint64_t base = 0;
        int bad_rounds = 0;
        for (int round = 0; round < 40; ++round) {
            CK(cudaMemset(gpu, 0, (size_t)n * ts));
            CK(cudaDeviceSynchronize());  // returns: the agent has left (or was never needed)
            submit_kernel<<<(n + 255) / 256, 256>>>(q, cpu, gpu, n, ts, base);
            base += n;
            wait_kernel<<<1, 1>>>(q, base, d_ok);
            CK(cudaDeviceSynchronize());
            int w = 0;
            CK(cudaMemcpy(&w, d_ok, sizeof(int), cudaMemcpyDeviceToHost));
            std::vector<char> got((size_t)n * ts);
            CK(cudaMemcpy(got.data(), gpu, got.size(), cudaMemcpyDeviceToHost));
            bool data = true;
            for (int i = 0; data && i < n; ++i) data = memcmp(got.data() + (size_t)i * ts, cpu + (size_t)i * 2 * ts, ts) == 0;
            bad_rounds += !(w == 1 && data);
        }
        poller.stop();
        gfd_ring_agent_stats_t st_ = {};
        gfd_ring_agent_stats(poller.ring(), &st_);
        ok = ok && bad_rounds == 0 && q->done_idx == base && st_.launches >= 2 && st_.timeouts == 0 &&
             st_.rejected == 0;
        char detail[200];
        snprintf(detail, sizeof(detail), "bad_rounds=%d done_idx=%llu launches=%llu queries=%llu idle_exits=%llu",
                 bad_rounds, (unsigned long long)q->done_idx, (unsigned long long)st_.launches,
                 (unsigned long long)st_.queries, (unsigned long long)st_.idle_exits);
        report("agent_relaunch_between_device_syncs", ok, detail);
    }
    CK(cudaFree(q));
    CK(cudaFree(d_ok));
    CK(cudaFree(gpu));
    CK(cudaFreeHost(cpu));
}

int main() {
    // load every kernel of this program now, before a resident agent runs
    cudaFuncAttributes fa;
    CK(cudaFuncGetAttributes(&fa, all_sm_basic));
    CK(cudaFuncGetAttributes(&fa, all_sm_tiled));
    CK(cudaFuncGetAttributes(&fa, submit_kernel));
    CK(cudaFuncGetAttributes(&fa, wait_kernel));
    all_sm_basic_case();
    all_sm_tiled_case();
    relaunch_case();
    return g_failures ? 1 : 0;
}
