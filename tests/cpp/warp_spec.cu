// WarpSpecSession + GFD_WARP_SPEC_KERNEL / GFD_WARP_SPEC_KERNEL_DB: the producer warps
// pull linear tiles from pinned host memory while compute warps reduce each chunk.
// Case matrix follows the reference test/test_db_small_tiles.cu (tile counts
// 1,2,3,4,5,7; tile 32 / chunk 16; 1 KiB tokens of value t+1) plus single-buffer,
// per-tile mode, auto chunking, the reference launch shape (one producer warp) and a
// tail of tokens beyond the last full tile (not transferred, as in the reference).
#include <gfd/gfd.h>
#include <gfd/warp_spec.cuh>

#include <cmath>

#include "common.h"

struct SumTokens {
    float* out;
    int dim;
    __device__ void operator()(gfd::warp_spec::ChunkView chunk) {
        for (uint32_t i = chunk.lane_id; i < chunk.size; i += 32) {
            const float* t = chunk.data<float>(i);
            float s = 0.f;
            for (int d = 0; d < dim; ++d) s += t[d];
            out[chunk.global_idx(i)] = s;
        }
    }
};

GFD_WARP_SPEC_KERNEL(sum_kernel, SumTokens);
GFD_WARP_SPEC_KERNEL_DB(sum_kernel_db, SumTokens);

static bool run_case(const char* name, int total_tokens, int tile, int chunk, int dim, bool db, int blocks,
                     bool per_tile, int producer_warps) {
    const size_t token_size = dim * sizeof(float);
    const size_t total = (size_t)total_tokens * token_size;
    float* cpu;
    CK(cudaMallocHost(&cpu, total));
    for (int t = 0; t < total_tokens; ++t)
        for (int d = 0; d < dim; ++d) cpu[(size_t)t * dim + d] = (float)(t + 1);
    float* gpu;
    CK(cudaMalloc(&gpu, total));
    CK(cudaMemset(gpu, 0, total));
    float* out;
    CK(cudaMalloc(&out, total_tokens * sizeof(float)));
    CK(cudaMemset(out, 0, total_tokens * sizeof(float)));

    gfd::WarpSpecConfig cfg;
    cfg.total_tokens = total_tokens;
    cfg.token_size = (uint32_t)token_size;
    cfg.cpu_src = cpu;
    cfg.gpu_dst = gpu;
    cfg.tokens_per_tile = tile;
    cfg.tokens_per_chunk = chunk;
    cfg.num_blocks = blocks;
    cfg.double_buffer = db;
    cfg.per_tile_mode = per_tile;
    cfg.producer_warps = producer_warps;
    bool ok;
    {
        gfd::WarpSpecSession s(cfg);
        if (producer_warps < 0) {
            // reference launch shape: one transfer warp + K (or 2K) compute warps
            auto p = s.get_launch_params();
            const int k = (int)cfg.chunks_per_tile();
            dim3 block((1 + (db ? 2 * k : k)) * 32);
            s.reset();
            if (db) sum_kernel_db<<<p.grid, block>>>(p.tq, p.gpu_buffer, p.cpu_base, SumTokens{out, dim});
            else sum_kernel<<<p.grid, block>>>(p.tq, p.gpu_buffer, p.cpu_base, SumTokens{out, dim});
        } else if (db) {
            s.launch(sum_kernel_db, SumTokens{out, dim});
        } else {
            s.launch(sum_kernel, SumTokens{out, dim});
        }
        s.synchronize();
        const int full = (total_tokens / tile) * tile;
        std::vector<float> h(total_tokens);
        CK(cudaMemcpy(h.data(), out, total_tokens * sizeof(float), cudaMemcpyDeviceToHost));
        ok = s.ok() && s.timeouts() == 0;
        for (int t = 0; ok && t < total_tokens; ++t) {
            const float want = t < full ? (float)(t + 1) * dim : 0.f;
            ok = std::fabs(h[t] - want) <= 1.0f;
        }
        ok = ok && device_equals(gpu, cpu, (size_t)full * token_size);
        std::vector<char> tail(total - (size_t)full * token_size);
        if (!tail.empty()) {
            CK(cudaMemcpy(tail.data(), (char*)gpu + (size_t)full * token_size, tail.size(), cudaMemcpyDeviceToHost));
            for (char c : tail) ok = ok && c == 0;
        }
        auto st = s.get_stats();
        char detail[160];
        snprintf(detail, sizeof(detail), "tokens=%d tile=%d chunk=%u K=%u blocks=%d landed=%llu", total_tokens, tile,
                 cfg.effective_tokens_per_chunk(), cfg.chunks_per_tile(), blocks,
                 (unsigned long long)st.descriptors_processed);
        ok = ok && st.descriptors_processed == (uint64_t)full && st.bytes_transferred == (uint64_t)full * token_size;
        report(name, ok, detail);
    }
    CK(cudaFree(out));
    CK(cudaFree(gpu));
    CK(cudaFreeHost(cpu));
    return ok;
}

int main() {
    int sms = 0;
    CK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, 0));
    const int tiles_list[] = {1, 2, 3, 4, 5, 7};
    char name[96];
    for (int tiles : tiles_list) {
        snprintf(name, sizeof(name), "db_small_tiles_%d", tiles);
        run_case(name, tiles * 32, 32, 16, 256, true, tiles < sms ? tiles : sms, false, 0);
    }
    for (int tiles : {1, 2, 3, 5}) {
        snprintf(name, sizeof(name), "db_k1_tiles_%d", tiles);
        run_case(name, tiles * 32, 32, 32, 256, true, 1, false, 0);
    }
    for (int tiles : {1, 2, 3}) {
        snprintf(name, sizeof(name), "db_k4_tiles_%d", tiles);
        run_case(name, tiles * 64, 64, 16, 256, true, 2, false, 0);
    }
    run_case("single_many_tiles", 8192, 128, 0, 1024, false, 0, false, 0);
    run_case("single_per_tile_mode", 4096, 128, 0, 256, false, 16, true, 0);
    run_case("single_tail_tokens", 1000, 128, 32, 64, false, 8, false, 2);
    run_case("db_ref_launch_shape", 2048, 128, 32, 256, true, 8, false, -1);
    run_case("single_ref_launch_shape", 2048, 128, 32, 256, false, 8, false, -1);
    run_case("single_one_block", 1024, 64, 16, 512, false, 1, false, 8);
    return g_failures ? 1 : 0;
}
