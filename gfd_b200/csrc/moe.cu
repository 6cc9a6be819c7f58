// MoE routing front end: fp32 router logits -> top-k experts per token -> one gather
// list that packs, expert by expert, the rows of the tokens routed to it in ascending
// token order -> the device-list gather (plan + pull).
//
// This is the dynamic scatter-gather workload of the reference's SG mode
// (examples/09_sg_warp_spec.cu:246-276: one list per expert, experts ascending, each
// list holding the tokens routed to that expert in ascending token order), done as three
// stream-ordered kernels with no host round trip:
//   topk_kernel   one warp per token: k rounds of a warp arg-max over the token's
//                 logits (ties -> lower expert id; NaN ranks below every number),
//                 selected ids to scratch, per-expert counts with atomics;
//   emit_kernel   one CTA per expert: its offset = sum of the counts of lower experts,
//                 then a block-wide scan over tokens of "routed to this expert" gives
//                 each row's position; entry j = {dst + j * row_bytes, src[t], row_bytes};
//   gfd_gather_device on the entries.

#include <cuda_runtime.h>

#include <cfloat>
#include <cstdint>

#include "internal.h"

namespace gfdb {
namespace {

constexpr int kMaxExperts = 1024;
constexpr int kMaxTopK = 32;

__device__ __forceinline__ float rank_key(float v) { return (v != v) ? -FLT_MAX * 2.0f : v; }  // NaN -> -inf

// true if (va, ia) ranks above (vb, ib)
__device__ __forceinline__ bool better(float va, int ia, float vb, int ib) {
    return va > vb || (va == vb && ia < ib);
}

__global__ void __launch_bounds__(256) topk_kernel(const float* __restrict__ logits, int64_t tokens, int experts,
                                                   int k, uint16_t* __restrict__ sel, uint32_t* __restrict__ counts) {
    const int lane = threadIdx.x & 31;
    const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
    const int per_lane = (experts + 31) / 32;  // <= 32
    for (int64_t t = warp; t < tokens; t += nwarps) {
        const float* row = logits + t * experts;
        uint32_t taken = 0;  // bit m: expert lane + 32 m already selected
        for (int r = 0; r < k; ++r) {
            float bv = -FLT_MAX * 2.0f;  // -inf
            int bi = 0x7fffffff;
            for (int m = 0; m < per_lane; ++m) {
                const int e = lane + 32 * m;
                if (e < experts && !((taken >> m) & 1u)) {
                    const float v = rank_key(row[e]);
                    if (better(v, e, bv, bi)) {
                        bv = v;
                        bi = e;
                    }
                }
            }
#pragma unroll
            for (int o = 16; o; o >>= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                if (better(ov, oi, bv, bi)) {
                    bv = ov;
                    bi = oi;
                }
            }
            if ((bi & 31) == lane) taken |= 1u << (bi >> 5);
            if (lane == 0) {
                sel[t * k + r] = static_cast<uint16_t>(bi);
                atomicAdd(&counts[bi], 1u);
            }
        }
    }
}

constexpr int kEmitThreads = 1024;

__global__ void __launch_bounds__(kEmitThreads) emit_kernel(const uint16_t* __restrict__ sel, int64_t tokens, int k,
                                                            const uint32_t* __restrict__ counts,
                                                            uint32_t* __restrict__ offsets,
                                                            const uint64_t* __restrict__ token_src, uint64_t dst_base,
                                                            uint64_t row_bytes, gfd_sg_entry* __restrict__ entries) {
    __shared__ uint32_t s_warp[32];
    __shared__ uint32_t s_base, s_tile;
    const int e = blockIdx.x;
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    // offset of this expert's segment: sum of the counts of experts below e
    uint32_t part = 0;
    for (int i = t; i < e; i += kEmitThreads) part += counts[i];
#pragma unroll
    for (int o = 16; o; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
    if (lane == 0) s_warp[warp] = part;
    __syncthreads();
    if (t == 0) {
        uint32_t sum = 0;
        for (int w = 0; w < kEmitThreads / 32; ++w) sum += s_warp[w];
        s_base = sum;
        offsets[e] = sum;
    }
    __syncthreads();
    uint32_t base = s_base;
    for (int64_t t0 = 0; t0 < tokens; t0 += kEmitThreads) {
        const int64_t tok = t0 + t;
        bool hit = false;
        if (tok < tokens)
            for (int r = 0; r < k; ++r) hit |= sel[tok * k + r] == e;
        const unsigned m = __ballot_sync(0xffffffffu, hit);
        __syncthreads();  // previous tile's readers of s_warp are done
        if (lane == 0) s_warp[warp] = __popc(m);
        __syncthreads();
        if (warp == 0) {
            const uint32_t c = s_warp[lane];
            uint32_t incl = c;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += y;
            }
            s_warp[lane] = incl - c;  // exclusive prefix of this warp's hits
            if (lane == 31) s_tile = incl;
        }
        __syncthreads();
        if (hit) {
            const uint64_t j = base + s_warp[warp] + __popc(m & ((1u << lane) - 1u));
            entries[j] = gfd_sg_entry{dst_base + j * row_bytes, reinterpret_cast<const void*>(token_src[tok]), row_bytes};
        }
        base += s_tile;
    }
}

}  // namespace
}  // namespace gfdb

using namespace gfdb;

extern "C" int gfd_moe_route_gather(gfd_ctx* ctx, const float* d_logits, int64_t tokens, int experts, int k,
                                    const uint64_t* d_token_src, size_t row_bytes, void* dst_base, size_t dst_bytes,
                                    uint32_t* d_counts, uint32_t* d_offsets, gfd_sg_entry* d_entries, void* stream,
                                    uint32_t flags) {
    if (!ctx) return GFD_ERR_INVALID;
    {
        std::lock_guard<std::mutex> lk(ctx->mu);
        CtxScope scope(ctx->cu_ctx);
        if (tokens <= 0 || experts <= 0 || experts > kMaxExperts || k <= 0 || k > experts || k > kMaxTopK ||
            row_bytes == 0)
            return set_error(ctx, GFD_ERR_INVALID, "moe_route: bad shape (tokens %lld, experts %d, k %d)",
                             (long long)tokens, experts, k);
        const uint64_t rows = static_cast<uint64_t>(tokens) * k;
        if (rows > 0x7fffffffull || rows * row_bytes > dst_bytes)
            return set_error(ctx, GFD_ERR_INVALID, "moe_route: destination holds fewer than tokens*k rows");
        struct {
            const void* p;
            uint64_t n;
            const char* what;
        } bufs[] = {{d_logits, static_cast<uint64_t>(tokens) * experts * sizeof(float), "logits"},
                    {d_token_src, static_cast<uint64_t>(tokens) * sizeof(uint64_t), "token_src"},
                    {d_counts, static_cast<uint64_t>(experts) * sizeof(uint32_t), "counts"},
                    {d_offsets, static_cast<uint64_t>(experts) * sizeof(uint32_t), "offsets"},
                    {d_entries, rows * sizeof(gfd_sg_entry), "entries"},
                    {dst_base, dst_bytes, "dst"}};
        for (const auto& b : bufs)
            if (!check_dev(ctx, reinterpret_cast<uint64_t>(b.p), b.n))
                return set_error(ctx, GFD_ERR_INVALID, "moe_route: %s is not device memory of GPU %d", b.what,
                                 ctx->device);
        if (ctx->d_sel_capacity < rows) {
            if (ctx->d_sel) cudaFree(ctx->d_sel);
            ctx->d_sel = nullptr;
            ctx->d_sel_capacity = 0;
            if (cudaMalloc(&ctx->d_sel, rows * sizeof(uint16_t)) != cudaSuccess) {
                cudaGetLastError();
                return set_error(ctx, GFD_ERR_NOMEM, "moe_route: selection scratch");
            }
            ctx->d_sel_capacity = rows;
        }
        cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
        cudaError_t e = cudaMemsetAsync(d_counts, 0, experts * sizeof(uint32_t), st);
        if (e != cudaSuccess) return cuda_error(ctx, e, "moe_route: clearing counts");
        const int64_t warps_needed = tokens;
        int grid = static_cast<int>((warps_needed + 7) / 8);
        if (grid > 8 * ctx->num_sms) grid = 8 * ctx->num_sms;
        topk_kernel<<<grid, 256, 0, st>>>(d_logits, tokens, experts, k, ctx->d_sel, d_counts);
        emit_kernel<<<experts, kEmitThreads, 0, st>>>(ctx->d_sel, tokens, k, d_counts, d_offsets, d_token_src,
                                                      reinterpret_cast<uint64_t>(dst_base), row_bytes, d_entries);
        e = cudaGetLastError();
        if (e != cudaSuccess) return cuda_error(ctx, e, "moe_route: kernel launch");
    }
    if (flags & GFD_MOE_ROUTE_ONLY) return GFD_OK;
    return gfd_gather_device(ctx, d_entries, static_cast<int64_t>(tokens) * k, dst_base, dst_bytes, stream, 0);
}
