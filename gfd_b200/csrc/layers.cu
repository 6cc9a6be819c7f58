// Layer pipeline: the GPU-initiated, page-table-driven KV fetch with dependent compute,
// written against the library's own WarpSpecSession API the way an application uses it
// (the reference's examples/07_warp_spec_simple.cu pattern: a functor, one macro, one
// session).  Built as libgfd_layers.so, a client of libgfd_b200.so, and exported through
// a small C ABI for tests and benchmarks.
//
// One launch covers every layer: token g of the launch is block g % per_layer of layer
// g / per_layer, read from pool block table[g] (page-table mode).  Tiles are claimed in
// order, so producer warps pull the tiles of layer l + 1 while the compute warps of the
// same CTAs scale the tiles of layer l already landed.
//
// Compute (RmsScale): per 64 KiB block, fp32 sum of squares and an in-place scale of the
// bf16 values by 1 / sqrt(ss / n + eps) -- the reference functor's first pass
// (examples/07_warp_spec_simple.cu:35-48) with every rounding fixed so the result is
// reproducible bit for bit: lane l of the warp owns 16-byte vectors l, l + 32, ...,
// accumulates x * x with fused multiply-adds in address order, the 32 lane sums combine
// by an xor butterfly (16, 8, 4, 2, 1), the divide and square root are the correctly
// rounded ones, and each scaled value rounds to bf16 to nearest even.

#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>

#include "gfd/warp_spec.cuh"
#include "gfd/warp_spec_session.h"

namespace {

__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

// fp32 -> bf16, round to nearest even (quiet NaN kept)
__device__ __forceinline__ uint32_t to_bf16(float f) {
    uint32_t u = __float_as_uint(f);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (u >> 16) | 0x40u;
    u += 0x7fffu + ((u >> 16) & 1u);
    return u >> 16;
}

__device__ __forceinline__ uint32_t scale_pair(uint32_t w, float s) {
    return to_bf16(__fmul_rn(bf16_lo(w), s)) | (to_bf16(__fmul_rn(bf16_hi(w), s)) << 16);
}

__device__ __forceinline__ float sq_pair(uint32_t w, float acc) {
    acc = __fmaf_rn(bf16_lo(w), bf16_lo(w), acc);
    return __fmaf_rn(bf16_hi(w), bf16_hi(w), acc);
}

struct NoCompute {
    __device__ void operator()(gfd::warp_spec::ChunkView) const {}
};

struct RmsScale {
    float* ss;  // per-token sum of squares (device), indexed by the launch's token index
    float eps;

    __device__ void operator()(gfd::warp_spec::ChunkView v) const {
        const uint32_t nvec = v.token_size / 16u;
        const float n = static_cast<float>(v.token_size / 2u);
        for (uint32_t i = 0; i < v.size; ++i) {
            uint4* p = v.data<uint4>(static_cast<int>(i));
            float acc = 0.0f;
            for (uint32_t j = static_cast<uint32_t>(v.lane_id); j < nvec; j += 32u) {
                const uint4 q = p[j];
                acc = sq_pair(q.x, acc);
                acc = sq_pair(q.y, acc);
                acc = sq_pair(q.z, acc);
                acc = sq_pair(q.w, acc);
            }
#pragma unroll
            for (int o = 16; o; o >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, o));
            const float s = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(acc, n), eps)));
            for (uint32_t j = static_cast<uint32_t>(v.lane_id); j < nvec; j += 32u) {
                uint4 q = p[j];
                q.x = scale_pair(q.x, s);
                q.y = scale_pair(q.y, s);
                q.z = scale_pair(q.z, s);
                q.w = scale_pair(q.w, s);
                p[j] = q;
            }
            if (v.lane_id == 0 && ss != nullptr) ss[v.global_idx(static_cast<int>(i))] = acc;
        }
    }
};

GFD_WARP_SPEC_KERNEL(layers_transfer_kernel, NoCompute);
GFD_WARP_SPEC_KERNEL(layers_rms_kernel, RmsScale);
GFD_WARP_SPEC_KERNEL_DB(layers_rms_kernel_db, RmsScale);

}  // namespace

struct gfd_layers {
    gfd::WarpSpecSession* session = nullptr;
    float* ss = nullptr;
    float eps = 1e-6f;
    bool double_buffer = false;
};

extern "C" {

// pool: pinned, device-mapped host memory of pool_bytes (0: to the end of its
// allocation); table: device array of total_blocks pool block ids; dst: device memory of
// total_blocks * block_bytes; ss: device array of total_blocks floats (may be NULL).
int gfd_layers_create(const void* pool, uint64_t pool_bytes, const uint32_t* table, uint32_t total_blocks,
                      uint32_t block_bytes,
                      void* dst, float* ss, uint32_t tokens_per_tile, int producer_warps, int double_buffer,
                      uint64_t wait_timeout_ms, gfd_layers** out) {
    if (out == nullptr) return 1;
    *out = nullptr;
    if (block_bytes == 0 || block_bytes % 16 != 0 || tokens_per_tile == 0 || total_blocks % tokens_per_tile != 0) {
        std::fprintf(stderr, "gfd_layers_create: block_bytes must be a multiple of 16 and total_blocks a multiple "
                             "of tokens_per_tile\n");
        return 1;
    }
    gfd::WarpSpecConfig cfg;
    cfg.total_tokens = total_blocks;
    cfg.token_size = block_bytes;
    cfg.cpu_src = const_cast<void*>(pool);
    cfg.gpu_dst = dst;
    cfg.tokens_per_tile = tokens_per_tile;
    cfg.producer_warps = producer_warps;
    cfg.double_buffer = double_buffer != 0;
    cfg.wait_timeout_ms = wait_timeout_ms;
    cfg.block_table = table;
    cfg.src_pool_bytes = pool_bytes;
    auto* l = new gfd_layers;
    l->session = new gfd::WarpSpecSession(cfg);
    l->ss = ss;
    l->double_buffer = cfg.double_buffer;
    if (!l->session->ok()) {
        delete l->session;
        delete l;
        return 1;
    }
    *out = l;
    return 0;
}

// Launches one pass over every layer on `stream`.  mode 0: transfer only; 1: transfer
// and RmsScale.  The previous pass must have completed (gfd_layers_sync).
int gfd_layers_run(gfd_layers* l, int mode, void* stream) {
    if (l == nullptr) return 1;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (mode == 0) {
        l->session->launch(layers_transfer_kernel, NoCompute{}, st);
    } else {
        RmsScale fn{l->ss, l->eps};
        if (l->double_buffer)
            l->session->launch(layers_rms_kernel_db, fn, st);
        else
            l->session->launch(layers_rms_kernel, fn, st);
    }
    return l->session->last_launch_ok() ? 0 : 1;
}

// Waits for the pass; reports tokens skipped for a bad block id and in-kernel waits that
// gave up.  Returns 0 when both are zero.
int gfd_layers_sync(gfd_layers* l, uint64_t* rejected, uint64_t* timeouts, uint64_t* bytes) {
    if (l == nullptr) return 1;
    l->session->synchronize();
    const auto st = l->session->get_stats();
    const uint64_t to = l->session->timeouts();
    const uint64_t rj = l->session->rejected();
    if (rejected) *rejected = rj;
    if (timeouts) *timeouts = to;
    if (bytes) *bytes = st.bytes_transferred;
    return (rj == 0 && to == 0) ? 0 : 1;
}

int gfd_layers_block_threads(const gfd_layers* l) {
    return l ? static_cast<int>(l->session->get_launch_params().block.x) : 0;
}

void gfd_layers_destroy(gfd_layers* l) {
    if (l == nullptr) return;
    delete l->session;
    delete l;
}

}  // extern "C"
