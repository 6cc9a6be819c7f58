/*
 * TEST INFRASTRUCTURE ONLY -- CPU oracle for the two callers either side of the gather:
 * MoE routing (which rows a GPU gathers, and where they land) and the per-block
 * RMS-scale compute of the layer pipeline.  Loaded only by tests/, __graft_entry__.smoke()
 * and bench.py's cpu_baseline leg; the product path never does.
 *
 * MoE routing: every token takes its k largest logits; the destination holds, expert by
 * expert in ascending id, the rows of the tokens routed to that expert in ascending
 * token order.  The list order is the reference's per-expert SG list construction
 * (examples/09_sg_warp_spec.cu:246-276: outer loop over experts, inner loop over tokens
 * t = 0.., one entry per routed token).  The reference routes round-robin
 * (examples/09_sg_warp_spec.cu:509); top-k over logits is the benchmark's routing and
 * is specified here: ties go to the lower expert id, NaN ranks below every number
 * (including -inf, against which the lower id wins).
 *
 * RMS scale: the reference's functor computes sum of squares over a token, then
 * rsqrtf(sum / n + 1e-6) (examples/07_warp_spec_simple.cu:35-59).  This restatement
 * fixes every rounding so the GPU result is reproducible bit for bit:
 *   - values are bf16; a block is read as 16-byte vectors of 8 values; lane l of 32
 *     owns vectors l, l+32, l+64, ... and accumulates, vector by vector and value by
 *     value in address order, acc = fmaf(x, x, acc) (one rounding per step);
 *   - the 32 lane sums combine by a butterfly: for o = 16, 8, 4, 2, 1 every lane adds
 *     the sum of lane l^o (the float sum is commutative, so all lanes agree);
 *   - mean = ss / n, s = 1 / sqrtf(mean + eps), each correctly rounded (IEEE);
 *   - y = bf16_rne(x * s) with the product correctly rounded to fp32 first.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

static float key_of(float v) { return isnan(v) ? -INFINITY : v; }

/* 1 when (va, ia) ranks above (vb, ib) */
static int ranks_above(float va, int ia, float vb, int ib) { return va > vb || (va == vb && ia < ib); }

/* sel[t*k + r]: r-th choice of token t.  counts[e], offsets[e]: rows routed to e and
 * the first row of e's segment.  row_token[j]: the token whose row lands at row j.
 * Returns 0, or -1 on a bad shape. */
int gfd_oracle_moe_route(const float* logits, int64_t tokens, int experts, int k, uint16_t* sel,
                         uint32_t* counts, uint32_t* offsets, int64_t* row_token) {
    if (tokens <= 0 || experts <= 0 || experts > 1024 || k <= 0 || k > experts || k > 32) return -1;
    memset(counts, 0, sizeof(uint32_t) * (size_t)experts);
    unsigned char taken[1024];
    for (int64_t t = 0; t < tokens; ++t) {
        const float* row = logits + t * experts;
        memset(taken, 0, (size_t)experts);
        for (int r = 0; r < k; ++r) {
            float bv = -INFINITY;
            int bi = 0x7fffffff;
            for (int e = 0; e < experts; ++e) {
                if (taken[e]) continue;
                const float v = key_of(row[e]);
                if (ranks_above(v, e, bv, bi)) {
                    bv = v;
                    bi = e;
                }
            }
            taken[bi] = 1;
            sel[t * k + r] = (uint16_t)bi;
            counts[bi]++;
        }
    }
    uint32_t acc = 0;
    for (int e = 0; e < experts; ++e) {
        offsets[e] = acc;
        acc += counts[e];
    }
    int64_t j = 0;
    for (int e = 0; e < experts; ++e)
        for (int64_t t = 0; t < tokens; ++t)
            for (int r = 0; r < k; ++r)
                if (sel[t * k + r] == e) {
                    row_token[j++] = t;
                    break;
                }
    return 0;
}

static float bf16_to_f32(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

static uint16_t f32_to_bf16_rne(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u); /* quiet NaN */
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

/* Scales one block of n bf16 values (n a multiple of 8) in place; returns its fp32 sum
 * of squares. */
float gfd_oracle_rms_scale(uint16_t* v, uint64_t n, float eps) {
    float lane[32];
    const uint64_t nvec = n / 8;
    for (int l = 0; l < 32; ++l) {
        float acc = 0.0f;
        for (uint64_t j = (uint64_t)l; j < nvec; j += 32)
            for (int e = 0; e < 8; ++e) {
                const float x = bf16_to_f32(v[j * 8 + (uint64_t)e]);
                acc = fmaf(x, x, acc);
            }
        lane[l] = acc;
    }
    for (int o = 16; o; o >>= 1) {
        float next[32];
        for (int l = 0; l < 32; ++l) next[l] = lane[l] + lane[l ^ o];
        memcpy(lane, next, sizeof(lane));
    }
    const float ss = lane[0];
    const float mean = ss / (float)n;
    const float s = 1.0f / sqrtf(mean + eps);
    for (uint64_t i = 0; i < n; ++i) v[i] = f32_to_bf16_rne(bf16_to_f32(v[i]) * s);
    return ss;
}

/* The layer pipeline over a pool: out block g = rms_scale(pool block table[g]); ss[g]
 * receives its sum of squares.  Returns -1, or the first g whose id is >= pool_blocks
 * (that block of out is left untouched and ss[g] = 0). */
int64_t gfd_oracle_layer_pipeline(uint16_t* out, float* ss, const uint16_t* pool, uint64_t pool_blocks,
                                  const uint32_t* table, uint64_t nblocks, uint64_t block_bytes, float eps) {
    int64_t first_bad = -1;
    const uint64_t n = block_bytes / 2;
    for (uint64_t g = 0; g < nblocks; ++g) {
        if (table[g] >= pool_blocks) {
            if (first_bad < 0) first_bad = (int64_t)g;
            ss[g] = 0.0f;
            continue;
        }
        memcpy(out + g * n, pool + (uint64_t)table[g] * n, block_bytes);
        ss[g] = gfd_oracle_rms_scale(out + g * n, n, eps);
    }
    return first_bad;
}
