/*
 * Seeded synthetic inputs for the benchmark configurations (libgfd_workload.so).
 *
 * Generator: xoshiro256** (Blackman & Vigna, public domain algorithm) seeded
 * through splitmix64.  Large buffers are filled in independent 1 MiB blocks, block b
 * seeded with splitmix64(seed ^ (b * 0x9E3779B97F4A7C15)), so the bytes do not
 * depend on the number of threads used.
 *
 * Normal values use Box-Muller in single precision (24-bit uniforms, logf / sqrtf /
 * sincosf), then bfloat16 with round-to-nearest-even on the bit pattern.
 */
#define _GNU_SOURCE
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <string.h>

typedef struct { uint64_t s[4]; } xo_t;

static uint64_t splitmix64(uint64_t* x) {
    uint64_t z = (*x += 0x9E3779B97F4A7C15ull);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

static void xo_seed(xo_t* g, uint64_t seed) {
    uint64_t x = seed;
    for (int i = 0; i < 4; ++i) g->s[i] = splitmix64(&x);
}

static inline uint64_t rotl(uint64_t v, int k) { return (v << k) | (v >> (64 - k)); }

static inline uint64_t xo_next(xo_t* g) {
    uint64_t* s = g->s;
    const uint64_t r = rotl(s[1] * 5, 7) * 9;
    const uint64_t t = s[1] << 17;
    s[2] ^= s[0];
    s[3] ^= s[1];
    s[1] ^= s[2];
    s[0] ^= s[3];
    s[2] ^= t;
    s[3] = rotl(s[3], 45);
    return r;
}

static inline uint16_t f32_to_bf16_rne(float f) {
    uint32_t b;
    memcpy(&b, &f, 4);
    if ((b & 0x7f800000u) == 0x7f800000u && (b & 0x007fffffu)) return (uint16_t)((b >> 16) | 0x40);
    b += 0x7fffu + ((b >> 16) & 1u);
    return (uint16_t)(b >> 16);
}

#define BLOCK (1u << 20)

static uint64_t block_seed(uint64_t seed, uint64_t b) {
    uint64_t x = seed ^ (b * 0x9E3779B97F4A7C15ull);
    return splitmix64(&x);
}

static void fill_bytes_block(uint8_t* p, uint64_t n, uint64_t seed) {
    xo_t g;
    xo_seed(&g, seed);
    uint64_t i = 0;
    for (; i + 8 <= n; i += 8) {
        uint64_t v = xo_next(&g);
        memcpy(p + i, &v, 8);
    }
    if (i < n) {
        uint64_t v = xo_next(&g);
        memcpy(p + i, &v, n - i);
    }
}

/* normal values: Box-Muller pairs in float; block b covers elements [b*BLOCK/esz, ...) */
static void fill_normal_block(void* out, int esz, uint64_t count, uint64_t seed, double mean,
                              double std) {
    xo_t g;
    xo_seed(&g, seed);
    const float m = (float)mean, sd = (float)std;
    for (uint64_t i = 0; i < count; i += 2) {
        const uint64_t r = xo_next(&g);
        /* two 24-bit uniforms; u1 in (0, 1], u2 in [0, 1) */
        const float u1 = ((float)((r >> 40) & 0xFFFFFF) + 1.0f) * (1.0f / 16777216.0f);
        const float u2 = (float)((r >> 16) & 0xFFFFFF) * (1.0f / 16777216.0f);
        const float rad = sqrtf(-2.0f * logf(u1));
        float sn, cs;
        sincosf(6.28318530718f * u2, &sn, &cs);
        const float z[2] = {m + sd * rad * cs, m + sd * rad * sn};
        for (int k = 0; k < 2 && i + k < count; ++k) {
            if (esz == 2) ((uint16_t*)out)[i + k] = f32_to_bf16_rne(z[k]);
            else ((float*)out)[i + k] = z[k];
        }
    }
}

typedef struct {
    int kind; /* 0 bytes, 1 bf16 normal, 2 f32 normal */
    uint8_t* base;
    uint64_t nbytes;
    uint64_t seed;
    double mean, std;
    uint64_t b0, b1; /* block range */
} job_t;

static void* run_job(void* arg) {
    job_t* j = (job_t*)arg;
    for (uint64_t b = j->b0; b < j->b1; ++b) {
        const uint64_t off = b * (uint64_t)BLOCK;
        uint64_t n = j->nbytes - off;
        if (n > BLOCK) n = BLOCK;
        const uint64_t s = block_seed(j->seed, b);
        if (j->kind == 0) fill_bytes_block(j->base + off, n, s);
        else if (j->kind == 1) fill_normal_block(j->base + off, 2, n / 2, s, j->mean, j->std);
        else fill_normal_block(j->base + off, 4, n / 4, s, j->mean, j->std);
    }
    return 0;
}

static void run_parallel(int kind, void* base, uint64_t nbytes, uint64_t seed, double mean,
                         double std, int threads) {
    if (threads < 1) threads = 1;
    if (threads > 64) threads = 64;
    const uint64_t nblocks = (nbytes + BLOCK - 1) / BLOCK;
    pthread_t th[64];
    int live[64] = {0};
    job_t jobs[64];
    for (int t = 0; t < threads; ++t) {
        jobs[t].kind = kind;
        jobs[t].base = (uint8_t*)base;
        jobs[t].nbytes = nbytes;
        jobs[t].seed = seed;
        jobs[t].mean = mean;
        jobs[t].std = std;
        jobs[t].b0 = nblocks * t / threads;
        jobs[t].b1 = nblocks * (t + 1) / threads;
    }
    for (int t = 1; t < threads; ++t) live[t] = pthread_create(&th[t], 0, run_job, &jobs[t]) == 0;
    run_job(&jobs[0]);
    for (int t = 1; t < threads; ++t) {
        if (live[t]) pthread_join(th[t], 0);
        else run_job(&jobs[t]);
    }
}

void gfdw_fill_bytes(void* buf, uint64_t nbytes, uint64_t seed, int threads) {
    run_parallel(0, buf, nbytes, seed, 0.0, 0.0, threads);
}

/* count bf16 values (nbytes = 2*count); BLOCK holds an even number of values */
void gfdw_fill_bf16_normal(void* buf, uint64_t count, uint64_t seed, double mean, double std,
                           int threads) {
    run_parallel(1, buf, count * 2, seed, mean, std, threads);
}

void gfdw_fill_f32_normal(void* buf, uint64_t count, uint64_t seed, double mean, double std,
                          int threads) {
    run_parallel(2, buf, count * 4, seed, mean, std, threads);
}

/* Fisher-Yates: out = permutation of 0..n-1 (i from n-1 down to 1, j uniform in [0, i]) */
void gfdw_permutation(uint32_t* out, uint32_t n, uint64_t seed) {
    xo_t g;
    xo_seed(&g, seed);
    for (uint32_t i = 0; i < n; ++i) out[i] = i;
    for (uint32_t i = n; i > 1; --i) {
        const uint32_t k = i - 1;
        /* unbiased bounded draw (Lemire) */
        uint64_t m = (uint64_t)(uint32_t)(xo_next(&g) >> 32) * (uint64_t)i;
        uint32_t l = (uint32_t)m;
        if (l < i) {
            const uint32_t th = (uint32_t)(-i) % i;
            while (l < th) {
                m = (uint64_t)(uint32_t)(xo_next(&g) >> 32) * (uint64_t)i;
                l = (uint32_t)m;
            }
        }
        const uint32_t j = (uint32_t)(m >> 32);
        const uint32_t tmp = out[k];
        out[k] = out[j];
        out[j] = tmp;
    }
}
