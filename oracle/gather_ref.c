/*
 * TEST INFRASTRUCTURE ONLY -- the CPU oracle for the scattered host->device gather.
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg may load this
 * file's library (oracle/_build/libgfd_oracle.so); the product path never does.
 *
 * Restates the reference's data path for GFD Direct and GFD Queue:
 *   - dst-contiguous lists: each entry's bytes are written at staging[dst - min_dst]
 *     (reference src/parallel_gather.cpp:100-107 via streaming_memcpy_g :10-27) and the
 *     staging buffer is DMA'd to min_dst (src/direct_submit.cpp:68-142); the copy
 *     engine copies bytes exactly, so GPU bytes == staging bytes;
 *   - other lists: one cuMemcpyHtoDAsync per entry (src/copy_engine.cpp:89-153,
 *     src/direct_submit.cpp:143-145), i.e. a memcpy per entry.
 * Both reduce to: for every entry in order, out[dst - base .. + size) = src bytes.
 * Overlapping destinations are left undefined by the reference (per-entry copies
 * spread over three streams run in any order); callers of the oracle do not use them.
 *
 * Parity pinning: tests/golden/ holds outputs of the reference's own
 * parallel_gather, compiled from the reference sources by oracle/Makefile and run on
 * seeded inputs (tests/golden/make_golden.py); tests/test_oracle.py checks this
 * restatement against them.
 */
#include <stdint.h>
#include <string.h>

typedef struct {
    uint64_t dst;     /* device address */
    const void* src;  /* host address */
    uint64_t size;    /* bytes */
} gfd_oracle_entry;   /* layout of gfd::SGEntry (reference include/gfd/copy_engine.h:29-33) */

/* Writes every entry into out[0, out_len) (out represents device bytes from out_base).
 * Returns -1 on success or the index of the first entry that falls outside the window. */
int64_t gfd_oracle_gather(uint8_t* out, uint64_t out_base, uint64_t out_len,
                          const gfd_oracle_entry* e, int64_t n) {
    for (int64_t i = 0; i < n; ++i) {
        if (e[i].size == 0) continue;
        if (e[i].dst < out_base || e[i].dst - out_base > out_len ||
            e[i].size > out_len - (e[i].dst - out_base))
            return i;
    }
    for (int64_t i = 0; i < n; ++i)
        if (e[i].size) memcpy(out + (e[i].dst - out_base), e[i].src, e[i].size);
    return -1;
}

/* 64-bit checksum of a byte range: FNV-1a over 8-byte little-endian words, tail bytes
 * zero-padded, length folded in at the end.  Used for size-independent parity checks. */
uint64_t gfd_oracle_checksum(const void* p, uint64_t n) {
    const uint8_t* b = (const uint8_t*)p;
    uint64_t h = 0xcbf29ce484222325ull;
    uint64_t i = 0;
    for (; i + 8 <= n; i += 8) {
        uint64_t w;
        memcpy(&w, b + i, 8);
        h ^= w;
        h *= 0x100000001b3ull;
    }
    if (i < n) {
        uint64_t w = 0;
        memcpy(&w, b + i, n - i);
        h ^= w;
        h *= 0x100000001b3ull;
    }
    h ^= n;
    h *= 0x100000001b3ull;
    return h;
}

/* Checksum of each of `count` consecutive records of `rec` bytes, then of the list of
 * checksums ("checksum of checksums"), so a mismatch can be localised per token. */
uint64_t gfd_oracle_checksum_records(const void* p, uint64_t rec, uint64_t count, uint64_t* per) {
    const uint8_t* b = (const uint8_t*)p;
    for (uint64_t i = 0; i < count; ++i) per[i] = gfd_oracle_checksum(b + i * rec, rec);
    return gfd_oracle_checksum(per, count * 8);
}

/* Checksums of scattered source records (the expected per-token checksums). */
void gfd_oracle_checksum_entries(const gfd_oracle_entry* e, int64_t n, uint64_t* per) {
    for (int64_t i = 0; i < n; ++i) per[i] = gfd_oracle_checksum(e[i].src, e[i].size);
}
