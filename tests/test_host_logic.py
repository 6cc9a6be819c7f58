"""Host-side table logic on the CPU (no GPU): run merging, misc rows, the stream layout
and the per-CTA partition the pull kernel relies on (gfd_b200/csrc/table.h, compiled
here with g++ through tests/host_logic.cpp).  The property checked is the reference's
gather semantics: replaying the table moves exactly the bytes the entries name
(src/parallel_gather.cpp:10-27)."""
import ctypes
import os
import subprocess
import tempfile

import numpy as np
import pytest

from gfd_b200 import workloads as wl

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ROW = np.dtype([("src", "<u8"), ("dst", "<u8"), ("len", "<u8"), ("start", "<u8")])


@pytest.fixture(scope="module")
def lib():
    out = os.path.join(tempfile.mkdtemp(prefix="gfdt_"), "libgfdt.so")
    subprocess.check_call(["g++", "-std=c++17", "-O2", "-shared", "-fPIC", "-Wall", "-Werror",
                           "-I", os.path.join(ROOT, "gfd_b200", "csrc"), "-I", os.path.join(ROOT, "include"),
                           os.path.join(ROOT, "tests", "host_logic.cpp"), "-o", out])
    l = ctypes.CDLL(out)
    vp, u32p = ctypes.c_void_p, ctypes.POINTER(ctypes.c_uint32)
    l.gfdt_build.argtypes = [vp, vp, vp, ctypes.c_int, vp, u32p, vp, u32p]
    l.gfdt_build.restype = ctypes.c_uint64
    l.gfdt_build_split.argtypes = [vp, vp, vp, ctypes.c_int, ctypes.c_uint64, vp, u32p, vp, u32p, vp, u32p]
    l.gfdt_build_split.restype = ctypes.c_uint64
    l.gfdt_partition.argtypes = [vp, ctypes.c_uint32, ctypes.c_uint64, ctypes.c_int, vp]
    l.gfdt_partition.restype = None
    l.gfdt_group.argtypes = [vp, ctypes.c_size_t, vp]
    l.gfdt_group.restype = ctypes.c_size_t
    l.gfdt_ce_plan.argtypes = [vp, vp, vp, ctypes.c_size_t, vp]
    l.gfdt_ce_plan.restype = ctypes.c_size_t
    l.gfdt_committed_run.argtypes = [vp, ctypes.c_uint64, ctypes.c_uint32, ctypes.POINTER(ctypes.c_int)]
    l.gfdt_committed_run.restype = ctypes.c_uint32
    l.gfdt_gate_new.argtypes = [ctypes.c_uint64]
    l.gfdt_gate_new.restype = vp
    l.gfdt_gate_ready.argtypes = [vp, ctypes.c_uint32, ctypes.c_int, ctypes.c_int, ctypes.c_uint64]
    l.gfdt_gate_ready.restype = ctypes.c_int
    l.gfdt_gate_free.argtypes = [vp]
    l.gfdt_gate_free.restype = None
    u32p = ctypes.POINTER(ctypes.c_uint32)
    l.gfdt_account.argtypes = [ctypes.c_int, ctypes.c_int, vp, vp, ctypes.c_int, vp, vp, u32p, vp, ctypes.c_uint32,
                               u32p, u32p]
    l.gfdt_account.restype = None
    u64p = ctypes.POINTER(ctypes.c_uint64)
    l.gfdt_pages_mapped.argtypes = [ctypes.c_uint64, ctypes.c_uint64, u64p, u64p]
    l.gfdt_pages_mapped.restype = ctypes.c_int
    return l


def build(lib, src, dst, size):
    n = len(src)
    src, dst, size = (np.ascontiguousarray(x, dtype=np.uint64) for x in (src, dst, size))
    rows, misc = np.zeros(max(n, 1), ROW), np.zeros(max(n, 1), ROW)
    nr, nm = ctypes.c_uint32(), ctypes.c_uint32()
    total = lib.gfdt_build(src.ctypes.data, dst.ctypes.data, size.ctypes.data, n, rows.ctypes.data, ctypes.byref(nr),
                           misc.ctypes.data, ctypes.byref(nm))
    return rows[:nr.value].copy(), misc[:nm.value].copy(), total


def apply(spans, src_mem, dst_mem):
    for s, d, n in spans:
        dst_mem[int(d):int(d) + int(n)] = src_mem[int(s):int(s) + int(n)]


def random_entries(seed, n, src_bytes, dst_bytes):
    """Entries into a src space and non-overlapping dst slots: runs of contiguous aligned
    entries (merge candidates), misaligned ones, empty ones."""
    rng = np.random.default_rng(seed)
    src, dst, size = [], [], []
    d = 0
    while len(src) < n:
        kind = rng.integers(0, 4)
        if kind == 0:  # a run of k contiguous aligned entries
            k = int(rng.integers(2, 6))
            ln = int(rng.integers(1, 64)) * 16
            s = int(rng.integers(0, (src_bytes - k * ln) // 16)) * 16
            for j in range(k):
                src.append(s + j * ln); dst.append(d); size.append(ln); d += ln
        elif kind == 1:  # misaligned
            ln = int(rng.integers(1, 300))
            s = int(rng.integers(0, src_bytes - ln))
            d += int(rng.integers(0, 16))
            src.append(s); dst.append(d); size.append(ln); d += ln
        elif kind == 2:  # empty
            src.append(int(rng.integers(0, src_bytes))); dst.append(d); size.append(0)
        else:  # aligned, not contiguous with the previous one
            ln = int(rng.integers(1, 64)) * 16
            s = int(rng.integers(0, (src_bytes - ln) // 16)) * 16
            d = (d + 16 + 15) // 16 * 16
            src.append(s); dst.append(d); size.append(ln); d += ln
    assert d <= dst_bytes
    return np.array(src, np.uint64), np.array(dst, np.uint64), np.array(size, np.uint64)


@pytest.mark.parametrize("seed", range(6))
def test_table_replays_entries_exactly(lib, seed):
    src_bytes, dst_bytes = 1 << 16, 1 << 20
    s, d, z = random_entries(seed, 400, src_bytes, dst_bytes)
    rows, misc, total = build(lib, s, d, z)
    src_mem = np.frombuffer(np.random.default_rng(seed).bytes(src_bytes), np.uint8)
    want = np.zeros(dst_bytes, np.uint8)
    got = np.zeros(dst_bytes, np.uint8)
    apply(zip(s, d, z), src_mem, want)
    apply(((r["src"], r["dst"], r["len"]) for r in rows), src_mem, got)
    apply(((r["src"], r["dst"], r["len"]) for r in misc), src_mem, got)
    assert np.array_equal(got, want)
    # the stream: starts are the prefix sums of the aligned rows, every aligned field
    assert int(total) == int(rows["len"].sum())
    assert np.array_equal(rows["start"], np.concatenate([[0], np.cumsum(rows["len"])[:-1]]).astype(np.uint64))
    assert not ((rows["src"] | rows["dst"] | rows["len"]) & 15).any()
    assert (((misc["src"] | misc["dst"] | misc["len"]) & 15) != 0).all()
    # runs merge: rows are fewer than the aligned non-empty entries when runs exist
    aligned = ((s | d | z) & 15) == 0
    assert len(rows) < int((aligned & (z > 0)).sum())
    assert len(misc) == int((~aligned & (z > 0)).sum())


def test_merging_rules(lib):
    # contiguous in both src and dst: one row
    rows, misc, total = build(lib, [0, 4096, 8192], [0, 4096, 8192], [4096] * 3)
    assert len(rows) == 1 and rows[0]["len"] == 12288 and total == 12288
    # contiguous in src only: two rows
    rows, _, _ = build(lib, [0, 4096], [0, 8192], [4096, 4096])
    assert len(rows) == 2 and list(rows["start"]) == [0, 4096]
    # a misaligned entry in between breaks the run even when the next one continues
    rows, misc, _ = build(lib, [0, 4096, 4096], [0, 4096, 4096], [4096, 8, 4096])
    assert len(rows) == 2 and len(misc) == 1
    # empty entries are skipped and do not break a run
    rows, misc, _ = build(lib, [0, 99, 4096], [0, 77, 4096], [4096, 0, 4096])
    assert len(rows) == 1 and len(misc) == 0
    # nothing at all
    rows, misc, total = build(lib, [], [], [])
    assert len(rows) == 0 and len(misc) == 0 and total == 0


def test_copy_engine_split_repacks_the_stream(lib):
    s = np.arange(10, dtype=np.uint64) * np.uint64(1 << 20)
    d = np.arange(10, dtype=np.uint64) * np.uint64(1 << 20)
    z = np.array([16, 1 << 20, 32, 1 << 20, 48, 64, 1 << 19, 80, 96, 112], np.uint64)
    d[1::2] += np.uint64(4096)  # break contiguity so every entry is its own row
    rows, misc, taken = np.zeros(10, ROW), np.zeros(10, ROW), np.zeros(10, ROW)
    nr, nm, nt = ctypes.c_uint32(), ctypes.c_uint32(), ctypes.c_uint32()
    total = lib.gfdt_build_split(s.ctypes.data, d.ctypes.data, z.ctypes.data, 10, 1 << 19, rows.ctypes.data,
                                 ctypes.byref(nr), misc.ctypes.data, ctypes.byref(nm), taken.ctypes.data,
                                 ctypes.byref(nt))
    rows, taken = rows[:nr.value], taken[:nt.value]
    assert sorted(taken["len"].tolist()) == [1 << 19, 1 << 20, 1 << 20]
    assert int(total) == int(rows["len"].sum()) == 16 + 32 + 48 + 64 + 80 + 96 + 112
    assert np.array_equal(rows["start"], np.concatenate([[0], np.cumsum(rows["len"])[:-1]]).astype(np.uint64))


@pytest.mark.parametrize("grid", [1, 7, 64, 296])
def test_partition_first_rows(lib, grid):
    s, d, z = random_entries(11 + grid, 2000, 1 << 18, 1 << 24)
    rows, _, total = build(lib, s, d, z)
    per = max(4096, (int(total) + grid - 1) // grid // 4096 * 4096 + 4096)
    first = np.zeros(grid, np.uint32)
    lib.gfdt_partition(rows.ctypes.data, len(rows), per, grid, first.ctypes.data)
    ends = rows["start"] + rows["len"]
    for c in range(grid):
        target = c * per
        if target >= int(total):
            continue
        r = int(first[c])
        assert rows["start"][r] <= target < ends[r], f"CTA {c}"


def test_workload_tables_merge_adjacent_blocks(lib):
    """Config 1's 2x-stride layout never merges; a contiguous slice of the pool merges
    into one row."""
    w = wl.Workload("cfg1", pool_bytes=512 * 4096, dst_bytes=256 * 4096, num_tokens=256, token_size=4096,
                    kind="bytes", seed=1, stride=2 * 4096)
    e = w.entries(0, 1 << 30)
    rows, misc, total = build(lib, e["src"], e["dst"], e["size"])
    assert len(rows) == 256 and len(misc) == 0 and total == 256 * 4096
    n = 64
    rows, _, _ = build(lib, np.arange(n, dtype=np.uint64) * 4096, np.arange(n, dtype=np.uint64) * 4096 + (1 << 30),
                       [4096] * n)
    assert len(rows) == 1


CE = np.dtype([("dst", "<u8"), ("src", "<u8"), ("width", "<u8"), ("height", "<u8"), ("dpitch", "<u8"),
               ("spitch", "<u8")])


def group(lib, src, dst, size):
    n = len(src)
    runs = np.zeros(max(n, 1), ROW)
    runs["src"][:n], runs["dst"][:n], runs["len"][:n] = src, dst, size
    out = np.zeros(max(n, 1), CE)
    k = lib.gfdt_group(runs.ctypes.data, n, out.ctypes.data)
    return out[:k].copy()


def test_strided_runs_become_2d_copies(lib):
    n = 256
    # config 1: token i at slot 2i, gathered contiguously -> one copy of 256 rows
    c = group(lib, np.arange(n, dtype=np.uint64) * 8192, np.arange(n, dtype=np.uint64) * 4096 + (1 << 30), [4096] * n)
    assert len(c) == 1 and c[0]["height"] == n and c[0]["spitch"] == 8192 and c[0]["dpitch"] == 4096
    # two strided groups back to back, then a lone run of another length
    src = list(np.arange(8) * 1000 + 0) + list(np.arange(8) * 3000 + 10 ** 6) + [5 * 10 ** 6]
    dst = list(np.arange(8) * 600) + list(np.arange(8) * 600 + 10 ** 5) + [2 * 10 ** 5]
    size = [500] * 16 + [64]
    c = group(lib, src, dst, size)
    assert [int(x) for x in c["height"]] == [8, 8, 1]
    # descending sources, overlapping pitches and uneven steps are not grouped
    assert len(group(lib, [8000, 4000, 0], [0, 4096, 8192], [4096] * 3)) == 3
    assert len(group(lib, [0, 100, 200], [0, 4096, 8192], [4096] * 3)) == 3
    assert len(group(lib, [0, 8192, 20000], [0, 4096, 8192], [4096] * 3)) == 2


@pytest.mark.parametrize("seed", range(4))
def test_grouped_copies_replay_runs_exactly(lib, seed):
    rng = np.random.default_rng(seed)
    src, dst, size = [], [], []
    d = 0
    while len(src) < 300:
        k = int(rng.integers(1, 12))
        w = int(rng.integers(1, 200))
        sp = w + int(rng.integers(0, 100))
        s0 = int(rng.integers(0, 50000))
        for j in range(k):
            src.append(s0 + j * sp); dst.append(d); size.append(w); d += w + int(rng.integers(0, 3)) * 0
    src_mem = np.frombuffer(rng.bytes(200000), np.uint8)
    want, got = np.zeros(d + 1, np.uint8), np.zeros(d + 1, np.uint8)
    apply(zip(src, dst, size), src_mem, want)
    for c in group(lib, np.array(src, np.uint64), np.array(dst, np.uint64), np.array(size, np.uint64)):
        for r in range(int(c["height"])):
            s0, d0, w = int(c["src"]) + r * int(c["spitch"]), int(c["dst"]) + r * int(c["dpitch"]), int(c["width"])
            got[d0:d0 + w] = src_mem[s0:s0 + w]
    assert np.array_equal(got, want)


@pytest.mark.parametrize("seed", range(4))
def test_copy_engine_plan_replays_entries_exactly(lib, seed):
    """CopyEngineManager's plan (append_run + group_strided): continuing entries of any
    alignment merge, evenly strided runs group, empty entries vanish, and replaying the
    copies lands what copying the entries one by one lands."""
    rng = np.random.default_rng(100 + seed)
    src, dst, size = [], [], []
    d = 0
    while len(src) < 400:
        kind = int(rng.integers(0, 4))
        s0 = int(rng.integers(0, 100000))
        if kind == 0:  # continuing pieces of one span, ragged lengths
            for _ in range(int(rng.integers(2, 6))):
                n = int(rng.integers(1, 300))
                src.append(s0); dst.append(d); size.append(n); s0 += n; d += n
        elif kind == 1:  # evenly strided rows
            w = int(rng.integers(1, 400))
            sp, dp = w + int(rng.integers(0, 300)), w + int(rng.integers(1, 50))
            for j in range(int(rng.integers(2, 10))):
                src.append(s0 + j * sp); dst.append(d + j * dp); size.append(w)
            d += int(rng.integers(2, 10)) * dp + w
            d = max(d, dst[-1] + w)
        elif kind == 2:  # empty
            src.append(s0); dst.append(d); size.append(0)
        else:  # lone span
            n = int(rng.integers(1, 5000))
            d += int(rng.integers(1, 40))
            src.append(s0); dst.append(d); size.append(n); d += n
    src_mem = np.frombuffer(rng.bytes(110000), np.uint8)
    want, got = np.zeros(d + 1, np.uint8), np.zeros(d + 1, np.uint8)
    apply(zip(src, dst, size), src_mem, want)
    s_, d_, n_ = (np.array(x, np.uint64) for x in (src, dst, size))
    out = np.zeros(len(src), CE)
    k = lib.gfdt_ce_plan(s_.ctypes.data, d_.ctypes.data, n_.ctypes.data, len(src), out.ctypes.data)
    assert 0 < k < sum(1 for x in size if x)  # some merging and grouping happened
    for c in out[:k]:
        assert c["width"] > 0 and (c["height"] == 1 or (c["spitch"] >= c["width"] and c["dpitch"] >= c["width"]))
        for r in range(int(c["height"])):
            s0, d0, w = int(c["src"]) + r * int(c["spitch"]), int(c["dst"]) + r * int(c["dpitch"]), int(c["width"])
            got[d0:d0 + w] = src_mem[s0:s0 + w]
    assert np.array_equal(got, want)


# ---- ring drain (drain.h) ----

from gfd_b200 import DESCRIPTOR_DTYPE, QUEUE_BYTES, QUEUE_SIZE  # noqa: E402


def ring():
    raw = np.zeros(QUEUE_BYTES + 64, np.uint8)
    off = (-raw.ctypes.data) % 64  # Descriptor is 64-byte aligned
    buf = raw[off:off + QUEUE_BYTES]
    return raw, buf, buf[:QUEUE_SIZE * 64].view(DESCRIPTOR_DTYPE)


def commit(entries, slots, flags=0):
    for s_ in slots:
        entries["flags"][s_ % QUEUE_SIZE] = flags
        entries["seq"][s_ % QUEUE_SIZE] = s_ + 1


def run(lib, buf, nxt, max_n=8192):
    u = ctypes.c_int()
    n = lib.gfdt_committed_run(buf.ctypes.data, nxt, max_n, ctypes.byref(u))
    return n, bool(u.value)


def test_committed_run_prefix_wrap_and_urgency(lib):
    raw, buf, e = ring()
    assert run(lib, buf, 0) == (0, False)
    commit(e, range(0, 10))
    commit(e, range(11, 20))  # slot 10 not committed yet: the run stops before it
    assert run(lib, buf, 0) == (10, False)
    commit(e, [10])
    assert run(lib, buf, 0) == (20, False)
    assert run(lib, buf, 0, max_n=7) == (7, False)
    # a stale marker from the previous lap of the ring is not a commit
    base = QUEUE_SIZE - 5
    commit(e, range(base, base + 5))  # the last five slots of lap 0
    e["seq"][0] = 1  # slot 0 still holds lap 0's marker for slot 0
    assert run(lib, buf, base) == (5, False)
    commit(e, range(QUEUE_SIZE, QUEUE_SIZE + 3))  # slots 0..2 of lap 1
    n, urgent = run(lib, buf, base)
    assert n == 8 and not urgent
    commit(e, [QUEUE_SIZE + 3], flags=1)  # FLAG_LAST_IN_BATCH
    assert run(lib, buf, base) == (9, True)


def test_batch_gate_follows_the_reference_rule(lib):
    g = lib.gfdt_gate_new(20000)
    try:
        assert lib.gfdt_gate_ready(g, 0, 0, 0, 0) == 0          # nothing committed
        assert lib.gfdt_gate_ready(g, 100, 0, 0, 1000) == 0     # small run: wait for it to settle
        assert lib.gfdt_gate_ready(g, 100, 0, 0, 15000) == 0    # unchanged for 14 us
        assert lib.gfdt_gate_ready(g, 120, 0, 0, 16000) == 0    # grew: the clock restarts
        assert lib.gfdt_gate_ready(g, 120, 0, 0, 30000) == 0
        assert lib.gfdt_gate_ready(g, 120, 0, 0, 36001) == 1    # quiet for 20 us: go
        assert lib.gfdt_gate_ready(g, 5, 1, 0, 36002) == 1      # a boundary flag: go at once
        assert lib.gfdt_gate_ready(g, 1024, 0, 0, 36003) == 1   # BATCH_THRESHOLD_SMALL reached
        assert lib.gfdt_gate_ready(g, 3, 0, 1, 36004) == 1      # forced (stop, explicit poll)
    finally:
        lib.gfdt_gate_free(g)


def account(lib, tiled, sg, flags, user, max_lists=512):
    n = len(flags)
    flags = np.ascontiguousarray(flags, np.uint32)
    user = np.ascontiguousarray(user, np.uint64)
    tile_id, tile_count = np.zeros(1024, np.uint16), np.zeros(1024, np.uint32)
    list_id = np.zeros(512, np.uint16)
    nt, nl, landed = ctypes.c_uint32(), ctypes.c_uint32(), ctypes.c_uint32()
    lib.gfdt_account(int(tiled), int(sg), flags.ctypes.data, user.ctypes.data, n, tile_id.ctypes.data,
                     tile_count.ctypes.data, ctypes.byref(nt), list_id.ctypes.data, max_lists, ctypes.byref(nl),
                     ctypes.byref(landed))
    assert nt.value != 0xffffffff, "tile scratch not cleared"
    return (dict(zip(tile_id[:nt.value].tolist(), tile_count[:nt.value].tolist())), list_id[:nl.value].tolist(),
            landed.value)


def test_drain_accounting_tiles_and_lists(lib):
    rng = np.random.default_rng(3)
    tiles = rng.integers(0, 1100, 3000)  # ids >= 1024 are beyond MAX_TILES and not counted
    user = (tiles.astype(np.uint64) << np.uint64(32)) | np.arange(3000, dtype=np.uint64)
    counts, lists, landed = account(lib, True, False, np.zeros(3000), user)
    want = {int(t): int((tiles == t).sum()) for t in np.unique(tiles) if t < 1024}
    assert counts == want and lists == [] and landed == 0
    # SG: a list lands at its FLAG_LAST_IN_TILE descriptor; ids >= 512 are not signalled
    ids = np.array([3, 3, 3, 7, 7, 600, 9], np.uint64)
    flags = np.array([0, 0, 4, 0, 4, 4, 4], np.uint32)
    counts, lists, landed = account(lib, False, True, flags, ids << np.uint64(32))
    assert counts == {} and lists == [3, 7, 9] and landed == 3
    # more landed lists than the table holds: all counted, the first ones recorded
    counts, lists, landed = account(lib, False, True, np.full(10, 4), np.arange(10, dtype=np.uint64) << np.uint64(32),
                                    max_lists=4)
    assert lists == [0, 1, 2, 3] and landed == 10


def test_pageable_ranges_need_every_page_mapped(lib):
    """The check that guards pageable sources (GATHER_PAGEABLE, gfd_b200/csrc/host_mem.h):
    a range is accepted only when every page it covers is mapped, so a hole is found on the
    host and never handed to the driver's staging copy; empty and wrapping ranges fail."""
    libc = ctypes.CDLL(None, use_errno=True)
    libc.mmap.restype = ctypes.c_void_p
    libc.mmap.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_long]
    libc.munmap.argtypes = [ctypes.c_void_p, ctypes.c_size_t]
    pg = os.sysconf("SC_PAGESIZE")
    a = libc.mmap(None, 4 * pg, 3, 0x22, -1, 0)  # PROT_READ|WRITE, MAP_PRIVATE|ANONYMOUS
    assert a not in (None, ctypes.c_void_p(-1).value)
    assert libc.munmap(a + 2 * pg, pg) == 0  # page 2 becomes a hole
    lo, hi = ctypes.c_uint64(), ctypes.c_uint64()

    def mapped(p, n):
        return lib.gfdt_pages_mapped(p, n, ctypes.byref(lo), ctypes.byref(hi)) == 1

    try:
        assert mapped(a + 100, 50) and (lo.value, hi.value) == (a, a + pg)
        assert mapped(a + pg - 8, 16) and (lo.value, hi.value) == (a, a + 2 * pg)  # two mapped pages
        assert mapped(a + 3 * pg, pg) and (lo.value, hi.value) == (a + 3 * pg, a + 4 * pg)
        assert not mapped(a + 2 * pg - 8, 16)  # runs into the hole
        assert not mapped(a + 2 * pg + 1, 1)  # inside the hole
        assert not mapped(a, 4 * pg)  # spans it
        assert not mapped(a, 0)
        assert not mapped(2**64 - 16, 32)  # wraps
    finally:
        libc.munmap(a, 2 * pg)
        libc.munmap(a + 3 * pg, pg)
