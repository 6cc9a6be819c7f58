"""Direct-submit parity: the sm_100a SM-pull gather against the CPU oracle.

Every case calls the C ABI (gfd_gather_sync / gfd_gather / gfd_gather_device)
through ctypes and compares the destination bytes with the oracle's output for the
same seeded inputs (bit-exact), or -- at full benchmark sizes -- per-token checksums
against checksums of the source tokens.
"""
import ctypes

import numpy as np
import pytest

import gfd_b200
from gfd_b200 import GFD_ERR_INVALID, GFD_OK, entries_array
from gfd_b200 import workloads as wl
from tests.golden.cases import CASES, ODD_CASES, build_case, checksum, oracle, oracle_gather

pytestmark = pytest.mark.gpu


def torch_u8(n):
    """A zeroed device buffer, ready before the library's own streams touch it (torch
    zeroes it on its stream; the library's calls run on other streams)."""
    import torch
    t = torch.zeros(max(n, 1), dtype=torch.uint8, device="cuda")
    torch.cuda.synchronize()
    return t


def to_np(t):
    return t.cpu().numpy()


def run_case(ctx, spec, flags=0):
    """Gathers a golden-recipe case from a pinned pool; returns (gpu bytes, oracle bytes)."""
    probe_pool, entries, out_len = build_case(spec)
    pool = ctx.pool(max(probe_pool.nbytes, 1))
    pool_arr = pool.array()[:probe_pool.nbytes]
    _, entries, out_len = build_case(spec, pool=pool_arr)
    dst = torch_u8(out_len)
    e = entries.copy()
    e["dst"] += np.uint64(dst.data_ptr())
    ctx.gather_sync(e, flags=flags)
    got = to_np(dst)[:out_len]
    want = np.zeros(out_len, np.uint8)
    eo = entries.copy()
    eo["dst"] += np.uint64(want.ctypes.data)
    assert oracle_gather(want, want.ctypes.data, eo) == -1
    pool.free()
    return got, want


@pytest.mark.parametrize("flags", [gfd_b200.GATHER_FORCE_PULL, gfd_b200.GATHER_DEFAULT, gfd_b200.GATHER_BULK_STAGE],
                         ids=["pull", "default", "bulk"])
@pytest.mark.parametrize("spec", CASES + ODD_CASES, ids=[c["name"] for c in CASES + ODD_CASES])
def test_golden_and_odd_cases(gpu_ctx, spec, flags):
    got, want = run_case(gpu_ctx, spec, flags=flags)
    assert np.array_equal(got, want)


@pytest.mark.parametrize("spec", CASES[:3], ids=[c["name"] for c in CASES[:3]])
def test_copy_engine_path_matches(gpu_ctx, spec):
    got, want = run_case(gpu_ctx, spec, flags=gfd_b200.GATHER_FORCE_CE)
    assert np.array_equal(got, want)


@pytest.mark.parametrize("n,size,stride", [(256, 4096, 8192), (2048, 16384, 32768), (1000, 100, 300)])
def test_copy_engine_strided_layouts(gpu_ctx, n, size, stride):
    """Evenly strided tokens on the copy-engine path go out as 2D copies (at most one per
    copy engine), and land exactly; a gap in the stride starts a new copy."""
    import torch
    pool = gpu_ctx.pool(n * stride + stride)
    wl.fill_bytes(pool.ptr, pool.nbytes, n + size)
    dst = torch.zeros(n * size, dtype=torch.uint8, device="cuda")
    torch.cuda.synchronize()
    src = np.arange(n, dtype=np.uint64) * np.uint64(stride)
    src[n // 2:] += np.uint64(stride)  # second half one slot further: two strided groups
    e = entries_array(np.uint64(dst.data_ptr()) + np.arange(n, dtype=np.uint64) * np.uint64(size),
                      np.uint64(pool.ptr) + src, size)
    before = gpu_ctx.stats()["ce_copies"]
    gpu_ctx.gather_sync(e, gfd_b200.GATHER_FORCE_CE)
    copies = gpu_ctx.stats()["ce_copies"] - before
    assert copies <= 6, copies  # two groups, each split by rows over the three copy engines when large
    want = np.zeros(n * size, np.uint8)
    host = pool.array()
    for i in range(n):
        want[i * size:(i + 1) * size] = host[int(src[i]):int(src[i]) + size]
    assert np.array_equal(to_np(dst), want)
    # the same layout scattered back (device -> host) through the copy engines
    back = gpu_ctx.pool(n * stride + stride)
    arr = back.array()
    arr[:] = 0
    es = entries_array(np.uint64(back.ptr) + src, np.uint64(dst.data_ptr()) +
                       np.arange(n, dtype=np.uint64) * np.uint64(size), size)
    gpu_ctx.scatter_sync(es, gfd_b200.GATHER_FORCE_CE)
    for i in range(0, n, max(1, n // 37)):
        assert np.array_equal(arr[int(src[i]):int(src[i]) + size], host[int(src[i]):int(src[i]) + size])
    back.free()
    pool.free()


def test_default_path_picks_copy_engine_for_strided_large_rows(gpu_ctx):
    """The default path sends an evenly strided layout of >= 16 KiB rows to the copy
    engines (2D copies) and keeps everything else on the SM pull; GATHER_FORCE_PULL
    keeps it on the pull."""
    import torch
    n, size = 512, 16384
    pool = gpu_ctx.pool(2 * n * size)
    wl.fill_bytes(pool.ptr, pool.nbytes, 5)
    dst = torch.zeros(n * size, dtype=torch.uint8, device="cuda")
    torch.cuda.synchronize()
    d = np.uint64(dst.data_ptr()) + np.arange(n, dtype=np.uint64) * np.uint64(size)
    strided = entries_array(d, np.uint64(pool.ptr) + np.arange(n, dtype=np.uint64) * np.uint64(2 * size), size)
    shuffled = entries_array(d, np.uint64(pool.ptr) + wl.permutation(2 * n, 9)[:n].astype(np.uint64) *
                             np.uint64(size), size)
    host = pool.array()

    def check(e):
        want = np.zeros(n * size, np.uint8)
        for i in range(n):
            s0 = int(e["src"][i]) - pool.ptr
            want[i * size:(i + 1) * size] = host[s0:s0 + size]
        assert np.array_equal(to_np(dst), want)

    for e, flags, expect_ce in ((strided, 0, True), (strided, gfd_b200.GATHER_FORCE_PULL, False),
                                (shuffled, 0, False)):
        dst.zero_()
        torch.cuda.synchronize()
        s0 = gpu_ctx.stats()
        gpu_ctx.gather_sync(e, flags)
        s1 = gpu_ctx.stats()
        used_ce = s1["ce_copies"] > s0["ce_copies"]
        used_pull = s1["pull_launches"] > s0["pull_launches"]
        assert used_ce == expect_ce and used_pull == (not expect_ce), (flags, used_ce, used_pull)
        check(e)
    pool.free()


@pytest.mark.parametrize("n,kind", [(1184, "uniform"), (1185, "uniform"), (2048, "uniform"), (2300, "ragged")])
def test_mid_size_calls_bit_exact(gpu_ctx, n, kind):
    """Host-entry pulls between one and two CTAs' worth of pieces per SM (the grid goes
    from one CTA per SM to two per SM with equal bytes): shuffled 4 KiB tokens around the
    switch (1184 / 1185 tokens on 148 SMs) and ragged 16-byte-multiple tokens mixed with
    misaligned ones, against the oracle."""
    import torch
    rng = np.random.default_rng(n)
    if kind == "uniform":
        sizes = np.full(n, 4096, np.uint64)
    else:
        sizes = (rng.integers(1, 513, size=n) * 16).astype(np.uint64)
        odd = rng.choice(n, size=n // 20, replace=False)
        sizes[odd] = rng.integers(1, 5000, size=len(odd)).astype(np.uint64)
    slot = 8192
    pool = gpu_ctx.pool(2 * n * slot)
    wl.fill_bytes(pool.ptr, pool.nbytes, 40 + n)
    order = wl.permutation(2 * n, n)[:n].astype(np.uint64)
    src = np.uint64(pool.ptr) + order * np.uint64(slot) + (sizes % np.uint64(16) != 0) * np.uint64(3)
    padded = (sizes + np.uint64(15)) // np.uint64(16) * np.uint64(16)  # every token starts 16-byte aligned
    offs = np.concatenate([[0], np.cumsum(padded)[:-1]]).astype(np.uint64)
    total = int(padded.sum())
    dst = torch.zeros(total, dtype=torch.uint8, device="cuda")
    torch.cuda.synchronize()
    e = entries_array(np.uint64(dst.data_ptr()) + offs, src, sizes)
    gpu_ctx.gather_sync(e, gfd_b200.GATHER_FORCE_PULL)
    want = np.zeros(total, np.uint8)
    eo = e.copy()
    eo["dst"] = np.uint64(want.ctypes.data) + offs
    assert oracle_gather(want, want.ctypes.data, eo) == -1
    assert np.array_equal(to_np(dst), want)
    pool.free()


def test_alignment_matrix(gpu_ctx):
    """Every src/dst misalignment and size class lands byte-exact (head, body, tail paths)."""
    pool = gpu_ctx.pool(1 << 20)
    src = pool.array()
    wl.fill_bytes(pool.ptr, pool.nbytes, 99)
    sizes = [1, 2, 15, 16, 17, 31, 100, 511, 512, 4095, 4096, 4097, 65536 + 3]
    soffs = [0, 1, 3, 4, 8, 12, 15]
    doffs = [0, 1, 4, 8, 15]
    dst_list, src_list, size_list = [], [], []
    cursor_s, cursor_d = 0, 0
    for s in sizes:
        for so in soffs:
            for do in doffs:
                cursor_s = (cursor_s + 64) // 64 * 64 + so
                cursor_d = (cursor_d + 64) // 64 * 64 + do
                if cursor_s + s > src.nbytes:
                    cursor_s = so
                src_list.append(cursor_s)
                dst_list.append(cursor_d)
                size_list.append(s)
                cursor_s += s
                cursor_d += s
    out_len = cursor_d + 64
    dst = torch_u8(out_len)
    e = entries_array(np.array(dst_list, np.uint64) + np.uint64(dst.data_ptr()),
                      np.array(src_list, np.uint64) + np.uint64(pool.ptr), np.array(size_list, np.uint64))
    gpu_ctx.gather_sync(e)
    want = np.zeros(out_len, np.uint8)
    eo = entries_array(np.array(dst_list, np.uint64) + np.uint64(want.ctypes.data),
                       np.array(src_list, np.uint64) + np.uint64(pool.ptr), np.array(size_list, np.uint64))
    oracle_gather(want, want.ctypes.data, eo)
    assert np.array_equal(to_np(dst)[:out_len], want)
    pool.free()


@pytest.mark.parametrize("flags", [gfd_b200.GATHER_FORCE_PULL, gfd_b200.GATHER_DEFAULT], ids=["pull", "default"])
@pytest.mark.parametrize("n_aligned,n_odd,size", [(16, 0, 4096), (12, 4, 4096), (17, 0, 4096), (0, 16, 1000),
                                                  (1, 0, 16), (3, 2, 65536), (8, 9, 2048)])
def test_small_calls_inline_tables(gpu_ctx, n_aligned, n_odd, size, flags):
    """Calls small enough for the row table to travel in the kernel parameters (at most
    16 stream + misc rows), at and just past that limit, with misaligned rows mixed in
    (forced onto the SM pull; with default flags the evenly strided ones may take the
    copy engines instead)."""
    pool = gpu_ctx.pool(4 << 20)
    wl.fill_bytes(pool.ptr, pool.nbytes, n_aligned * 31 + n_odd)
    offs, douts, sizes = [], [], []
    cur_d = 0
    for i in range(n_aligned + n_odd):
        odd = i >= n_aligned
        offs.append(i * 2 * (size + 64) + (7 if odd else 0))  # 2x stride, odd rows misaligned
        sz = size + (3 if odd else 0)
        douts.append(cur_d + (5 if odd else 0))
        sizes.append(sz)
        cur_d = (douts[-1] + sz + 63) // 64 * 64
    out_len = cur_d + 64
    dst = torch_u8(out_len)
    e = entries_array(np.array(douts, np.uint64) + np.uint64(dst.data_ptr()),
                      np.array(offs, np.uint64) + np.uint64(pool.ptr), np.array(sizes, np.uint64))
    gpu_ctx.gather_sync(e, flags)
    want = np.zeros(out_len, np.uint8)
    eo = e.copy()
    eo["dst"] = np.array(douts, np.uint64) + np.uint64(want.ctypes.data)
    assert oracle_gather(want, want.ctypes.data, eo) == -1
    assert np.array_equal(to_np(dst)[:out_len], want)
    pool.free()


def test_contiguous_runs_merge_and_stay_exact(gpu_ctx):
    """Entries that continue each other in src and dst (merged into one row)."""
    pool = gpu_ctx.pool(8 << 20)
    wl.fill_bytes(pool.ptr, pool.nbytes, 5)
    rng = np.random.default_rng(5)
    sizes = (rng.integers(1, 64, 3000) * 16).astype(np.uint64)
    # runs of 1..8 contiguous entries, runs separated by gaps in src
    src = np.zeros_like(sizes)
    cur = 0
    for i, s in enumerate(sizes):
        if rng.random() < 0.3:
            cur += 4096
        src[i] = cur
        cur += int(s)
    assert cur < pool.nbytes
    dst_off = np.concatenate([[0], np.cumsum(sizes)[:-1]]).astype(np.uint64)
    total = int(sizes.sum())
    dst = torch_u8(total)
    e = entries_array(dst_off + np.uint64(dst.data_ptr()), src + np.uint64(pool.ptr), sizes)
    gpu_ctx.gather_sync(e)
    want = np.zeros(total, np.uint8)
    oracle_gather(want, want.ctypes.data, entries_array(dst_off + np.uint64(want.ctypes.data),
                                                        src + np.uint64(pool.ptr), sizes))
    assert np.array_equal(to_np(dst), want)
    pool.free()


def test_scattered_destinations(gpu_ctx):
    """dst not contiguous (reverse order, gaps): the reference's per-entry CE branch."""
    pool = gpu_ctx.pool(4 << 20)
    wl.fill_bytes(pool.ptr, pool.nbytes, 8)
    n, size = 300, 4096
    dst_off = (np.arange(n)[::-1] * 2 * size).astype(np.uint64)
    src_off = (np.arange(n) * 3 * size % (pool.nbytes - size)).astype(np.uint64)
    out_len = 2 * n * size
    dst = torch_u8(out_len)
    gpu_ctx.gather_sync(entries_array(dst_off + np.uint64(dst.data_ptr()), src_off + np.uint64(pool.ptr), size))
    want = np.zeros(out_len, np.uint8)
    oracle_gather(want, want.ctypes.data,
                  entries_array(dst_off + np.uint64(want.ctypes.data), src_off + np.uint64(pool.ptr), size))
    assert np.array_equal(to_np(dst), want)
    pool.free()


def test_empty_and_zero_size(gpu_ctx):
    dst = torch_u8(4096)
    assert gpu_ctx.gather_sync_rc(np.zeros(0, gfd_b200.SG_ENTRY_DTYPE)) == GFD_OK
    pool = gpu_ctx.pool(4096)
    pool.array()[:] = 7
    e = entries_array([dst.data_ptr(), dst.data_ptr() + 16], [pool.ptr, pool.ptr], [0, 16])
    gpu_ctx.gather_sync(e)
    got = to_np(dst)
    assert np.all(got[16:32] == 7) and not got[:16].any() and not got[32:].any()
    pool.free()


def test_validation_rejects_bad_entries(gpu_ctx):
    import torch
    torch.cuda.empty_cache()  # the 64 MiB tensor below gets its own allocation
    dst = torch_u8(64 << 20)
    pool = gpu_ctx.pool(8 << 20)
    pageable = np.ones(4096, np.uint8)
    good = entries_array([dst.data_ptr()], [pool.ptr], [4096])
    # pageable source
    rc = gpu_ctx.gather_sync_rc(np.concatenate([good, entries_array([dst.data_ptr()], [pageable.ctypes.data], [4096])]))
    assert rc == GFD_ERR_INVALID and "pinned" in gpu_ctx.last_error()
    # destination running past the end of its device allocation
    rc = gpu_ctx.gather_sync_rc(entries_array([dst.data_ptr() + (64 << 20) - 64], [pool.ptr], [4 << 20]))
    assert rc == GFD_ERR_INVALID and "device allocation" in gpu_ctx.last_error()
    # destination in host memory
    rc = gpu_ctx.gather_sync_rc(entries_array([pageable.ctypes.data], [pool.ptr], [64]))
    assert rc == GFD_ERR_INVALID
    # source running past the pool
    rc = gpu_ctx.gather_sync_rc(entries_array([dst.data_ptr()], [pool.ptr + pool.nbytes - 64], [128]))
    assert rc == GFD_ERR_INVALID
    assert not to_np(dst).any(), "a rejected call must not copy anything"
    assert gpu_ctx.stats()["rejected"] >= 4
    pool.free()


def _libc_mmap():
    libc = ctypes.CDLL(None, use_errno=True)
    libc.mmap.restype = ctypes.c_void_p
    libc.mmap.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_long]
    libc.munmap.argtypes = [ctypes.c_void_p, ctypes.c_size_t]
    libc.munmap.restype = ctypes.c_int
    return libc


@pytest.mark.parametrize("flags", [0, gfd_b200.GATHER_FORCE_PULL], ids=["default", "pull"])
def test_pageable_sources_with_flag(gpu_ctx, flags):
    """GATHER_PAGEABLE: entries from pageable numpy memory (copy engine) and from a pinned
    pool (SM pull) in one call, odd sizes and continuing runs included, land exactly as the
    oracle's gather of the same entries, through the sync and the async entry point."""
    import torch
    rng = np.random.default_rng(23)
    pinned = gpu_ctx.pool(8 << 20)
    pinned.array()[:] = rng.integers(0, 256, 8 << 20, dtype=np.uint8)
    heap = rng.integers(0, 256, 8 << 20, dtype=np.uint8)  # ordinary (pageable) numpy memory
    srcs, sizes = [], []
    for i in range(400):
        n = int(rng.integers(1, 9000))
        base, nb = (heap.ctypes.data, heap.nbytes) if i % 3 else (pinned.ptr, pinned.nbytes)
        s = int(rng.integers(0, nb - 2 * n))
        srcs.append(base + s)
        sizes.append(n)
        if i % 7 == 2:  # the next bytes of the same source: merged into one run
            srcs.append(base + s + n)
            sizes.append(n)
    sizes = np.array(sizes, np.uint64)
    offs = np.concatenate([[0], np.cumsum(sizes)[:-1]]).astype(np.uint64)
    total = int(sizes.sum())
    want = np.zeros(total, np.uint8)
    assert oracle_gather(want, want.ctypes.data, entries_array(offs + np.uint64(want.ctypes.data), srcs, sizes)) == -1
    dst = torch_u8(total)
    e = entries_array(offs + np.uint64(dst.data_ptr()), srcs, sizes)
    assert gpu_ctx.gather_sync_rc(e, flags) == GFD_ERR_INVALID  # without the flag: pinned only
    # the flag relies on the source check, so it is refused together with TRUSTED
    assert gpu_ctx.gather_sync_rc(e, flags | gfd_b200.GATHER_PAGEABLE | gfd_b200.GATHER_TRUSTED) == GFD_ERR_INVALID
    assert not to_np(dst).any()
    ce0 = gpu_ctx.stats()["ce_copies"]
    gpu_ctx.gather_sync(e, flags | gfd_b200.GATHER_PAGEABLE)
    assert np.array_equal(to_np(dst)[:total], want)
    assert gpu_ctx.stats()["ce_copies"] > ce0
    dst.zero_()
    torch.cuda.synchronize()  # the fill runs on torch's stream, the gather on another
    s = torch.cuda.Stream()
    assert gpu_ctx.gather(e, s.cuda_stream, flags | gfd_b200.GATHER_PAGEABLE) == GFD_OK
    s.synchronize()
    assert np.array_equal(to_np(dst)[:total], want)
    pinned.free()


def test_pageable_flag_still_rejects_unmapped_and_device_sources(gpu_ctx):
    """With GATHER_PAGEABLE a source must still be mapped host memory: a range that runs
    into an unmapped page, and device memory as a source, are rejected before anything is
    copied (the hole is found on the host, so nothing ever reads it)."""
    import os
    libc = _libc_mmap()
    pg = os.sysconf("SC_PAGESIZE")
    a = libc.mmap(None, 3 * pg, 3, 0x22, -1, 0)  # PROT_READ|WRITE, MAP_PRIVATE|ANONYMOUS
    assert a not in (None, ctypes.c_void_p(-1).value)
    ctypes.memset(a, 5, 3 * pg)
    assert libc.munmap(a + pg, pg) == 0  # a hole in the middle
    try:
        dst = torch_u8(1 << 20)
        ok = entries_array([dst.data_ptr()], [a + 16], [64])
        assert gpu_ctx.gather_sync_rc(ok, gfd_b200.GATHER_PAGEABLE) == GFD_OK
        assert np.all(to_np(dst)[:64] == 5)
        dst.zero_()
        for src, n in [(a + pg - 32, 64), (a + pg + 8, 16), (a + 2 * pg - 8, 16)]:
            bad = np.concatenate([ok, entries_array([dst.data_ptr() + 4096], [src], [n])])
            assert gpu_ctx.gather_sync_rc(bad, gfd_b200.GATHER_PAGEABLE) == GFD_ERR_INVALID
            assert "pageable" in gpu_ctx.last_error()
        dev_src = torch_u8(4096)
        bad = entries_array([dst.data_ptr()], [dev_src.data_ptr()], [64])
        assert gpu_ctx.gather_sync_rc(bad, gfd_b200.GATHER_PAGEABLE) == GFD_ERR_INVALID
        assert not to_np(dst).any(), "a rejected call must not copy anything"
    finally:
        libc.munmap(a, pg)
        libc.munmap(a + 2 * pg, pg)


def test_async_gather_on_torch_stream(gpu_ctx):
    import torch
    spec = CASES[4]
    probe, entries, out_len = build_case(spec)
    pool = gpu_ctx.pool(probe.nbytes)
    _, entries, out_len = build_case(spec, pool=pool.array()[:probe.nbytes])
    s = torch.cuda.Stream()
    outs = []
    for k in range(6):  # more calls than staging slots
        dst = torch_u8(out_len)
        e = entries.copy()
        e["dst"] += np.uint64(dst.data_ptr())
        assert gpu_ctx.gather(e, stream=s.cuda_stream) == GFD_OK
        outs.append(dst)
    s.synchronize()
    want = np.zeros(out_len, np.uint8)
    eo = entries.copy()
    eo["dst"] += np.uint64(want.ctypes.data)
    oracle_gather(want, want.ctypes.data, eo)
    for d in outs:
        assert np.array_equal(to_np(d), want)
    pool.free()


@pytest.mark.parametrize("n,seed", [(4096, 1), (4097, 2), (12288, 3), (20000, 4)])
def test_gather_device_long_lists(gpu_ctx, n, seed):
    """Lists longer than one 4096-entry plan tile (multi-CTA plan): contiguous runs that
    cross tile boundaries, misaligned entries and rejected entries mixed in; every
    landed byte against the oracle, the first rejected index reported."""
    import torch
    pool = gpu_ctx.pool(64 << 20)
    wl.fill_bytes(pool.ptr, pool.nbytes, seed)
    rng = np.random.default_rng(seed)
    sizes = rng.choice([16, 64, 512, 1024, 4096, 48, 5], size=n).astype(np.uint64)
    src = np.zeros(n, np.uint64)
    cur = 0
    for i in range(n):
        # long contiguous runs (mean ~300 entries) so that many of them span tile edges;
        # one run is forced to continue across each tile boundary
        if rng.random() < 1.0 / 300 and (i % 4096) != 0:
            cur += int(rng.integers(1, 64)) * 16
        src[i] = cur
        cur += int(sizes[i])
    assert cur < pool.nbytes
    dst_off = np.concatenate([[0], np.cumsum(sizes)[:-1]]).astype(np.uint64)
    total = int(sizes.sum())
    dst = torch_u8(total + 4096)
    e = entries_array(dst_off + np.uint64(dst.data_ptr()), src + np.uint64(pool.ptr), sizes)
    bad = sorted(rng.choice(n, 3, replace=False).tolist())
    for b in bad:  # outside the destination window: skipped and reported
        e["dst"][b] = np.uint64(dst.data_ptr() + total + 4096 + 64)
    d_e = torch.from_numpy(e.view(np.uint8).copy()).cuda()
    gpu_ctx.gather_device(d_e.data_ptr(), n, dst.data_ptr(), total + 4096)
    rc, first_bad = gpu_ctx.gather_device_status()
    assert rc == GFD_ERR_INVALID and first_bad == bad[0]
    keep = np.ones(n, bool)
    keep[bad] = False
    want = np.zeros(total + 4096, np.uint8)
    eo = entries_array(dst_off[keep] + np.uint64(want.ctypes.data), src[keep] + np.uint64(pool.ptr), sizes[keep])
    assert oracle_gather(want, want.ctypes.data, eo) == -1
    assert np.array_equal(to_np(dst), want)
    pool.free()


def test_gather_device_entries(gpu_ctx):
    """Entry list resident in device memory: GPU validation + ballot/scan run merging."""
    import torch
    pool = gpu_ctx.pool(16 << 20)
    wl.fill_bytes(pool.ptr, pool.nbytes, 21)
    rng = np.random.default_rng(21)
    n = 5000
    sizes = rng.choice([16, 48, 512, 4096, 4100, 7, 1000], size=n).astype(np.uint64)
    src = np.zeros(n, np.uint64)
    cur = 0
    for i in range(n):
        if rng.random() < 0.5:
            cur += int(rng.integers(1, 200)) * 16
        src[i] = cur
        cur += int(sizes[i])
    assert cur < pool.nbytes
    dst_off = np.concatenate([[0], np.cumsum(sizes)[:-1]]).astype(np.uint64)
    total = int(sizes.sum())
    dst = torch_u8(total)
    e = entries_array(dst_off + np.uint64(dst.data_ptr()), src + np.uint64(pool.ptr), sizes)
    d_e = torch.from_numpy(e.view(np.uint8).copy()).cuda()
    gpu_ctx.gather_device(d_e.data_ptr(), n, dst.data_ptr(), total)
    rc, bad = gpu_ctx.gather_device_status()
    assert rc == GFD_OK and bad == -1
    want = np.zeros(total, np.uint8)
    oracle_gather(want, want.ctypes.data, entries_array(dst_off + np.uint64(want.ctypes.data),
                                                        src + np.uint64(pool.ptr), sizes))
    assert np.array_equal(to_np(dst), want)

    # an entry outside the dst window is skipped and reported; the rest still lands
    e2 = e.copy()
    e2["dst"][17] = np.uint64(dst.data_ptr() + total)  # past the window
    dst.zero_()
    d_e2 = torch.from_numpy(e2.view(np.uint8).copy()).cuda()
    gpu_ctx.gather_device(d_e2.data_ptr(), n, dst.data_ptr(), total)
    rc, bad = gpu_ctx.gather_device_status()
    assert rc == GFD_ERR_INVALID and bad == 17
    got = to_np(dst)
    d17, s17 = int(dst_off[17]), int(sizes[17])
    mask = np.ones(total, bool)
    mask[d17:d17 + s17] = False
    assert np.array_equal(got[mask], want[mask])
    pool.free()


def _source_token_checksums(entries):
    per = np.zeros(len(entries), np.uint64)
    e = np.ascontiguousarray(entries)
    oracle().gfd_oracle_checksum_entries(e.ctypes.data, len(e), per.ctypes.data)
    return per


def _dst_token_checksums(dst_np, size, n):
    per = np.zeros(n, np.uint64)
    oracle().gfd_oracle_checksum_records(dst_np.ctypes.data, size, n, per.ctypes.data)
    return per


def _oracle_dst(entries, dst_ptr, total):
    """The oracle's destination bytes for entries aimed at [dst_ptr, dst_ptr + total)."""
    want = np.zeros(total, np.uint8)
    eo = entries.copy()
    eo["dst"] = eo["dst"] - np.uint64(dst_ptr) + np.uint64(want.ctypes.data)
    assert oracle_gather(want, want.ctypes.data, eo) == -1
    return want


def test_cfg2_full_size_full_compare(gpu_ctx):
    """BASELINE config 2 at full size: 2048 x 64 KiB blocks from a 4 GiB pool, through the
    path the benchmark times (gfd_gather_device, entries resident in HBM) and through the
    public host-entry call (gfd_gather_sync): all 128 MiB compared byte for byte with the
    oracle, plus per-token checksums against the source tokens."""
    import torch
    w = wl.cfg2()
    pool = gpu_ctx.pool(w.pool_bytes)
    w.fill_pool(pool.ptr)
    dst = torch_u8(w.total_bytes)
    e = w.entries(pool.ptr, dst.data_ptr())
    want = _oracle_dst(e, dst.data_ptr(), w.total_bytes)
    src_sums = _source_token_checksums(e)
    # host entries, default path
    gpu_ctx.gather_sync(e)
    got = to_np(dst)
    assert np.array_equal(got, want)
    assert np.array_equal(_dst_token_checksums(got, w.token_size, w.num_tokens), src_sums)
    # device entries, the benchmarked call (plan + pull)
    dst.fill_(0xA5)
    d_e = torch.from_numpy(e.view(np.uint8).copy()).cuda()
    gpu_ctx.gather_device(d_e.data_ptr(), w.num_tokens, dst.data_ptr(), w.total_bytes)
    assert gpu_ctx.gather_device_status() == (GFD_OK, -1)
    got = to_np(dst)
    assert np.array_equal(got, want)
    assert np.array_equal(_dst_token_checksums(got, w.token_size, w.num_tokens), src_sums)
    pool.free()


def test_bulk_stage_cfg2_full_compare(gpu_ctx):
    """The cp.async.bulk pull (GFD_GATHER_BULK_STAGE) on config 2 at full size: 2048 x
    64 KiB random blocks, all 128 MiB compared with the oracle, twice in a row (the second
    call reuses the kernel's barriers and buffers from a clean launch), and a call that
    mixes aligned rows with misaligned ones."""
    import torch
    w = wl.cfg2()
    pool = gpu_ctx.pool(w.pool_bytes)
    w.fill_pool(pool.ptr)
    dst = torch_u8(w.total_bytes)
    e = w.entries(pool.ptr, dst.data_ptr())
    want = _oracle_dst(e, dst.data_ptr(), w.total_bytes)
    for _ in range(2):
        dst.fill_(0xA5)
        torch.cuda.synchronize()  # the fill runs on torch's stream, the gather on another
        gpu_ctx.gather_sync(e, flags=gfd_b200.GATHER_BULK_STAGE)
        assert np.array_equal(to_np(dst), want)
    # every 7th entry starts 8 bytes later in its source block and is 16 bytes shorter:
    # those become misaligned rows (bytes they no longer cover stay zero)
    e2 = e.copy()
    e2["src"][::7] += np.uint64(8)
    e2["size"][::7] -= np.uint64(16)
    want2 = _oracle_dst(e2, dst.data_ptr(), w.total_bytes)
    dst.zero_()
    torch.cuda.synchronize()  # the fill runs on torch's stream, the gather on another
    gpu_ctx.gather_sync(e2, flags=gfd_b200.GATHER_BULK_STAGE)
    assert np.array_equal(to_np(dst), want2)
    pool.free()


@pytest.mark.parametrize("size", wl.CFG3_SIZES)
def test_cfg3_sizes_full(gpu_ctx, size):
    """Config 3's 2048-token points at full size, default path, forced SM pull and the
    bulk-copy pull: full compare with the oracle and per-token checksums."""
    import torch
    w = wl.cfg3(2048, size)
    pool = gpu_ctx.pool(w.pool_bytes)
    w.fill_pool(pool.ptr)
    dst = torch_u8(w.total_bytes)
    e = w.entries(pool.ptr, dst.data_ptr())
    want = _oracle_dst(e, dst.data_ptr(), w.total_bytes)
    for flags in (gfd_b200.GATHER_DEFAULT, gfd_b200.GATHER_FORCE_PULL, gfd_b200.GATHER_BULK_STAGE):
        dst.fill_(0xA5)
        torch.cuda.synchronize()  # the fill runs on torch's stream, the gather on another
        gpu_ctx.gather_sync(e, flags=flags)
        got = to_np(dst)[:w.total_bytes]
        assert np.array_equal(got, want), f"flags {flags}"
        assert np.array_equal(_dst_token_checksums(got, size, 2048), _source_token_checksums(e))
    pool.free()


@pytest.mark.parametrize("count", wl.CFG3_COUNTS)
def test_cfg3_counts_full(gpu_ctx, count):
    """Config 3's 4 KiB points ({16 .. 8192} tokens), host entries and device entries."""
    import torch
    w = wl.cfg3(count, 4096)
    pool = gpu_ctx.pool(w.pool_bytes)
    w.fill_pool(pool.ptr)
    dst = torch_u8(w.total_bytes)
    e = w.entries(pool.ptr, dst.data_ptr())
    want = _oracle_dst(e, dst.data_ptr(), w.total_bytes)
    gpu_ctx.gather_sync(e)
    assert np.array_equal(to_np(dst)[:w.total_bytes], want)
    dst.zero_()
    d_e = torch.from_numpy(e.view(np.uint8).copy()).cuda()
    gpu_ctx.gather_device(d_e.data_ptr(), count, dst.data_ptr(), w.total_bytes)
    assert gpu_ctx.gather_device_status() == (GFD_OK, -1)
    assert np.array_equal(to_np(dst)[:w.total_bytes], want)
    pool.free()


def test_repeated_calls_stable(gpu_ctx):
    spec = CASES[6]
    for _ in range(3):
        got, want = run_case(gpu_ctx, spec)
        assert np.array_equal(got, want)


@pytest.mark.parametrize("n", [2048, 9000])
def test_gather_device_in_cuda_graph(gpu_ctx, n):
    """gfd_gather_device captured once into a CUDA graph (after a first call sized its
    scratch) and replayed with a different entry list written into the same device
    buffer each time: every replay lands the bytes of the list it finds there.  The
    9000-entry case captures the multi-CTA plan (count, scan, emit) as well."""
    import torch
    size = 4096
    pool = gpu_ctx.pool(4 * n * size)
    wl.fill_bytes(pool.ptr, pool.nbytes, 77)
    dst = torch_u8(n * size)
    d_off = np.arange(n, dtype=np.uint64) * np.uint64(size)

    def entries_for(seed):
        src = wl.permutation(4 * n, seed)[:n].astype(np.uint64) * np.uint64(size)
        return src, entries_array(d_off + np.uint64(dst.data_ptr()), src + np.uint64(pool.ptr), size)

    _, e0 = entries_for(1)
    d_e = torch.from_numpy(e0.view(np.uint8).copy()).cuda()
    s = torch.cuda.Stream()
    gpu_ctx.gather_device(d_e.data_ptr(), n, dst.data_ptr(), n * size, stream=s.cuda_stream)  # sizes the scratch
    s.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        gpu_ctx.gather_device(d_e.data_ptr(), n, dst.data_ptr(), n * size, stream=s.cuda_stream)
    for seed in (2, 3, 4):
        src, e = entries_for(seed)
        d_e.copy_(torch.from_numpy(e.view(np.uint8).copy()))
        dst.zero_()
        torch.cuda.synchronize()
        g.replay()
        torch.cuda.synchronize()
        rc, bad = gpu_ctx.gather_device_status()
        assert rc == GFD_OK and bad == -1
        want = np.zeros(n * size, np.uint8)
        eo = entries_array(d_off + np.uint64(want.ctypes.data), src + np.uint64(pool.ptr), size)
        assert oracle_gather(want, want.ctypes.data, eo) == -1
        assert np.array_equal(to_np(dst), want), f"replay with list {seed}"
    del g
    pool.free()


@pytest.mark.parametrize("n", [1, 17, 300, 512, 513])
def test_gather_device_short_lists(gpu_ctx, n):
    """Device lists up to 512 entries take one kernel with no plan (a warp per entry);
    513 takes the plan.  Mixed sizes and alignments land exactly; an entry outside the
    destination window and one outside every source range are skipped and the first is
    reported; the next call reports clean again."""
    import torch
    pool = gpu_ctx.pool(64 << 20)
    wl.fill_bytes(pool.ptr, pool.nbytes, n)
    rng = np.random.default_rng(n)
    sizes = rng.choice([7, 16, 100, 4096, 4100, 65536], size=n).astype(np.uint64)
    src = rng.integers(0, (pool.nbytes - 65536) // 16, size=n).astype(np.uint64) * np.uint64(16)
    src += (rng.random(n) < 0.2).astype(np.uint64) * np.uint64(3)  # some misaligned sources
    dst_off = np.concatenate([[0], np.cumsum(sizes)[:-1]]).astype(np.uint64)
    total = int(sizes.sum())
    dst = torch_u8(total)
    e = entries_array(dst_off + np.uint64(dst.data_ptr()), src + np.uint64(pool.ptr), sizes)

    def run(entries):
        dst.zero_()
        d_e = torch.from_numpy(entries.view(np.uint8).copy()).cuda()
        gpu_ctx.gather_device(d_e.data_ptr(), n, dst.data_ptr(), total)
        return gpu_ctx.gather_device_status()

    want = np.zeros(total, np.uint8)
    assert oracle_gather(want, want.ctypes.data, entries_array(dst_off + np.uint64(want.ctypes.data),
                                                               src + np.uint64(pool.ptr), sizes)) == -1
    assert run(e) == (GFD_OK, -1)
    assert np.array_equal(to_np(dst), want)
    if n >= 17:
        bad = e.copy()
        bad["dst"][9] = np.uint64(dst.data_ptr() + total)   # past the window
        bad["src"][13] = np.uint64(8)                         # not host memory this context knows
        rc, first = run(bad)
        assert rc == gfd_b200.GFD_ERR_INVALID and first == 9
        got, mask = to_np(dst), np.ones(total, bool)
        for i in (9, 13):
            mask[int(dst_off[i]):int(dst_off[i] + sizes[i])] = False
        assert np.array_equal(got[mask], want[mask])
        assert run(e) == (GFD_OK, -1)  # state left clean for the next launch
        assert np.array_equal(to_np(dst), want)
    pool.free()


def test_gather_device_short_list_of_large_entries(gpu_ctx):
    """A short device list of a few large entries spreads over the whole grid and lands
    exactly, at a good fraction of the link -- also when one of them sits three bytes off
    its destination's alignment (4-byte funnel-shift copies instead of byte copies)."""
    import torch
    pool = gpu_ctx.pool(64 << 20)
    wl.fill_bytes(pool.ptr, pool.nbytes, 41)
    sizes = np.array([6 << 20, (6 << 20) + 5, 1 << 20, 100], np.uint64)
    src = np.array([0, (20 << 20) + 3, 40 << 20, (50 << 20) + 3], np.uint64)
    dst_off = np.array([0, 6 << 20, (12 << 20) + 16, (13 << 20) + 64], np.uint64)
    total = int(dst_off[-1] + sizes[-1])
    dst = torch_u8(total)
    e = entries_array(dst_off + np.uint64(dst.data_ptr()), src + np.uint64(pool.ptr), sizes)
    d_e = torch.from_numpy(e.view(np.uint8).copy()).cuda()
    s = torch.cuda.Stream()
    for _ in range(2):  # the second call is timed (first-touch effects out of the way)
        dst.zero_()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(s)
        gpu_ctx.gather_device(d_e.data_ptr(), len(e), dst.data_ptr(), total, stream=s.cuda_stream)
        b.record(s)
        s.synchronize()
    assert gpu_ctx.gather_device_status() == (GFD_OK, -1)
    want = np.zeros(total, np.uint8)
    assert oracle_gather(want, want.ctypes.data, entries_array(dst_off + np.uint64(want.ctypes.data),
                                                               src + np.uint64(pool.ptr), sizes)) == -1
    assert np.array_equal(to_np(dst), want)
    gbs = int(sizes.sum()) / (a.elapsed_time(b) * 1e-3) / 1e9
    print(f"short list of large entries: {gbs:.1f} GB/s")
    assert gbs > 25, f"{gbs:.1f} GB/s: large entries did not spread over the grid"
    pool.free()


def test_shared_segment_pool(gpu_ctx):
    """A pool in a shared memfd segment (gfd_b200.shared_pool, the layout the multi-rank
    bench shares between rank processes), registered with the context: random 64 KiB
    blocks gathered through gfd_gather_device and gfd_gather_sync, compared with the oracle."""
    import torch
    from gfd_b200.shared_pool import SharedSegment
    bs, blocks, n = 65536, 1024, 256
    with SharedSegment.create(blocks * bs) as seg:
        wl.fill_bytes(seg.ptr, seg.nbytes, 77)
        gpu_ctx.register(seg.ptr, seg.nbytes)
        try:
            ids = wl.permutation(blocks, 78)[:n].astype(np.uint64)
            dst = torch_u8(n * bs)
            e = gfd_b200.entries_array(np.uint64(dst.data_ptr()) + np.arange(n, dtype=np.uint64) * np.uint64(bs),
                                       np.uint64(seg.ptr) + ids * np.uint64(bs), bs)
            want = _oracle_dst(e, dst.data_ptr(), n * bs)
            d_e = torch.from_numpy(e.view(np.uint8).copy()).cuda()
            gpu_ctx.gather_device(d_e.data_ptr(), n, dst.data_ptr(), n * bs)
            assert gpu_ctx.gather_device_status() == (GFD_OK, -1)
            assert np.array_equal(to_np(dst), want)
            dst.zero_()
            torch.cuda.synchronize()  # the fill runs on torch's stream, the gather on another
            gpu_ctx.gather_sync(e)
            assert np.array_equal(to_np(dst), want)
        finally:
            torch.cuda.synchronize()
            gpu_ctx.unregister(seg.ptr)


def _device_entries_case(pool_ptr, dst_ptr, n=300, bs=8192, seed=91):
    ids = wl.permutation(4096, seed)[:n].astype(np.uint64)
    return gfd_b200.entries_array(np.uint64(dst_ptr) + np.arange(n, dtype=np.uint64) * np.uint64(bs),
                                  np.uint64(pool_ptr) + ids * np.uint64(bs), bs)


def test_gather_device_peer_dst_flag(gpu_ctx):
    """GFD_GATHER_PEER_DST with a window in this GPU's own memory lands the same bytes as
    the plain call; unknown flags are refused before anything is launched."""
    import torch
    bs, n = 8192, 2048
    pool = gpu_ctx.pool(4096 * bs)
    wl.fill_bytes(pool.ptr, 4096 * bs, 92)
    dst = torch_u8(n * bs)
    e = _device_entries_case(pool.ptr, dst.data_ptr(), n, bs)
    want = _oracle_dst(e, dst.data_ptr(), n * bs)
    d_e = torch.from_numpy(e.view(np.uint8).copy()).cuda()
    gpu_ctx.gather_device(d_e.data_ptr(), n, dst.data_ptr(), n * bs, flags=gfd_b200.GATHER_PEER_DST)
    assert gpu_ctx.gather_device_status() == (GFD_OK, -1)
    assert np.array_equal(to_np(dst), want)
    with pytest.raises(gfd_b200.GfdError):
        gpu_ctx.gather_device(d_e.data_ptr(), n, dst.data_ptr(), n * bs, flags=64)
    pool.free()


def test_gather_device_into_peer_gpu(gpu_ctx):
    """A context on GPU 0 pulls from its pinned pool and stores into a buffer on GPU 1
    (GFD_GATHER_PEER_DST: peer access is enabled by the call and the driver must confirm
    write access first); without the flag the same window is refused."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    if not torch.cuda.can_device_access_peer(0, 1):
        pytest.skip("GPU 0 cannot reach GPU 1")
    bs, n = 8192, 2048
    pool = gpu_ctx.pool(4096 * bs)
    wl.fill_bytes(pool.ptr, 4096 * bs, 93)
    dst = torch.zeros(n * bs, dtype=torch.uint8, device="cuda:1")
    e = _device_entries_case(pool.ptr, dst.data_ptr(), n, bs, seed=94)
    want = _oracle_dst(e, dst.data_ptr(), n * bs)
    d_e = torch.from_numpy(e.view(np.uint8).copy()).to("cuda:0")
    with pytest.raises(gfd_b200.GfdError):
        gpu_ctx.gather_device(d_e.data_ptr(), n, dst.data_ptr(), n * bs)
    gpu_ctx.gather_device(d_e.data_ptr(), n, dst.data_ptr(), n * bs, flags=gfd_b200.GATHER_PEER_DST)
    assert gpu_ctx.gather_device_status() == (GFD_OK, -1)
    torch.cuda.synchronize(0)
    assert np.array_equal(dst.cpu().numpy(), want)
    pool.free()
