"""gfd_gather_device_noalloc: the allocation-free entry point.

It exists for callers that may not allocate device memory themselves (operator
plugins inside an engine that owns all device memory through its own pooling
allocator, latency-critical paths where cudaMalloc / cudaFree must not run).  Its
scratch is a fixed device array shared by every call on a GPU, so these tests check
that calls in a row -- with different entry lists, through the short-list kernel and
through the plan + pull kernels -- each produce exactly the bytes of the existing
gfd_gather_device entry point and of the CPU oracle; that a rejected entry is reported
and leaves its destination untouched without spoiling the next call; that a list
longer than GFD_NOALLOC_MAX_ENTRIES is refused; and that a CUDA context destroyed and
replaced by another between two calls still gets correct bytes.

Collected last (file name) so a run that stops at the first failure has already
run every other test; it also passes when run alone in a fresh process.
"""
import ctypes

import numpy as np
import pytest

import gfd_b200
from gfd_b200 import GFD_ERR_INVALID, GFD_OK, entries_array
from gfd_b200 import workloads as wl
from tests.golden.cases import oracle_gather

pytestmark = pytest.mark.gpu

MAX_ENTRIES = 4096  # GFD_NOALLOC_MAX_ENTRIES in include/gfd_b200.h


def _make_entries(rng, pool_ptr, pool_bytes, n, dst_ptr):
    """n tokens of mixed sizes (aligned, unaligned, contiguous runs) from the pool."""
    sizes = rng.choice([16, 64, 512, 4096, 4100, 7, 1000, 65536], size=n).astype(np.uint64)
    src = np.zeros(n, np.uint64)
    cur = 0
    for i in range(n):
        if rng.random() < 0.6:
            cur += int(rng.integers(1, 64)) * 16 + (int(rng.integers(0, 16)) if rng.random() < 0.1 else 0)
        src[i] = cur
        cur += int(sizes[i])
    assert cur <= pool_bytes
    dst_off = np.concatenate([[0], np.cumsum(sizes)[:-1]]).astype(np.uint64)
    return entries_array(dst_off + np.uint64(dst_ptr), src + np.uint64(pool_ptr), sizes), int(sizes.sum())


def _oracle_bytes(entries, dst_ptr, total, fill=0):
    """The oracle's destination bytes for entries aimed at [dst_ptr, dst_ptr + total)."""
    want = np.full(total, fill, np.uint8)
    e = entries.copy()
    e["dst"] = e["dst"] - np.uint64(dst_ptr) + np.uint64(want.ctypes.data)
    assert oracle_gather(want, want.ctypes.data, e) == -1
    return want


def _noalloc(lib, d_entries, n, src_ptr, src_bytes, dst_ptr, dst_bytes, stream, status):
    return lib.gfd_gather_device_noalloc(ctypes.c_void_p(d_entries), n, ctypes.c_void_p(src_ptr), src_bytes,
                                         ctypes.c_void_p(dst_ptr), dst_bytes, ctypes.c_void_p(stream),
                                         ctypes.c_void_p(status))


def test_noalloc_matches_gather_device_and_oracle_twice(gpu_ctx):
    import torch
    lib = gfd_b200.load()
    pool = gpu_ctx.pool(256 << 20)
    wl.fill_bytes(pool.ptr, pool.nbytes, 77)
    rng = np.random.default_rng(77)
    stream = torch.cuda.Stream()
    status = torch.full((2,), 99, dtype=torch.int64, device="cuda")
    for n in (MAX_ENTRIES, 300):  # two calls in a row; the second reuses a dirtier scratch
        e, total = _make_entries(rng, pool.ptr, pool.nbytes, n, 0)
        ref_dst = torch.zeros(total, dtype=torch.uint8, device="cuda")
        new_dst = torch.full((total,), 0xEE, dtype=torch.uint8, device="cuda")
        e_ref = e.copy()
        e_ref["dst"] += np.uint64(ref_dst.data_ptr())
        e_new = e.copy()
        e_new["dst"] += np.uint64(new_dst.data_ptr())
        d_ref = torch.from_numpy(e_ref.view(np.uint8).copy()).cuda()
        d_new = torch.from_numpy(e_new.view(np.uint8).copy()).cuda()
        torch.cuda.synchronize()
        # existing entry point
        gpu_ctx.gather_device(d_ref.data_ptr(), n, ref_dst.data_ptr(), total)
        rc, bad = gpu_ctx.gather_device_status()
        assert rc == GFD_OK and bad == -1
        # allocation-free entry point
        rc = _noalloc(lib, d_new.data_ptr(), n, pool.ptr, pool.nbytes, new_dst.data_ptr(), total,
                      stream.cuda_stream, status.data_ptr())
        assert rc == GFD_OK
        stream.synchronize()
        assert status.cpu().tolist() == [GFD_OK, -1]
        assert torch.equal(new_dst, ref_dst), f"n={n}: outputs differ from gfd_gather_device"
        want = _oracle_bytes(e, 0, total)
        assert np.array_equal(new_dst.cpu().numpy(), want), f"n={n}: output differs from the oracle"
    pool.free()


def test_noalloc_plan_path_reports_a_bad_entry_then_recovers(gpu_ctx):
    """A full-size list (plan + pull kernels) with one source outside the window: the
    status names it, its destination keeps its old bytes, every other entry lands; the
    next call (short-list kernel, same scratch) reports success."""
    import torch
    lib = gfd_b200.load()
    pool = gpu_ctx.pool(128 << 20)
    wl.fill_bytes(pool.ptr, pool.nbytes, 5)
    rng = np.random.default_rng(5)
    e, total = _make_entries(rng, pool.ptr, pool.nbytes - (1 << 20), MAX_ENTRIES, 0)
    bad = 1234
    # every size is at least 7 bytes, so this source runs past the declared window
    e["src"][bad] = np.uint64(pool.ptr + pool.nbytes - 4)
    dst = torch.full((total,), 0x5A, dtype=torch.uint8, device="cuda")
    dst_off = e["dst"].copy()
    e["dst"] += np.uint64(dst.data_ptr())
    d = torch.from_numpy(e.view(np.uint8).copy()).cuda()
    status = torch.full((2,), 99, dtype=torch.int64, device="cuda")
    torch.cuda.synchronize()
    assert _noalloc(lib, d.data_ptr(), MAX_ENTRIES, pool.ptr, pool.nbytes, dst.data_ptr(), total, 0,
                    status.data_ptr()) == GFD_OK
    torch.cuda.synchronize()
    assert status.cpu().tolist() == [GFD_ERR_INVALID, bad]
    good = np.ones(MAX_ENTRIES, bool)
    good[bad] = False
    want = _oracle_bytes(e[good], dst.data_ptr(), total, fill=0x5A)
    got = dst.cpu().numpy()
    lo = int(dst_off[bad])
    assert np.all(got[lo:lo + int(e["size"][bad])] == 0x5A), "the rejected entry's destination was written"
    assert np.array_equal(got, want)
    # the short-list kernel right after, on the same scratch header
    e2, total2 = _make_entries(rng, pool.ptr, pool.nbytes - (1 << 20), 40, 0)
    dst2 = torch.zeros(total2, dtype=torch.uint8, device="cuda")
    e2["dst"] += np.uint64(dst2.data_ptr())
    d2 = torch.from_numpy(e2.view(np.uint8).copy()).cuda()
    torch.cuda.synchronize()
    assert _noalloc(lib, d2.data_ptr(), 40, pool.ptr, pool.nbytes, dst2.data_ptr(), total2, 0,
                    status.data_ptr()) == GFD_OK
    torch.cuda.synchronize()
    assert status.cpu().tolist() == [GFD_OK, -1]
    assert np.array_equal(dst2.cpu().numpy(), _oracle_bytes(e2, dst2.data_ptr(), total2))
    pool.free()


def test_noalloc_rejects_oversized_list(gpu_ctx):
    import torch
    lib = gfd_b200.load()
    pool = gpu_ctx.pool(2 << 20)
    dst = torch.zeros(64, dtype=torch.uint8, device="cuda")
    e = entries_array(np.full(MAX_ENTRIES + 1, dst.data_ptr(), np.uint64), pool.ptr, 0)
    d = torch.from_numpy(e.view(np.uint8).copy()).cuda()
    rc = _noalloc(lib, d.data_ptr(), MAX_ENTRIES + 1, pool.ptr, pool.nbytes, dst.data_ptr(), 64, 0, 0)
    assert rc == GFD_ERR_INVALID
    # a source outside the declared window is reported, and nothing else is touched
    pool.array()[:64] = 5
    e = entries_array([dst.data_ptr(), dst.data_ptr() + 32], [pool.ptr, pool.ptr + pool.nbytes - 16], [32, 32])
    d = torch.from_numpy(e.view(np.uint8).copy()).cuda()
    status = torch.zeros(2, dtype=torch.int64, device="cuda")
    assert _noalloc(lib, d.data_ptr(), 2, pool.ptr, pool.nbytes, dst.data_ptr(), 64, 0, status.data_ptr()) == GFD_OK
    torch.cuda.synchronize()
    assert status.cpu().tolist() == [GFD_ERR_INVALID, 1]
    got = dst.cpu().numpy()
    assert np.all(got[:32] == 5) and not got[32:].any()
    pool.free()


class _Driver:
    """The few driver-API calls a caller that manages its own CUDA contexts makes."""

    def __init__(self):
        self.cu = ctypes.CDLL("libcuda.so.1")

    def __call__(self, name, *args):
        rc = getattr(self.cu, name)(*args)
        assert rc == 0, f"{name} returned {rc}"


def test_noalloc_after_context_turnover():
    """Two driver-API contexts in turn on one GPU (the first destroyed before the second
    is created, so the second may be handed the same handle): each call resolves the
    scratch of its own context and lands the oracle's bytes."""
    lib = gfd_b200.load()
    cu = _Driver()
    cu("cuInit", 0)
    dev = ctypes.c_int()
    cu("cuDeviceGet", ctypes.byref(dev), 0)
    rng = np.random.default_rng(11)
    handles = []
    for n in (MAX_ENTRIES, 300):  # plan + pull kernels, then the short-list kernel
        ctx = ctypes.c_void_p()
        cu("cuCtxCreate_v2", ctypes.byref(ctx), 0, dev)  # created current on this thread
        handles.append(ctx.value)
        try:
            pool_bytes = 96 << 20
            host = ctypes.c_void_p()
            # CU_MEMHOSTALLOC_PORTABLE | CU_MEMHOSTALLOC_DEVICEMAP
            cu("cuMemHostAlloc", ctypes.byref(host), ctypes.c_size_t(pool_bytes), 0x1 | 0x2)
            try:
                wl.fill_bytes(host.value, pool_bytes, 11 + n)
                e, total = _make_entries(rng, host.value, pool_bytes, n, 0)
                dptr, dent, dstat = ctypes.c_uint64(), ctypes.c_uint64(), ctypes.c_uint64()
                cu("cuMemAlloc_v2", ctypes.byref(dptr), ctypes.c_size_t(total))
                cu("cuMemAlloc_v2", ctypes.byref(dent), ctypes.c_size_t(e.nbytes))
                cu("cuMemAlloc_v2", ctypes.byref(dstat), ctypes.c_size_t(16))
                try:
                    cu("cuMemsetD8_v2", dptr, ctypes.c_ubyte(0xEE), ctypes.c_size_t(total))
                    e_dev = e.copy()
                    e_dev["dst"] += np.uint64(dptr.value)
                    cu("cuMemcpyHtoD_v2", dent, e_dev.ctypes.data_as(ctypes.c_void_p), ctypes.c_size_t(e.nbytes))
                    rc = _noalloc(lib, dent.value, n, host.value, pool_bytes, dptr.value, total, 0, dstat.value)
                    assert rc == GFD_OK
                    cu("cuCtxSynchronize")
                    got = np.empty(total, np.uint8)
                    st = np.empty(2, np.int64)
                    cu("cuMemcpyDtoH_v2", got.ctypes.data_as(ctypes.c_void_p), dptr, ctypes.c_size_t(total))
                    cu("cuMemcpyDtoH_v2", st.ctypes.data_as(ctypes.c_void_p), dstat, ctypes.c_size_t(16))
                    assert st.tolist() == [GFD_OK, -1]
                    assert np.array_equal(got, _oracle_bytes(e, 0, total)), f"context {len(handles)}: wrong bytes"
                finally:
                    for p in (dptr, dent, dstat):
                        if p.value:
                            cu("cuMemFree_v2", p)
            finally:
                cu("cuMemFreeHost", host)
        finally:
            cu("cuCtxDestroy_v2", ctx)
