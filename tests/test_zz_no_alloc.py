"""gfd_gather_device_noalloc: the allocation-free entry point.

It exists for callers that may not allocate device memory themselves (operator
plugins inside an engine that owns all device memory through its own pooling
allocator, latency-critical paths where cudaMalloc / cudaFree must not run).  Its
scratch is a fixed device array shared by every call on a GPU, so this test checks
that two calls in a row -- the second with a different, smaller entry list -- each
produce exactly the bytes of the existing gfd_gather_device entry point, and that a
list longer than GFD_NOALLOC_MAX_ENTRIES is refused without touching the output.

Collected last (file name) so a run that stops at the first failure has already
run every other test; it also passes when run alone in a fresh process.
"""
import ctypes

import numpy as np
import pytest

import gfd_b200
from gfd_b200 import GFD_ERR_INVALID, GFD_OK, entries_array
from gfd_b200 import workloads as wl

pytestmark = pytest.mark.gpu

MAX_ENTRIES = 4096  # GFD_NOALLOC_MAX_ENTRIES in include/gfd_b200.h


def _make_entries(rng, pool, n, dst_ptr):
    """n tokens of mixed sizes (aligned, unaligned, contiguous runs) from the pool."""
    sizes = rng.choice([16, 64, 512, 4096, 4100, 7, 1000, 65536], size=n).astype(np.uint64)
    src = np.zeros(n, np.uint64)
    cur = 0
    for i in range(n):
        if rng.random() < 0.6:
            cur += int(rng.integers(1, 64)) * 16 + (int(rng.integers(0, 16)) if rng.random() < 0.1 else 0)
        src[i] = cur
        cur += int(sizes[i])
    assert cur <= pool.nbytes
    dst_off = np.concatenate([[0], np.cumsum(sizes)[:-1]]).astype(np.uint64)
    return entries_array(dst_off + np.uint64(dst_ptr), src + np.uint64(pool.ptr), sizes), int(sizes.sum())


def _noalloc(lib, d_entries, n, pool, dst, dst_bytes, stream, status):
    return lib.gfd_gather_device_noalloc(ctypes.c_void_p(d_entries), n, ctypes.c_void_p(pool.ptr), pool.nbytes,
                                         ctypes.c_void_p(dst.data_ptr()), dst_bytes, ctypes.c_void_p(stream),
                                         ctypes.c_void_p(status))


def test_noalloc_matches_gather_device_twice(gpu_ctx):
    import torch
    lib = gfd_b200.load()
    pool = gpu_ctx.pool(256 << 20)
    wl.fill_bytes(pool.ptr, pool.nbytes, 77)
    rng = np.random.default_rng(77)
    stream = torch.cuda.Stream()
    status = torch.full((2,), 99, dtype=torch.int64, device="cuda")
    for n in (MAX_ENTRIES, 300):  # two calls in a row; the second reuses a dirtier scratch
        e, total = _make_entries(rng, pool, n, 0)
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
        rc = _noalloc(lib, d_new.data_ptr(), n, pool, new_dst, total, stream.cuda_stream, status.data_ptr())
        assert rc == GFD_OK
        stream.synchronize()
        assert status.cpu().tolist() == [GFD_OK, -1]
        assert torch.equal(new_dst, ref_dst), f"n={n}: outputs differ"
    pool.free()


def test_noalloc_rejects_oversized_list(gpu_ctx):
    import torch
    lib = gfd_b200.load()
    pool = gpu_ctx.pool(2 << 20)
    dst = torch.zeros(64, dtype=torch.uint8, device="cuda")
    e = entries_array(np.full(MAX_ENTRIES + 1, dst.data_ptr(), np.uint64), pool.ptr, 0)
    d = torch.from_numpy(e.view(np.uint8).copy()).cuda()
    rc = _noalloc(lib, d.data_ptr(), MAX_ENTRIES + 1, pool, dst, 64, 0, 0)
    assert rc == GFD_ERR_INVALID
    # a source outside the declared window is reported, and nothing else is touched
    pool.array()[:64] = 5
    e = entries_array([dst.data_ptr(), dst.data_ptr() + 32], [pool.ptr, pool.ptr + pool.nbytes - 16], [32, 32])
    d = torch.from_numpy(e.view(np.uint8).copy()).cuda()
    status = torch.zeros(2, dtype=torch.int64, device="cuda")
    assert _noalloc(lib, d.data_ptr(), 2, pool, dst, 64, 0, status.data_ptr()) == GFD_OK
    torch.cuda.synchronize()
    assert status.cpu().tolist() == [GFD_ERR_INVALID, 1]
    got = dst.cpu().numpy()
    assert np.all(got[:32] == 5) and not got[32:].any()
    pool.free()
