"""Device -> host scatter (gfd_scatter / gfd_scatter_sync): the same pull kernel with the
roles swapped, checked bit for bit against the CPU oracle's memcpy semantics (every
entry's bytes land at its host destination, in entry order)."""
import numpy as np
import pytest

import gfd_b200
from gfd_b200 import GFD_ERR_INVALID, GFD_OK, entries_array
from gfd_b200 import workloads as wl
from tests.golden.cases import checksum, oracle_gather

pytestmark = pytest.mark.gpu


def device_bytes(nbytes, seed):
    import torch
    host = np.empty(nbytes, np.uint8)
    wl.fill_bytes(host.ctypes.data, nbytes, seed)
    return torch.from_numpy(host).cuda(), host


def expected(pool_before, host_src, src_base, pool_base, e):
    """Oracle: the pool after scattering entries e (src offsets into host_src)."""
    want = pool_before.copy()
    eo = e.copy()
    eo["src"] = e["src"] - np.uint64(src_base) + np.uint64(host_src.ctypes.data)
    eo["dst"] = e["dst"] - np.uint64(pool_base) + np.uint64(want.ctypes.data)
    assert oracle_gather(want, want.ctypes.data, eo) == -1
    return want


@pytest.mark.parametrize("n,size,stride", [(256, 4096, 8192), (2048, 512, 1024), (100, 65536, 65536),
                                           (1000, 1040, 3000)])
def test_scatter_matches_oracle(gpu_ctx, n, size, stride):
    src, host_src = device_bytes(n * size, n + size)
    pool = gpu_ctx.pool(n * stride + 4096)
    arr = pool.array()
    arr[:] = 0x5A
    before = arr.copy()
    perm = wl.permutation(n, 7)
    dst = np.uint64(pool.ptr) + perm.astype(np.uint64) * np.uint64(stride)
    e = entries_array(dst, np.uint64(src.data_ptr()) + np.arange(n, dtype=np.uint64) * np.uint64(size), size)
    gpu_ctx.scatter_sync(e)
    assert np.array_equal(arr, expected(before, host_src, src.data_ptr(), pool.ptr, e))
    pool.free()


def test_scatter_alignment_matrix(gpu_ctx):
    """Every src/dst misalignment and size class (head, 16-byte body, narrow paths, tail)."""
    src, host_src = device_bytes(1 << 20, 3)
    pool = gpu_ctx.pool(4 << 20)
    arr = pool.array()
    arr[:] = 0
    before = arr.copy()
    rows = []
    cs, cd = 0, 0
    for size in [1, 2, 15, 16, 17, 100, 511, 512, 4095, 4096, 4097, 65536 + 3]:
        for so in [0, 1, 4, 8, 15]:
            for do in [0, 1, 3, 8, 12]:
                cs = (cs + 64) // 64 * 64 + so
                cd = (cd + 64) // 64 * 64 + do
                if cs + size > (1 << 20):
                    cs = so
                rows.append((cd, cs, size))
                cd += size
    d = np.array([r[0] for r in rows], np.uint64) + np.uint64(pool.ptr)
    s = np.array([r[1] for r in rows], np.uint64) + np.uint64(src.data_ptr())
    z = np.array([r[2] for r in rows], np.uint64)
    assert int(d.max() - np.uint64(pool.ptr) + z.max()) < pool.nbytes
    e = entries_array(d, s, z)
    gpu_ctx.scatter_sync(e)
    assert np.array_equal(arr, expected(before, host_src, src.data_ptr(), pool.ptr, e))
    pool.free()


def test_scatter_copy_engine_and_async(gpu_ctx):
    import torch
    src, host_src = device_bytes(512 * 4096, 11)
    pool = gpu_ctx.pool(1024 * 4096)
    arr = pool.array()
    perm = wl.permutation(1024, 11)[:512]
    e = entries_array(np.uint64(pool.ptr) + perm.astype(np.uint64) * np.uint64(4096),
                      np.uint64(src.data_ptr()) + np.arange(512, dtype=np.uint64) * np.uint64(4096), 4096)
    for flags in (gfd_b200.GATHER_FORCE_CE, gfd_b200.GATHER_DEFAULT):
        arr[:] = 0
        before = arr.copy()
        stream = torch.cuda.Stream()
        assert gpu_ctx.scatter(e, stream=stream.cuda_stream, flags=flags) == GFD_OK
        stream.synchronize()
        assert np.array_equal(arr, expected(before, host_src, src.data_ptr(), pool.ptr, e))
    pool.free()


def test_gather_scatter_round_trip_cfg2(gpu_ctx):
    """cfg2 blocks gathered into HBM, then scattered back to their own slots of a second
    pool: per-block checksums equal the first pool's."""
    import torch
    w = wl.cfg2()
    pool = gpu_ctx.pool(w.pool_bytes)
    w.fill_pool(pool.ptr)
    dst = torch.empty(w.total_bytes, dtype=torch.uint8, device="cuda")
    gpu_ctx.gather_sync(w.entries(pool.ptr, dst.data_ptr()))
    back = gpu_ctx.pool(w.pool_bytes)
    e = w.entries(back.ptr, dst.data_ptr())
    e["dst"], e["src"] = e["src"].copy(), e["dst"].copy()  # host slot <- HBM block
    gpu_ctx.scatter_sync(e)
    a = pool.array().reshape(-1, 65536)
    b = back.array().reshape(-1, 65536)
    for blk in w.block_ids[::16]:
        assert checksum(a[blk]) == checksum(b[blk])
    back.free()
    pool.free()


def test_scatter_validation(gpu_ctx):
    import torch
    src = torch.zeros(8192, dtype=torch.uint8, device="cuda")
    torch.cuda.synchronize()
    pool = gpu_ctx.pool(8192)
    pageable = np.zeros(8192, np.uint8)
    # src in host memory, dst in device memory: the gather's direction, rejected here
    e = entries_array([src.data_ptr()], [pool.ptr], 4096)
    assert gpu_ctx.scatter_sync_rc(e) == GFD_ERR_INVALID
    # pageable host destination
    e = entries_array([pageable.ctypes.data], [src.data_ptr()], 4096)
    assert gpu_ctx.scatter_sync_rc(e) == GFD_ERR_INVALID
    # a source range running past the end of its device allocation (validation is per
    # allocation: torch's caching allocator backs this tensor with a larger segment)
    e = entries_array([pool.ptr], [src.data_ptr() + 8000], 1 << 30)
    assert gpu_ctx.scatter_sync_rc(e) == GFD_ERR_INVALID
    assert gpu_ctx.scatter_sync_rc(entries_array([], [], 0)) == GFD_OK
    pool.free()
