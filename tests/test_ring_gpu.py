"""GPU-queued submit through this library's ring consumer, driven from the host: the test
writes descriptors into a ring in pinned memory the way a GPU producer does (fields,
then the commit marker), and checks what the reference's consumer guarantees
(src/cpu_polling.cpp:337-436, src/batch_processor.cpp:605-831): every valid
descriptor's bytes land at its destination (bit-exact against the oracle), markers go
back to 0, read_idx / done_idx reach the end of each drained run, the ring wraps.
Descriptors that fail validation are skipped and reported, and their run still
completes."""
import numpy as np
import pytest

import gfd_b200
from gfd_b200 import QUEUE_BYTES, QUEUE_SIZE, DescriptorRing, Ring, entries_array
from gfd_b200 import workloads as wl
from tests.golden.cases import oracle_gather

pytestmark = pytest.mark.gpu


def expected(dst_bytes, src_pool, src_host, e):
    """Oracle: the destination buffer (starting zeroed) after gathering entries e, whose
    dst fields are offsets into it and src fields addresses in src_pool."""
    want = np.zeros(dst_bytes, np.uint8)
    eo = e.copy()
    eo["src"] = e["src"] - np.uint64(src_pool.ptr) + np.uint64(src_host.ctypes.data)
    eo["dst"] = e["dst"] + np.uint64(want.ctypes.data)
    assert oracle_gather(want, want.ctypes.data, eo) == -1
    return want


@pytest.fixture()
def ring_setup(gpu_ctx):
    q = gpu_ctx.pool(QUEUE_BYTES)
    ring = DescriptorRing(q)
    r = Ring(gpu_ctx, ring.ptr)
    yield gpu_ctx, ring, r
    r.close()
    q.free()


def test_ring_batches_wrap_and_land(ring_setup):
    """Three runs of 7000 descriptors (the third wraps past slot 16384), mixed sizes
    including misaligned and zero-size ones."""
    import torch
    ctx, ring, r = ring_setup
    n, rounds = 7000, 3
    sizes = np.array([4096, 1040, 0, 64, 4096, 17], np.uint64)[np.arange(n) % 6]
    offs = np.concatenate([[0], np.cumsum(sizes)[:-1]]).astype(np.uint64)
    total = int(sizes.sum())
    src = ctx.pool(2 * n * 4096)
    wl.fill_bytes(src.ptr, src.nbytes, 11)
    host = src.array()
    dst = torch.zeros(total, dtype=torch.uint8, device="cuda")
    base = 0
    for rnd in range(rounds):
        perm = wl.permutation(2 * n, 100 + rnd)[:n].astype(np.uint64)
        s_addr = np.uint64(src.ptr) + perm * np.uint64(4096)
        dst.zero_()
        torch.cuda.synchronize()
        flags = np.zeros(n, np.uint32)
        flags[-1] = gfd_b200.FLAG_LAST_IN_BATCH
        ring.produce(base, s_addr, np.uint64(dst.data_ptr()) + offs, sizes, flags)
        assert r.poll() >= 1
        r.wait(base + n)
        base += n
        e = entries_array(offs, s_addr, sizes)
        assert np.array_equal(dst.cpu().numpy(), expected(total, src, host, e)), f"round {rnd}"
        assert ring.read_idx == base and ring.done_idx == base
        slots = (base - n + np.arange(n)) % QUEUE_SIZE
        assert not ring.entries["seq"][slots].any(), "markers not cleared"
    c = r.counters()
    assert c["consumed"] == n * rounds
    assert c["bytes"] == total * rounds
    src.free()


def test_ring_skips_invalid_descriptors(ring_setup):
    """Sources outside pinned memory and destinations outside device memory are skipped
    (and reported); the run still completes and the valid descriptors land."""
    import torch
    ctx, ring, r = ring_setup
    n = 300
    src = ctx.pool(n * 4096)
    wl.fill_bytes(src.ptr, src.nbytes, 5)
    pageable = np.ones(n * 4096, np.uint8)
    dst = torch.zeros(n * 4096, dtype=torch.uint8, device="cuda")
    s_addr = np.uint64(src.ptr) + np.arange(n, dtype=np.uint64) * np.uint64(4096)
    d_addr = np.uint64(dst.data_ptr()) + np.arange(n, dtype=np.uint64) * np.uint64(4096)
    bad_src = np.arange(n) % 7 == 3
    bad_dst = np.arange(n) % 11 == 5
    s_addr[bad_src] = np.uint64(pageable.ctypes.data) + np.arange(n, dtype=np.uint64)[bad_src] * np.uint64(4096)
    d_addr[bad_dst] = np.uint64(pageable.ctypes.data)  # host memory as a destination
    ring.produce(0, s_addr, d_addr, 4096, np.where(np.arange(n) == n - 1, 1, 0))
    r.poll()
    r.wait(n)
    assert ring.done_idx == n and ring.read_idx == n
    assert "rejected" in ctx.last_error()
    ok = ~(bad_src | bad_dst)
    e = entries_array((np.arange(n, dtype=np.uint64) * np.uint64(4096))[ok], s_addr[ok], 4096)
    assert np.array_equal(dst.cpu().numpy(), expected(n * 4096, src, src.array(), e))
    assert pageable.min() == 1 and pageable.max() == 1  # nothing written to host memory
    src.free()


def test_ring_run_with_nothing_to_move(ring_setup):
    """A run whose descriptors are all rejected or empty still advances the indices (the
    drain launches its completion alone)."""
    ctx, ring, r = ring_setup
    n = 40
    pageable = np.zeros(4096, np.uint8)
    sizes = np.where(np.arange(n) % 2 == 0, 0, 4096).astype(np.uint64)
    ring.produce(0, np.full(n, pageable.ctypes.data, np.uint64), 0, sizes)
    r.poll()
    r.wait(n)
    assert ring.done_idx == n and ring.read_idx == n
    assert not ring.entries["seq"][:n].any()
    assert r.counters()["bytes"] == 0


def test_ring_doorbell_thread(ring_setup):
    """With the doorbell thread running, runs committed one after another complete
    without explicit polls; the last run of each batch carries FLAG_LAST_IN_BATCH."""
    import torch
    ctx, ring, r = ring_setup
    n = 512
    src = ctx.pool(n * 8192)
    wl.fill_bytes(src.ptr, src.nbytes, 9)
    dst = torch.zeros(n * 8192, dtype=torch.uint8, device="cuda")
    r.start()
    try:
        base = 0
        for size in (8192, 4096, 100):
            s_addr = np.uint64(src.ptr) + np.arange(n, dtype=np.uint64) * np.uint64(size)
            dst.zero_()
            torch.cuda.synchronize()
            ring.produce(base, s_addr, np.uint64(dst.data_ptr()) + np.arange(n, dtype=np.uint64) * np.uint64(size),
                         size, np.where(np.arange(n) == n - 1, 1, 0))
            r.wait(base + n)
            base += n
            e = entries_array(np.arange(n, dtype=np.uint64) * np.uint64(size), s_addr, size)
            got = dst.cpu().numpy()
            assert np.array_equal(got, expected(n * 8192, src, src.array(), e)), f"size {size}"
    finally:
        r.stop()
    src.free()
