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


def test_ring_started_completes_runs_without_polls(ring_setup):
    """With the ring started (the agent consumes it), runs committed one after another
    complete without explicit polls; the last slot of each run carries FLAG_LAST_IN_BATCH."""
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


# ---------------------------------------------------------------------------
# The same protocol consumed by the ring agent (gfd_ring_start): a device-resident
# kernel polls the markers, copies the descriptors out, validates them (asking the host
# once about each range it has not seen) and pulls the bytes; no host thread reads a
# descriptor.
# ---------------------------------------------------------------------------
@pytest.fixture()
def agent_setup(gpu_ctx):
    q = gpu_ctx.pool(QUEUE_BYTES)
    ring = DescriptorRing(q)
    r = Ring(gpu_ctx, ring.ptr)
    yield gpu_ctx, ring, r
    r.close()
    q.free()


def test_agent_wraps_and_lands_mixed_sizes(agent_setup):
    """Three runs of 7000 descriptors (the third wraps past slot 16384) with aligned,
    misaligned and zero-size descriptors, consumed by the agent; the destination is a
    tensor the agent learns about through a range query."""
    import torch
    ctx, ring, r = agent_setup
    n, rounds = 7000, 3
    sizes = np.array([4096, 1040, 0, 64, 4096, 17], np.uint64)[np.arange(n) % 6]
    offs = np.concatenate([[0], np.cumsum(sizes)[:-1]]).astype(np.uint64)
    total = int(sizes.sum())
    src = ctx.pool(2 * n * 4096)
    wl.fill_bytes(src.ptr, src.nbytes, 21)
    dst = torch.zeros(total, dtype=torch.uint8, device="cuda")
    torch.cuda.synchronize()
    r.start()
    try:
        base = 0
        for rnd in range(rounds):
            perm = wl.permutation(2 * n, 200 + rnd)[:n].astype(np.uint64)
            s_addr = np.uint64(src.ptr) + perm * np.uint64(4096)
            flags = np.zeros(n, np.uint32)
            flags[-1] = gfd_b200.FLAG_LAST_IN_BATCH
            ring.produce(base, s_addr, np.uint64(dst.data_ptr()) + offs, sizes, flags)
            r.wait(base + n)
            base += n
            e = entries_array(offs, s_addr, sizes)
            assert np.array_equal(dst.cpu().numpy(), expected(total, src, src.array(), e)), f"round {rnd}"
            assert ring.read_idx == base and ring.done_idx == base
            slots = (base - n + np.arange(n)) % QUEUE_SIZE
            assert not ring.entries["seq"][slots].any(), "markers not cleared"
            dst.zero_()
            torch.cuda.synchronize()
    finally:
        r.stop()
    stats = r.agent_stats()
    assert stats["launches"] >= 1 and stats["timeouts"] == 0 and stats["rejected"] == 0
    assert stats["queries"] >= 1  # the destination tensor was learnt, not declared
    c = r.counters()
    assert c["consumed"] == n * rounds and c["bytes"] == total * rounds
    src.free()


def test_agent_rejects_invalid_descriptors(agent_setup):
    """Pageable sources and host-memory destinations are refused by the host's answer to
    the agent's range query: skipped and counted, nothing written to host memory, and the
    run still completes."""
    import torch
    ctx, ring, r = agent_setup
    n = 300
    src = ctx.pool(n * 4096)
    wl.fill_bytes(src.ptr, src.nbytes, 5)
    pageable = np.ones(n * 4096, np.uint8)
    dst = torch.zeros(n * 4096, dtype=torch.uint8, device="cuda")
    r.allow(dst.data_ptr())  # declared: no query for the real destination
    s_addr = np.uint64(src.ptr) + np.arange(n, dtype=np.uint64) * np.uint64(4096)
    d_addr = np.uint64(dst.data_ptr()) + np.arange(n, dtype=np.uint64) * np.uint64(4096)
    bad_src = np.arange(n) % 7 == 3
    bad_dst = np.arange(n) % 11 == 5
    s_addr[bad_src] = np.uint64(pageable.ctypes.data) + np.arange(n, dtype=np.uint64)[bad_src] * np.uint64(4096)
    d_addr[bad_dst] = np.uint64(pageable.ctypes.data)
    torch.cuda.synchronize()
    r.start()
    try:
        ring.produce(0, s_addr, d_addr, 4096, np.where(np.arange(n) == n - 1, 1, 0))
        r.wait(n)
    finally:
        r.stop()
    assert ring.done_idx == n and ring.read_idx == n
    stats = r.agent_stats()
    assert stats["rejected"] == int((bad_src | bad_dst).sum()) and stats["timeouts"] == 0
    ok = ~(bad_src | bad_dst)
    e = entries_array((np.arange(n, dtype=np.uint64) * np.uint64(4096))[ok], s_addr[ok], 4096)
    assert np.array_equal(dst.cpu().numpy(), expected(n * 4096, src, src.array(), e))
    assert pageable.min() == 1 and pageable.max() == 1
    src.free()


def test_agent_leaves_when_idle_and_comes_back(agent_setup):
    """Default mode: after the linger time with nothing committed the agent exits (so a
    device-wide synchronize returns) and the next commit brings it back."""
    import time
    import torch
    ctx, ring, r = agent_setup
    n = 256
    src = ctx.pool(n * 8192)
    wl.fill_bytes(src.ptr, src.nbytes, 13)
    dst = torch.zeros(n * 4096, dtype=torch.uint8, device="cuda")
    torch.cuda.synchronize()
    r.start()
    try:
        base = 0
        for rnd in range(5):
            s_addr = np.uint64(src.ptr) + np.arange(n, dtype=np.uint64) * np.uint64(8192) + np.uint64(rnd * 16)
            ring.produce(base, s_addr, np.uint64(dst.data_ptr()) + np.arange(n, dtype=np.uint64) * np.uint64(4096),
                         4096)
            r.wait(base + n)
            base += n
            torch.cuda.synchronize()  # returns once the agent has left
            e = entries_array(np.arange(n, dtype=np.uint64) * np.uint64(4096), s_addr, 4096)
            assert np.array_equal(dst.cpu().numpy(), expected(n * 4096, src, src.array(), e)), f"round {rnd}"
            time.sleep(0.002)
    finally:
        r.stop()
    assert r.agent_stats()["launches"] >= 5
    src.free()


def test_agent_query_wait_runs_out(gpu_ctx, monkeypatch):
    """Fault injected on the host: the service thread drops the agent's range queries.
    The agent's mailbox wait gives up after the context's limit (100 ms here), counts the
    give-up, rejects the descriptor and completes the run; declared windows still land,
    and the context keeps working."""
    import torch
    monkeypatch.setenv("GFD_RING_TEST_DROP_QUERIES", "1")
    q = gpu_ctx.pool(QUEUE_BYTES)
    ring = DescriptorRing(q)
    gpu_ctx.set_timeout_ns(100_000_000)
    r = Ring(gpu_ctx, ring.ptr)
    try:
        n = 64
        src = gpu_ctx.pool(n * 4096)
        wl.fill_bytes(src.ptr, src.nbytes, 17)
        known = torch.zeros(n * 4096, dtype=torch.uint8, device="cuda")
        unknown = torch.full((4096,), 7, dtype=torch.uint8, device="cuda")
        # exactly this window: `unknown` may sit in the same caching-allocator segment
        r.allow(known.data_ptr(), known.numel())
        s_addr = np.uint64(src.ptr) + np.arange(n, dtype=np.uint64) * np.uint64(4096)
        d_addr = np.uint64(known.data_ptr()) + np.arange(n, dtype=np.uint64) * np.uint64(4096)
        d_addr[10] = np.uint64(unknown.data_ptr())  # never declared: needs an answer that never comes
        torch.cuda.synchronize()
        r.start()
        try:
            ring.produce(0, s_addr, d_addr, 4096, np.where(np.arange(n) == n - 1, 1, 0))
            for _ in range(50):  # each wait is bounded by the same 100 ms
                try:
                    r.wait(n)
                    break
                except gfd_b200.GfdError as exc:
                    assert exc.code == gfd_b200.GFD_ERR_TIMEOUT
        finally:
            r.stop()
        stats = r.agent_stats()
        assert stats["timeouts"] >= 1 and stats["rejected"] == 1
        assert ring.done_idx == n
        ok = np.arange(n) != 10
        e = entries_array((np.arange(n, dtype=np.uint64) * np.uint64(4096))[ok], s_addr[ok], 4096)
        assert np.array_equal(known.cpu().numpy(), expected(n * 4096, src, src.array(), e))
        assert int(unknown.min()) == 7 and int(unknown.max()) == 7
        x = torch.arange(10, device="cuda")
        assert int((x * 2).sum()) == 90  # the context still runs work
        src.free()
    finally:
        r.close()
        gpu_ctx.set_timeout_ns(10_000_000_000)
        q.free()
