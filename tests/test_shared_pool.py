"""Host logic of the shared pool (gfd_b200.shared_pool) on CPU: the link-rate
apportionment and one memfd segment seen by two gloo rank processes."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from gfd_b200.shared_pool import SharedSegment, forward_plan, rate_shares


@pytest.mark.parametrize("rates,total", [
    ([1.0, 1.0], 4096),
    ([21.0, 21.5, 22.0, 21.2, 36.0, 35.8, 36.1, 36.3], 8 * 2048),  # this pool's two link groups
    ([3.0, 1.0, 0.0], 10),
    ([0.0, 0.0], 5),
    ([50.0, 0.001], 2),
    ([7.0], 0),
])
def test_rate_shares_sum_and_proportion(rates, total):
    shares = rate_shares(rates, total)
    assert len(shares) == len(rates)
    assert sum(shares) == total
    assert all(s >= 0 for s in shares)
    pos = [max(r, 0.0) for r in rates]
    if sum(pos) > 0:
        live = [i for i, r in enumerate(pos) if r > 0]
        for i, r in enumerate(pos):
            if r == 0:
                assert shares[i] == 0
        if total >= len(live):
            assert all(shares[i] >= 1 for i in live)
        exact = [total * r / sum(pos) for r in pos]
        # largest remainder keeps every share within one unit of its exact value, except
        # where a live rank had to be lifted to one unit
        assert sum(abs(s - e) for s, e in zip(shares, exact)) <= len(rates) + 1
    else:
        assert max(shares) - min(shares) <= 1


def test_rate_shares_two_groups_finish_together():
    rates = [21.0] * 4 + [36.0] * 4
    shares = rate_shares(rates, 8 * 2048)
    times = [s / r for s, r in zip(shares, rates)]
    assert max(times) / min(times) < 1.001
    # against equal shards the slowest rank's time shrinks by the rate ratio
    equal_t = 2048 / 21.0
    assert max(times) < equal_t * 0.8


def test_rate_shares_rejects_bad_input():
    with pytest.raises(ValueError):
        rate_shares([], 5)
    with pytest.raises(ValueError):
        rate_shares([1.0], -1)


@pytest.mark.parametrize("shares,need", [
    ([2048] * 4, [2048] * 4),                                           # nothing to forward
    ([1515, 1518, 1519, 1512, 2571, 2582, 2582, 2585], [2048] * 8),     # this pool's two link groups
    ([0, 4096], [2048, 2048]),                                          # one rank pulls everything
    ([3, 1, 8, 0], [3, 3, 3, 3]),
    ([5, 0, 0], [1, 2, 2]),
])
def test_forward_plan_covers_every_block_once(shares, need):
    own, transfers = forward_plan(shares, need)
    assert own == [min(s, n) for s, n in zip(shares, need)]
    pulled = list(own)
    for d, r, first, count in transfers:
        assert count > 0 and shares[d] > need[d] and need[r] > shares[r]
        pulled[d] += count
    assert pulled == list(shares)
    for r, n in enumerate(need):
        covered = [0] * n
        for k in range(own[r]):
            covered[k] += 1
        for d, rr, first, count in transfers:
            if rr == r:
                for k in range(first, first + count):
                    covered[k] += 1
        assert covered == [1] * n


def test_forward_plan_rejects_bad_input():
    with pytest.raises(ValueError):
        forward_plan([1, 2], [2, 2])
    with pytest.raises(ValueError):
        forward_plan([1], [1, 0])
    with pytest.raises(ValueError):
        forward_plan([-1, 3], [1, 1])


def test_segment_create_write_close():
    with SharedSegment.create(1 << 20) as seg:
        a = np.frombuffer(seg.map, dtype=np.uint8)
        a[:4] = [1, 2, 3, 4]
        assert seg.ptr != 0
        pid, fd = seg.pid_fd()
        assert pid == os.getpid() and fd >= 0
        # a second mapping of the same segment in this process sees the bytes
        other = SharedSegment.attach(pid, fd, 1 << 20)
        b = np.frombuffer(other.map, dtype=np.uint8)
        assert list(b[:4]) == [1, 2, 3, 4]
        del a, b
        other.close()
    assert seg.fd == -1 and seg.ptr == 0


def test_segment_attach_rejects_short_segment():
    with SharedSegment.create(4096) as seg:
        pid, fd = seg.pid_fd()
        with pytest.raises(ValueError):
            SharedSegment.attach(pid, fd, 8192)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    import bench
    d = bench.Dist(world, backend="gloo", timeout_s=30)
    n = 1 << 20
    seg = SharedSegment.create(n) if rank == 0 else None
    pid, fd = seg.pid_fd() if seg is not None else (0, 0)
    pids, fds = d.all_values(float(pid)), d.all_values(float(fd))
    if rank == 0:
        np.frombuffer(seg.map, dtype=np.uint8)[:4096] = np.arange(4096) % 251
    d.barrier()
    if rank != 0:
        seg = SharedSegment.attach(int(pids[0]), int(fds[0]), n)
    view = np.frombuffer(seg.map, dtype=np.uint8)
    seen_first = bool(np.array_equal(view[:4096], np.arange(4096) % 251))
    # every rank writes its own page; afterwards every rank sees all of them
    view[4096 * (rank + 1):4096 * (rank + 2)] = rank + 1
    d.barrier()
    seen_all = all(int(view[4096 * (r + 1)]) == r + 1 for r in range(world))
    out[rank] = (seen_first, seen_all)
    del view
    d.barrier()
    seg.close()
    d.close()


def test_segment_shared_between_rank_processes():
    world = 2
    port = _free_port()
    mgr = mp.Manager()
    out = mgr.dict()
    mp.spawn(_rank_main, args=(world, port, out), nprocs=world, join=True)
    for r in range(world):
        assert out[r] == (True, True)
