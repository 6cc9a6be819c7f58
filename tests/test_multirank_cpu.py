"""Host-side multi-rank logic of bench.py on CPU: two gloo ranks (127.0.0.1) run the
same barrier / max-over-ranks / aggregation code the GPU bench runs over NCCL."""
import os
import socket

import pytest
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    import bench
    d = bench.Dist(world, backend="gloo")
    d.barrier()
    # rank r's step k takes (k + 1) * (r + 1) ms: the slowest rank is the last one
    mine = [(k + 1) * (rank + 1) * 1e-3 for k in range(4)]
    slowest = d.max_vec(mine)
    value = bench.aggregate_gbs(1 << 27, world, slowest)
    peak_sum = d.sum_vec([50.0 + rank])[0]  # concurrent per-link peaks summed over ranks
    per_rank = d.all_values(float(rank))
    blobs = d.all_bytes(bytes([rank] * 5 + [255 - rank] * 67))  # an IPC handle + offset is 72 bytes
    assert blobs == [bytes([r] * 5 + [255 - r] * 67) for r in range(world)]
    out[rank] = (slowest, value, peak_sum, per_rank)
    d.barrier()
    d.close()


@pytest.mark.parametrize("world", [2, 3])
def test_max_over_ranks_and_aggregate(world):
    port = _free_port()
    mgr = mp.Manager()
    out = mgr.dict()
    mp.spawn(_rank_main, args=(world, port, out), nprocs=world, join=True)
    expect = [(k + 1) * world * 1e-3 for k in range(4)]
    for r in range(world):
        slowest, value, peak_sum, per_rank = out[r]
        assert per_rank == [float(k) for k in range(world)]
        assert slowest == pytest.approx(expect)
        assert peak_sum == pytest.approx(sum(50.0 + k for k in range(world)))
        assert value == pytest.approx(world * (1 << 27) * 4 / sum(expect) / 1e9)


def _leaving_rank_main(rank, world, port, out):
    """Rank 1 leaves between steps (after the first barrier, before the second): rank 0
    must get an error from its next collective, not hang."""
    import time
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    import bench
    d = bench.Dist(world, backend="gloo", timeout_s=5)
    d.barrier()
    if rank == 1:
        out[rank] = "left"
        os._exit(0)  # gone without a goodbye, as a crashed rank would be
    t0 = time.monotonic()
    try:
        d.barrier()
        out[rank] = ("no error", time.monotonic() - t0)
    except Exception as exc:  # gloo reports the closed peer or the timeout
        out[rank] = (type(exc).__name__, time.monotonic() - t0)
    os._exit(0)


def test_rank_that_leaves_ends_the_next_collective_with_an_error():
    port = _free_port()
    mgr = mp.Manager()
    out = mgr.dict()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_leaving_rank_main, args=(r, 2, port, out)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=60)
        assert not p.is_alive(), "a rank hung"
    assert out[1] == "left"
    kind, seconds = out[0]
    assert kind != "no error"
    assert seconds < 30
