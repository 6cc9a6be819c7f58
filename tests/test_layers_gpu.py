"""Layer pipeline (WarpSpecSession page-table mode + RMS-scale compute warps) against
the CPU oracle (oracle/route_ref.c): landed bytes, scaled values and per-block sums of
squares, bit for bit."""
import numpy as np
import pytest

from gfd_b200 import layers
from gfd_b200 import workloads as wl
from tests.golden.cases import checksum, oracle_layer_pipeline

pytestmark = pytest.mark.gpu


def run_pipeline(ctx, pool, table, block_bytes, mode, tokens_per_tile=32, double_buffer=False,
                 producer_warps=0, prefill=0):
    import torch
    d_table = torch.from_numpy(table.astype(np.int32)).cuda()
    dst = torch.full((len(table) * block_bytes,), prefill, dtype=torch.uint8, device="cuda")
    ss = torch.zeros(len(table), dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    with layers.LayerPipeline(pool.ptr, pool.nbytes, d_table.data_ptr(), len(table), block_bytes, dst.data_ptr(),
                              ss.data_ptr(), tokens_per_tile=tokens_per_tile, producer_warps=producer_warps,
                              double_buffer=double_buffer, wait_timeout_ms=5000) as lp:
        lp.run(mode)
        rejected, timeouts, nbytes = lp.sync()
    return dst.cpu().numpy(), ss.cpu().numpy(), rejected, timeouts, nbytes


def make_pool(ctx, blocks, block_bytes, seed):
    pool = ctx.pool(blocks * block_bytes)
    wl.fill_bf16_normal(pool.ptr, pool.nbytes // 2, seed)
    return pool


@pytest.mark.parametrize("block_bytes,per_layer,layers_n,tpt,db,pw", [
    (65536, 64, 4, 32, False, 0),     # cfg4 block size
    (65536, 64, 4, 32, True, 0),      # double-buffered compute sets
    (4096, 256, 3, 128, False, 2),    # small blocks, 2 producer warps
    (1040, 96, 2, 32, False, 0),      # 16-byte multiple, not a power of two
])
def test_rms_pipeline_matches_oracle(gpu_ctx, block_bytes, per_layer, layers_n, tpt, db, pw):
    pool_blocks = 512
    pool = make_pool(gpu_ctx, pool_blocks, block_bytes, 40 + layers_n)
    table = wl.cfg4_table(layers_n, per_layer, pool_blocks, seed=9)
    got, ss, rejected, timeouts, nbytes = run_pipeline(gpu_ctx, pool, table, block_bytes, layers.RMS,
                                                       tokens_per_tile=tpt, double_buffer=db, producer_warps=pw)
    assert (rejected, timeouts) == (0, 0)
    assert nbytes == len(table) * block_bytes
    want, want_ss, bad = oracle_layer_pipeline(pool.array(np.uint16), table, block_bytes)
    assert bad == -1
    assert np.array_equal(ss, want_ss)
    assert np.array_equal(got.view(np.uint16), want)
    pool.free()


def test_transfer_only_lands_blocks(gpu_ctx):
    block_bytes = 65536
    pool = make_pool(gpu_ctx, 256, block_bytes, 3)
    table = wl.cfg4_table(2, 128, 256, seed=21)
    got, _, rejected, timeouts, _ = run_pipeline(gpu_ctx, pool, table, block_bytes, layers.TRANSFER)
    assert (rejected, timeouts) == (0, 0)
    view = pool.array().reshape(-1, block_bytes)
    assert np.array_equal(got.reshape(-1, block_bytes), view[table])
    pool.free()


def test_bad_block_id_is_skipped_and_counted(gpu_ctx):
    """Ids are checked on the device at every launch: an id beyond the pool is skipped
    (its destination keeps the prefill), counted, and the other blocks land."""
    block_bytes = 4096
    pool = make_pool(gpu_ctx, 64, block_bytes, 8)
    table = wl.permutation(64, 8)[:32].copy()
    table[5] = 64           # one past the pool
    table[17] = 0xFFFFFFFF
    got, _, rejected, _, _ = run_pipeline(gpu_ctx, pool, table, block_bytes, layers.TRANSFER, prefill=0xAB)
    assert rejected == 2
    got = got.reshape(-1, block_bytes)
    view = pool.array().reshape(-1, block_bytes)
    for i, b in enumerate(table):
        if i in (5, 17):
            assert (got[i] == 0xAB).all()
        else:
            assert np.array_equal(got[i], view[b])
    pool.free()


def test_launch_shape_above_kernel_limit_is_refused(gpu_ctx):
    """12 producer warps + two compute sets of 8 warps = 896 threads, above the kernels'
    640-thread bound: the session refuses the launch instead of launching."""
    import torch
    pool = make_pool(gpu_ctx, 64, 65536, 1)
    table = wl.permutation(64, 1)[:32].copy()
    d_table = torch.from_numpy(table.astype(np.int32)).cuda()
    dst = torch.zeros(32 * 65536, dtype=torch.uint8, device="cuda")
    torch.cuda.synchronize()
    with layers.LayerPipeline(pool.ptr, pool.nbytes, d_table.data_ptr(), 32, 65536, dst.data_ptr(),
                              tokens_per_tile=32, producer_warps=12, double_buffer=True) as lp:
        assert lp.block_threads == 896
        with pytest.raises(RuntimeError):
            lp.run(layers.RMS)
    assert not dst.cpu().numpy().any()
    pool.free()


def test_cfg4_full_pass(gpu_ctx):
    """The benchmark pass: 32 layers x 1024 blocks of 64 KiB from a 4 GiB pool.  Transfer
    mode: 2048 sampled blocks' checksums against their pool blocks.  RMS mode: sums of
    squares and full bytes of 512 sampled blocks against the oracle."""
    bb = wl.CFG4_BLOCK_BYTES
    pool = gpu_ctx.pool(wl.CFG4_POOL_BLOCKS * bb)
    wl.cfg4_fill_pool(pool.ptr)
    table = wl.cfg4_table()
    got, _, rejected, timeouts, _ = run_pipeline(gpu_ctx, pool, table, bb, layers.TRANSFER)
    assert (rejected, timeouts) == (0, 0)
    g = got.reshape(-1, bb)
    view = pool.array().reshape(-1, bb)
    rng = np.random.default_rng(4)
    for i in rng.choice(len(table), 2048, replace=False):
        assert checksum(g[i]) == checksum(view[table[i]])
    got, ss, rejected, timeouts, _ = run_pipeline(gpu_ctx, pool, table, bb, layers.RMS)
    assert (rejected, timeouts) == (0, 0)
    sample = np.sort(rng.choice(len(table), 512, replace=False))
    want, want_ss, _ = oracle_layer_pipeline(pool.array(np.uint16), table[sample], bb)
    assert np.array_equal(ss[sample], want_ss)
    assert np.array_equal(got.reshape(-1, bb)[sample].reshape(-1).view(np.uint16), want)
    pool.free()
