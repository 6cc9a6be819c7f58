"""MoE gather through SGWarpSpecSession with GPU-submitted lists (libgfd_moe_sg.so):
the per-expert destination layout must equal the oracle's, bit for bit, including the
benchmark shard whose 32,768 entries pass through the 16,384-entry pool in waves."""
import numpy as np
import pytest

from gfd_b200 import GFD_OK, moe_sg
from gfd_b200 import workloads as wl
from tests.golden.cases import oracle_moe_route

pytestmark = pytest.mark.gpu


def route_and_sg(ctx, sg, logits, k, pool_ptr, token_rows, row_bytes, rows_per_list=0):
    import torch
    tokens, experts = logits.shape
    d_logits = torch.from_numpy(np.ascontiguousarray(logits)).cuda()
    src = np.uint64(pool_ptr) + token_rows.astype(np.uint64) * np.uint64(row_bytes)
    d_src = torch.from_numpy(src.view(np.int64)).cuda()
    dst = torch.zeros(tokens * k * row_bytes, dtype=torch.uint8, device="cuda")
    cnt = torch.zeros(2 * experts, dtype=torch.int32, device="cuda")
    ent = torch.zeros(tokens * k * 24, dtype=torch.uint8, device="cuda")
    # one explicit stream for both calls: to gfd_moe_route_gather a NULL stream means the
    # context's own stream, which is not ordered with the legacy default stream
    s = torch.cuda.Stream()
    stream = s.cuda_stream
    sg.prepare()
    ctx.moe_route_gather(d_logits.data_ptr(), tokens, experts, k, d_src.data_ptr(), row_bytes, dst.data_ptr(),
                         dst.numel(), cnt.data_ptr(), cnt.data_ptr() + 4 * experts, ent.data_ptr(), stream=stream,
                         route_only=True)
    sg.run(ent.data_ptr(), cnt.data_ptr(), cnt.data_ptr() + 4 * experts, experts, stream, rows_per_list=rows_per_list)
    rc, timeouts, moved = sg.sync()
    return dst.cpu().numpy(), rc, timeouts, moved


def expected(pool_arr, token_rows, row_token, row_bytes):
    view = pool_arr[:len(pool_arr) // row_bytes * row_bytes].reshape(-1, row_bytes)
    return view[token_rows[row_token].astype(np.int64)].reshape(-1)


@pytest.mark.parametrize("tokens,experts,k,row_bytes,rpl", [(256, 64, 8, 14336, 0), (1000, 16, 2, 4096, 0),
                                                         (64, 8, 1, 512, 0), (1000, 16, 2, 4096, 100),
                                                         (256, 64, 8, 14336, 7)])
def test_sg_session_matches_oracle(gpu_ctx, tokens, experts, k, row_bytes, rpl):
    pool = gpu_ctx.pool(4096 * row_bytes)
    wl.fill_bytes(pool.ptr, pool.nbytes, tokens)
    logits = np.empty((tokens, experts), np.float32)
    wl.fill_f32_normal(logits.ctypes.data, logits.size, tokens + 1)
    rows = wl.permutation(4096, tokens)[:tokens]
    with moe_sg.MoESG(wait_timeout_ms=5000) as sg:
        for _ in range(2):  # the session is reused across passes
            got, rc, timeouts, moved = route_and_sg(gpu_ctx, sg, logits, k, pool.ptr, rows, row_bytes, rpl)
            assert (rc, timeouts) == (GFD_OK, 0)
            assert moved == tokens * k * row_bytes
            _, _, _, row_token = oracle_moe_route(logits, k)
            assert np.array_equal(got, expected(pool.array(), rows, row_token, row_bytes))
    pool.free()


@pytest.mark.parametrize("rpl", [0, 128])
def test_sg_session_cfg5_shard(gpu_ctx, rpl):
    shard = wl.MoEShard(0)
    pool = gpu_ctx.pool(shard.pool_bytes)
    shard.fill_pool(pool.ptr)
    logits = shard.logits()
    rows = shard.token_rows()
    with moe_sg.MoESG(wait_timeout_ms=5000) as sg:
        got, rc, timeouts, moved = route_and_sg(gpu_ctx, sg, logits, shard.k, pool.ptr, rows, shard.row_bytes, rpl)
    assert (rc, timeouts) == (GFD_OK, 0)
    assert moved == shard.dst_bytes
    _, _, _, row_token = oracle_moe_route(logits, shard.k)
    assert np.array_equal(got, expected(pool.array(), rows, row_token, shard.row_bytes))
    pool.free()
