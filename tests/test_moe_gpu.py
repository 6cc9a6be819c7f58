"""MoE routing front end on the GPU (gfd_moe_route_gather) against the CPU oracle.

Routing (top-k, ties to the lower expert id, NaN lowest), the per-expert counts and
offsets, the gather list and the gathered bytes are all compared bit for bit with
oracle/route_ref.c + a numpy gather of the same pool rows.
"""
import ctypes

import numpy as np
import pytest

import gfd_b200
from gfd_b200 import GFD_ERR_INVALID, GFD_OK
from gfd_b200 import workloads as wl
from tests.golden.cases import oracle_moe_route

pytestmark = pytest.mark.gpu


def dev(nbytes):
    import torch
    return torch.zeros(max(int(nbytes), 1), dtype=torch.uint8, device="cuda")


def run_route(ctx, logits, k, pool, token_rows, row_bytes, route_only=False):
    import torch
    tokens, experts = logits.shape
    d_logits = torch.from_numpy(np.ascontiguousarray(logits)).cuda()
    src = np.uint64(pool.ptr) + token_rows.astype(np.uint64) * np.uint64(row_bytes)
    d_src = torch.from_numpy(src.view(np.int64)).cuda()
    dst = dev(tokens * k * row_bytes)
    d_counts = torch.zeros(experts, dtype=torch.int32, device="cuda")
    d_offsets = torch.zeros(experts, dtype=torch.int32, device="cuda")
    d_entries = dev(tokens * k * 24)
    stream = torch.cuda.current_stream().cuda_stream
    ctx.moe_route_gather(d_logits.data_ptr(), tokens, experts, k, d_src.data_ptr(), row_bytes, dst.data_ptr(),
                         dst.numel(), d_counts.data_ptr(), d_offsets.data_ptr(), d_entries.data_ptr(),
                         stream=stream, route_only=route_only)
    torch.cuda.synchronize()
    entries = d_entries.cpu().numpy()[:tokens * k * 24].view(gfd_b200.SG_ENTRY_DTYPE)
    return (dst.cpu().numpy(), d_counts.cpu().numpy().view(np.uint32), d_offsets.cpu().numpy().view(np.uint32),
            entries, dst.data_ptr())


def expected_bytes(pool_arr, token_rows, row_token, row_bytes):
    rows = token_rows[row_token].astype(np.int64)
    view = pool_arr[:len(pool_arr) // row_bytes * row_bytes].reshape(-1, row_bytes)
    return view[rows].reshape(-1)


def check(ctx, logits, k, row_bytes, pool_rows, seed):
    tokens, experts = logits.shape
    pool = ctx.pool(pool_rows * row_bytes)
    wl.fill_bytes(pool.ptr, pool.nbytes, seed)
    token_rows = wl.permutation(pool_rows, seed)[:tokens]
    got, counts, offsets, entries, dst_base = run_route(ctx, logits, k, pool, token_rows, row_bytes)
    rc, bad = ctx.gather_device_status()
    assert rc == GFD_OK and bad == -1
    _, want_counts, want_offsets, row_token = oracle_moe_route(logits, k)
    assert np.array_equal(counts, want_counts)
    assert np.array_equal(offsets, want_offsets)
    j = np.arange(tokens * k, dtype=np.uint64)
    assert np.array_equal(entries["dst"], np.uint64(dst_base) + j * np.uint64(row_bytes))
    assert np.array_equal(entries["size"], np.full(tokens * k, row_bytes, np.uint64))
    want_src = np.uint64(pool.ptr) + token_rows[row_token].astype(np.uint64) * np.uint64(row_bytes)
    assert np.array_equal(entries["src"], want_src)
    assert np.array_equal(got, expected_bytes(pool.array(), token_rows, row_token, row_bytes))
    pool.free()


@pytest.mark.parametrize("tokens,experts,k,row_bytes", [
    (256, 64, 8, 14336),     # cfg5 shape, fewer tokens
    (1500, 40, 3, 4096),     # experts not a multiple of 32, tokens not a multiple of 1024
    (37, 8, 8, 100),         # k == experts, unaligned 100-byte rows
    (1024, 1, 1, 512),       # one expert
    (300, 1024, 32, 256),    # the largest expert count and k
])
def test_route_gather_matches_oracle(gpu_ctx, tokens, experts, k, row_bytes):
    logits = np.empty((tokens, experts), np.float32)
    wl.fill_f32_normal(logits.ctypes.data, logits.size, tokens + experts)
    check(gpu_ctx, logits, k, row_bytes, pool_rows=4096, seed=tokens)


def test_ties_nan_inf(gpu_ctx):
    rng = np.random.default_rng(11)
    x = (np.round(rng.standard_normal((512, 64)) * 2) / 2).astype(np.float32)
    flat = x.reshape(-1)
    idx = rng.choice(flat.size, flat.size // 10, replace=False)
    flat[idx] = np.array([np.nan, -np.inf, np.inf, -0.0, 0.0], np.float32)[rng.integers(0, 5, idx.size)]
    x[5, :] = np.nan        # a token whose logits are all NaN: experts 0..k-1
    x[6, :] = 1.0           # all tied: experts 0..k-1
    check(gpu_ctx, x, 8, 2048, pool_rows=1024, seed=5)


def test_cfg5_full_shard(gpu_ctx):
    """The benchmark shard (GPU 0 seeds): 4096 x 64 logits, top-8, 262,144-row pool of
    14,336-byte bf16 rows; every landed byte compared."""
    shard = wl.MoEShard(0)
    pool = gpu_ctx.pool(shard.pool_bytes)
    shard.fill_pool(pool.ptr)
    logits = shard.logits()
    token_rows = shard.token_rows()
    got, counts, offsets, entries, _ = run_route(gpu_ctx, logits, shard.k, pool, token_rows, shard.row_bytes)
    assert gpu_ctx.gather_device_status() == (GFD_OK, -1)
    _, want_counts, want_offsets, row_token = oracle_moe_route(logits, shard.k)
    assert np.array_equal(counts, want_counts) and np.array_equal(offsets, want_offsets)
    assert np.array_equal(got, expected_bytes(pool.array(), token_rows, row_token, shard.row_bytes))
    pool.free()


def test_route_only_then_gather_device(gpu_ctx):
    """GFD_MOE_ROUTE_ONLY writes the list without pulling; gfd_gather_device on that list
    gives the same bytes."""
    import torch
    logits = np.empty((200, 16), np.float32)
    wl.fill_f32_normal(logits.ctypes.data, logits.size, 77)
    pool = gpu_ctx.pool(512 * 1024)
    wl.fill_bytes(pool.ptr, pool.nbytes, 77)
    rows = wl.permutation(512, 77)[:200]
    got, _, _, entries, dst_base = run_route(gpu_ctx, logits, 2, pool, rows, 1024, route_only=True)
    assert not got.any()
    dst = dev(200 * 2 * 1024)
    e = entries.copy()
    e["dst"] = e["dst"] - np.uint64(dst_base) + np.uint64(dst.data_ptr())
    d_entries = torch.from_numpy(e.view(np.uint8).copy()).cuda()
    gpu_ctx.gather_device(d_entries.data_ptr(), len(e), dst.data_ptr(), dst.numel())
    torch.cuda.synchronize()
    _, _, _, row_token = oracle_moe_route(logits, 2)
    assert np.array_equal(dst.cpu().numpy(), expected_bytes(pool.array(), rows, row_token, 1024))
    pool.free()


def test_invalid_arguments(gpu_ctx):
    import torch
    lib, h = gpu_ctx.lib, gpu_ctx.handle
    logits = torch.zeros(64 * 8, dtype=torch.float32, device="cuda")
    src = torch.zeros(64, dtype=torch.int64, device="cuda")
    dst = dev(64 * 8 * 256)
    cnt = torch.zeros(2048, dtype=torch.int32, device="cuda")
    ent = dev(64 * 8 * 24)
    host_logits = np.zeros(64 * 8, np.float32)

    def call(lg, tokens, experts, k, dst_bytes):
        return lib.gfd_moe_route_gather(h, ctypes.c_void_p(lg), tokens, experts, k, ctypes.c_void_p(src.data_ptr()),
                                        256, ctypes.c_void_p(dst.data_ptr()), dst_bytes,
                                        ctypes.c_void_p(cnt.data_ptr()), ctypes.c_void_p(cnt.data_ptr() + 4096),
                                        ctypes.c_void_p(ent.data_ptr()), None, gfd_b200.MOE_ROUTE_ONLY)

    assert call(logits.data_ptr(), 64, 8, 9, dst.numel()) == GFD_ERR_INVALID        # k > experts
    assert call(logits.data_ptr(), 64, 8, 0, dst.numel()) == GFD_ERR_INVALID        # k == 0
    assert call(logits.data_ptr(), 1, 1025, 1, dst.numel()) == GFD_ERR_INVALID       # too many experts
    assert call(logits.data_ptr(), 64, 8, 8, dst.numel() - 1) == GFD_ERR_INVALID    # dst too small
    assert call(host_logits.ctypes.data, 64, 8, 8, dst.numel()) == GFD_ERR_INVALID  # logits not on device
    assert call(logits.data_ptr(), 64, 8, 8, dst.numel()) == GFD_OK
    torch.cuda.synchronize()


def test_sources_outside_pools_rejected(gpu_ctx):
    """Token rows in pageable host memory: routing succeeds, the gather rejects them."""
    import torch
    logits = np.zeros((32, 4), np.float32)
    pageable = np.zeros(32 * 256, np.uint8)
    rows_src = np.uint64(pageable.ctypes.data) + np.arange(32, dtype=np.uint64) * np.uint64(256)
    d_logits = torch.from_numpy(logits).cuda()
    d_src = torch.from_numpy(rows_src.view(np.int64)).cuda()
    dst = dev(32 * 2 * 256)
    cnt = torch.zeros(8, dtype=torch.int32, device="cuda")
    ent = dev(32 * 2 * 24)
    gpu_ctx.moe_route_gather(d_logits.data_ptr(), 32, 4, 2, d_src.data_ptr(), 256, dst.data_ptr(), dst.numel(),
                             cnt.data_ptr(), cnt.data_ptr() + 16, ent.data_ptr())
    rc, bad = gpu_ctx.gather_device_status()
    assert rc == GFD_ERR_INVALID and bad == 0
    assert not dst.cpu().numpy().any()
