"""CPU checks of the routing and RMS-scale oracles (oracle/route_ref.c).

The reference has no CPU implementation of either: its MoE example routes round-robin
on the GPU (examples/09_sg_warp_spec.cu:246-276, 509) and its RMS functor is device code
(examples/07_warp_spec_simple.cu:35-59).  So the oracle is pinned here against
independent numpy formulations of the same specification:
  - top-k: a stable lexicographic sort on (-key, expert id) with NaN as -inf;
  - list order: the reference's submitter loops (experts outer, tokens inner);
  - RMS scale: fma emulated in float64 (x*x of a bf16 value is exact there), the
    32-lane butterfly, correctly rounded divide / sqrt, bf16 round to nearest even.
"""
import ctypes
import os

import numpy as np
import pytest

from tests.golden.cases import oracle, oracle_layer_pipeline, oracle_moe_route

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def numpy_topk(logits, k):
    key = np.where(np.isnan(logits), -np.inf, logits).astype(np.float32)
    t, e = logits.shape
    ids = np.broadcast_to(np.arange(e), (t, e))
    sel = np.zeros((t, k), np.uint16)
    for i in range(t):
        order = np.lexsort((ids[i], -key[i].astype(np.float64)))
        sel[i] = order[:k]
    return sel


def reference_list_order(sel, experts):
    """examples/09_sg_warp_spec.cu:246-270: for each expert, the tokens routed to it in
    ascending token order."""
    routed = [set(r.tolist()) for r in sel]
    rows = []
    for e in range(experts):
        for t in range(len(sel)):
            if e in routed[t]:
                rows.append(t)
    return np.array(rows, np.int64)


def special_logits(tokens, experts, seed):
    rng = np.random.default_rng(seed)
    x = np.round(rng.standard_normal((tokens, experts)) * 2) / 2  # many ties
    x = x.astype(np.float32)
    flat = x.reshape(-1)
    idx = rng.choice(flat.size, size=flat.size // 20, replace=False)
    specials = np.array([np.nan, -np.inf, np.inf, -0.0, 0.0], np.float32)
    flat[idx] = specials[rng.integers(0, len(specials), idx.size)]
    return x


@pytest.mark.parametrize("tokens,experts,k,seed", [(64, 64, 8, 1), (300, 40, 3, 2), (17, 8, 8, 3),
                                                   (50, 1, 1, 4), (20, 1024, 32, 5)])
def test_topk_matches_numpy(tokens, experts, k, seed):
    logits = special_logits(tokens, experts, seed)
    sel, counts, offsets, row_token = oracle_moe_route(logits, k)
    want = numpy_topk(logits, k)
    assert np.array_equal(sel, want)
    assert np.array_equal(counts, np.bincount(want.reshape(-1), minlength=experts).astype(np.uint32))
    assert np.array_equal(offsets, np.concatenate([[0], np.cumsum(counts)[:-1]]).astype(np.uint32))
    assert np.array_equal(row_token, reference_list_order(want, experts))


def test_nan_ranks_lowest_and_ties_take_lower_id():
    logits = np.array([[np.nan, 1.0, 1.0, -np.inf],
                       [np.nan, np.nan, -np.inf, np.nan]], np.float32)
    sel, _, _, _ = oracle_moe_route(logits, 3)
    assert sel[0].tolist() == [1, 2, 0]  # 1.0 tie -> lower id; NaN (-inf) ties -inf -> lower id 0
    assert sel[1].tolist() == [0, 1, 2]  # NaN == -inf in rank; ids ascending


def test_bad_shapes_rejected():
    lib = oracle()
    logits = np.zeros((4, 8), np.float32)
    buf = np.zeros(1024, np.int64)
    for experts, k in [(8, 0), (8, 9), (2000, 1)]:
        assert lib.gfd_oracle_moe_route(logits.ctypes.data, 4, experts, k, buf.ctypes.data, buf.ctypes.data,
                                        buf.ctypes.data, buf.ctypes.data) == -1


def bf16_to_f32(u16):
    return (u16.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(f):
    u = f.astype(np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return u.astype(np.uint16)


def numpy_rms(block_u16, eps=np.float32(1e-6)):
    x = bf16_to_f32(block_u16)
    n = x.size
    vec = x.reshape(-1, 8)
    lanes = np.zeros(32, np.float32)
    for l in range(32):
        acc = np.float32(0)
        for j in range(l, vec.shape[0], 32):
            for e in range(8):
                v = np.float64(vec[j, e])
                acc = np.float32(v * v + np.float64(acc))  # fma: x*x exact in float64
        lanes[l] = acc
    for o in (16, 8, 4, 2, 1):
        lanes = (lanes + lanes[np.arange(32) ^ o]).astype(np.float32)
    ss = lanes[0]
    mean = np.float32(ss / np.float32(n))
    s = np.float32(np.float32(1) / np.sqrt(np.float32(mean + eps)))
    return f32_to_bf16(x * s), ss


@pytest.mark.parametrize("nbytes,seed", [(4096, 1), (1040, 2), (16384, 3)])
def test_rms_oracle_matches_numpy(nbytes, seed):
    rng = np.random.default_rng(seed)
    vals = rng.standard_normal(nbytes // 2).astype(np.float32)
    block = f32_to_bf16(vals)
    want, want_ss = numpy_rms(block)
    got = block.copy()
    ss = oracle().gfd_oracle_rms_scale(got.ctypes.data, got.size, ctypes.c_float(1e-6))
    assert np.float32(ss) == want_ss
    assert np.array_equal(got, want)
    # and the value is the RMS scale of the specification within bf16 rounding
    x = bf16_to_f32(block).astype(np.float64)
    exact = x / np.sqrt(np.mean(x * x) + 1e-6)
    assert np.max(np.abs(bf16_to_f32(got) - exact)) <= np.max(np.abs(exact)) * 2 ** -7


def test_layer_pipeline_oracle_bad_id_leaves_block():
    rng = np.random.default_rng(7)
    block_bytes = 1024
    pool = f32_to_bf16(rng.standard_normal(8 * block_bytes // 2).astype(np.float32))
    table = np.array([3, 0, 9, 7], np.uint32)
    out, ss, bad = oracle_layer_pipeline(pool, table, block_bytes)
    assert bad == 2 and ss[2] == 0
    n = block_bytes // 2
    assert not out[2 * n:3 * n].any()
    blk = pool[3 * n:4 * n].copy()
    want, want_ss = numpy_rms(blk)
    assert np.array_equal(out[:n], want) and ss[0] == want_ss


def test_layers_library_exports():
    from gfd_b200 import layers
    lib = layers.lib()
    for name in ("gfd_layers_create", "gfd_layers_run", "gfd_layers_sync", "gfd_layers_block_threads",
                 "gfd_layers_destroy"):
        assert hasattr(lib, name)
