"""Seeded gather cases shared by the golden-fixture generator and the tests.

Each case is a recipe (no stored inputs): a host pool filled from a seed or from
the data pattern of a reference test/example, and an entry list whose dst values are
byte offsets into a contiguous output.  The reference patterns are:
  ex02        examples/02_direct_transfer.cu:50-54   1024 x 4 KiB at 2x stride, token i = byte i&0xFF
  sg_e2e      test/test_sg_e2e.cu:42-44              4 x 4 KiB, float i+1, contiguous source
  sg_gpu      test/test_sg_gpu_submit.cu:181-191     4 lists x 8 x 4 KiB, linear source
  db_tiles    test/test_db_small_tiles.cu:44-49      token t = 256 floats of (t+1)
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

# Cases run through the reference's parallel_gather.  Every dst offset is a multiple
# of 64 bytes: the reference's streaming copy (_mm512_stream_si512,
# src/parallel_gather.cpp:17-19) faults on staging addresses that are not 64-byte
# aligned, so lists with odd token sizes cannot go through that path (its serial
# branch, src/direct_submit.cpp:129-142, is a plain memcpy).  ODD_CASES cover those
# inputs against the restated memcpy semantics only.
CASES = [
    {"name": "ex02_1024x4KiB_stride2", "kind": "byte_index", "n": 1024, "size": 4096, "stride": 8192, "workers": 7},
    {"name": "sg_e2e_4x4KiB_float", "kind": "float_index", "n": 4, "size": 4096, "stride": 4096, "workers": 0},
    {"name": "sg_gpu_32x4KiB_float", "kind": "float_index", "n": 32, "size": 4096, "stride": 4096, "workers": 3},
    {"name": "db_tiles_7x1KiB_token_value", "kind": "token_value", "n": 7, "size": 1024, "stride": 1024, "workers": 2},
    {"name": "cfg1_256x4KiB_stride2_seed1", "kind": "random", "n": 256, "size": 4096, "stride": 8192, "seed": 1, "workers": 15},
    {"name": "small_2048x512B_stride2_seed13", "kind": "random", "n": 2048, "size": 512, "stride": 1024, "seed": 13, "workers": 15},
    {"name": "kv_16x64KiB_perm_seed14", "kind": "kv", "n": 16, "size": 65536, "pool_blocks": 64, "seed": 14, "workers": 5},
]

ODD_CASES = [
    {"name": "odd_100_sizes_seed12", "kind": "odd", "n": 100, "pool": 1 << 20, "seed": 12, "workers": 0},
]

_ORACLE = None


def oracle():
    """The C oracle (oracle/_build/libgfd_oracle.so); builds it on first use."""
    global _ORACLE
    if _ORACLE is None:
        path = os.path.join(ROOT, "oracle", "_build", "libgfd_oracle.so")
        if not os.path.exists(path):
            import subprocess
            subprocess.check_call(["make", "-C", os.path.join(ROOT, "oracle"), "_build/libgfd_oracle.so"],
                                  stdout=subprocess.DEVNULL)
        lib = ctypes.CDLL(path)
        lib.gfd_oracle_gather.argtypes = [ctypes.c_void_p, ctypes.c_uint64, ctypes.c_uint64,
                                          ctypes.c_void_p, ctypes.c_int64]
        lib.gfd_oracle_gather.restype = ctypes.c_int64
        lib.gfd_oracle_checksum.argtypes = [ctypes.c_void_p, ctypes.c_uint64]
        lib.gfd_oracle_checksum.restype = ctypes.c_uint64
        lib.gfd_oracle_checksum_records.argtypes = [ctypes.c_void_p, ctypes.c_uint64, ctypes.c_uint64,
                                                    ctypes.c_void_p]
        lib.gfd_oracle_checksum_records.restype = ctypes.c_uint64
        lib.gfd_oracle_checksum_entries.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p]
        lib.gfd_oracle_checksum_entries.restype = None
        lib.gfd_oracle_moe_route.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_int,
                                             ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
        lib.gfd_oracle_moe_route.restype = ctypes.c_int
        lib.gfd_oracle_rms_scale.argtypes = [ctypes.c_void_p, ctypes.c_uint64, ctypes.c_float]
        lib.gfd_oracle_rms_scale.restype = ctypes.c_float
        lib.gfd_oracle_layer_pipeline.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                                  ctypes.c_uint64, ctypes.c_void_p, ctypes.c_uint64,
                                                  ctypes.c_uint64, ctypes.c_float]
        lib.gfd_oracle_layer_pipeline.restype = ctypes.c_int64
        _ORACLE = lib
    return _ORACLE


def checksum(a: np.ndarray) -> int:
    a = np.ascontiguousarray(a)
    return int(oracle().gfd_oracle_checksum(a.ctypes.data, a.nbytes))


def checksum_py(b: bytes) -> int:
    """Pure-Python restatement of gfd_oracle_checksum (for cross-checking the C code)."""
    h = 0xCBF29CE484222325
    m = (1 << 64) - 1
    n = len(b)
    pad = b + bytes((-n) % 8)
    for i in range(0, len(pad), 8):
        h ^= int.from_bytes(pad[i:i + 8], "little")
        h = (h * 0x100000001B3) & m
    h ^= n
    return (h * 0x100000001B3) & m


def aligned_zeros(nbytes: int, align: int = 4096) -> np.ndarray:
    raw = np.zeros(nbytes + align, dtype=np.uint8)
    off = (-raw.ctypes.data) % align
    return raw[off:off + nbytes]


def oracle_gather(out: np.ndarray, out_base: int, entries: np.ndarray) -> int:
    e = np.ascontiguousarray(entries)
    return int(oracle().gfd_oracle_gather(out.ctypes.data, out_base, out.nbytes, e.ctypes.data, len(e)))


def oracle_moe_route(logits: np.ndarray, k: int):
    """Top-k routing + per-expert row order (oracle/route_ref.c).

    Returns (sel [tokens, k] uint16, counts, offsets, row_token int64[tokens * k])."""
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    tokens, experts = logits.shape
    sel = np.zeros((tokens, k), np.uint16)
    counts = np.zeros(experts, np.uint32)
    offsets = np.zeros(experts, np.uint32)
    row_token = np.zeros(tokens * k, np.int64)
    rc = oracle().gfd_oracle_moe_route(logits.ctypes.data, tokens, experts, k, sel.ctypes.data,
                                       counts.ctypes.data, offsets.ctypes.data, row_token.ctypes.data)
    assert rc == 0, "bad routing shape"
    return sel, counts, offsets, row_token


def oracle_layer_pipeline(pool_u16: np.ndarray, table: np.ndarray, block_bytes: int, eps: float = 1e-6):
    """RMS-scaled page-table fetch (oracle/route_ref.c).  Returns (out uint16, ss float32, first_bad)."""
    pool_u16 = np.ascontiguousarray(pool_u16)
    table = np.ascontiguousarray(table, dtype=np.uint32)
    n = block_bytes // 2
    out = np.zeros(len(table) * n, np.uint16)
    ss = np.zeros(len(table), np.float32)
    bad = oracle().gfd_oracle_layer_pipeline(out.ctypes.data, ss.ctypes.data, pool_u16.ctypes.data,
                                             pool_u16.nbytes // block_bytes, table.ctypes.data, len(table),
                                             block_bytes, eps)
    return out, ss, int(bad)


def build_case(spec, pool=None):
    """Returns (pool uint8 array, entries with dst = output offsets, output length).

    `pool` may be a caller-provided uint8 array (e.g. pinned memory) of sufficient size.
    """
    from gfd_b200 import SG_ENTRY_DTYPE
    from gfd_b200 import workloads as wl

    kind = spec["kind"]
    n = spec["n"]
    if kind in ("byte_index", "float_index", "token_value", "random"):
        size, stride = spec["size"], spec["stride"]
        pool_bytes = stride * (n - 1) + size if stride >= size else n * size
        pool_bytes = max(pool_bytes, n * stride)
        if pool is None:
            pool = np.zeros(pool_bytes, dtype=np.uint8)
        pool = pool[:pool_bytes]
        src_off = np.arange(n, dtype=np.uint64) * np.uint64(stride)
        sizes = np.full(n, size, dtype=np.uint64)
        if kind == "byte_index":
            for i in range(n):
                pool[i * stride:i * stride + size] = i & 0xFF
        elif kind == "float_index":
            f = pool[:n * size].view(np.float32)
            f[:] = np.arange(1, f.shape[0] + 1, dtype=np.float32)
        elif kind == "token_value":
            for t in range(n):
                pool[t * stride:t * stride + size].view(np.float32)[:] = float(t + 1)
        else:
            wl.fill_bytes(pool.ctypes.data, pool.nbytes, spec["seed"])
    elif kind == "odd":
        pool_bytes = spec["pool"]
        if pool is None:
            pool = np.zeros(pool_bytes, dtype=np.uint8)
        pool = pool[:pool_bytes]
        wl.fill_bytes(pool.ctypes.data, pool.nbytes, spec["seed"])
        rng = np.random.default_rng(spec["seed"])
        sizes = rng.integers(1, 5000, size=n).astype(np.uint64)
        src_off = np.array([rng.integers(0, pool_bytes - int(s)) for s in sizes], dtype=np.uint64)
    elif kind == "kv":
        size = spec["size"]
        pool_bytes = spec["pool_blocks"] * size
        if pool is None:
            pool = np.zeros(pool_bytes, dtype=np.uint8)
        pool = pool[:pool_bytes]
        wl.fill_bf16_normal(pool.ctypes.data, pool_bytes // 2, spec["seed"])
        perm = wl.permutation(spec["pool_blocks"], spec["seed"])
        src_off = perm[:n].astype(np.uint64) * np.uint64(size)
        sizes = np.full(n, size, dtype=np.uint64)
    else:
        raise ValueError(kind)
    dst_off = np.concatenate([[0], np.cumsum(sizes)[:-1]]).astype(np.uint64)
    e = np.empty(n, dtype=SG_ENTRY_DTYPE)
    e["dst"] = dst_off
    e["src"] = np.uint64(pool.ctypes.data) + src_off
    e["size"] = sizes
    return pool, e, int(sizes.sum())
