"""Seeded synthetic workloads with the shapes of the benchmark configurations.

cfg1  256 tokens x 4 KiB, uniform random bytes (seed 1), pool of 512 slots, token i
      at slot 2i (2x stride), gathered into one contiguous 1 MiB buffer.
cfg2  KV block fetch: 65,536 blocks x 64 KiB (4 GiB pool), block = bf16
      [16 tok][8 heads][128 dim][K,V] ~ N(0,1) (seed 2); 2048 blocks chosen by a
      Fisher-Yates permutation (seed 2), gathered contiguously in index order.
cfg3  token-size sweep: 2048 tokens x {512 B .. 64 KiB} and {16 .. 8192} tokens x
      4 KiB, uniform random bytes, 2x stride.
cfg4  layer pipeline: 32 layers x 1024 blocks of 64 KiB from the cfg2-shaped pool
      (seed 4); layer l uses the first 1024 ids of a permutation seeded 4 + l.
cfg5  MoE gather: per GPU g, fp32 logits [4096 x 64] ~ N(0,1) (seed 5+g), top-8
      routing, pool of 262,144 rows x 7168 bf16 ~ N(0, 0.02) (seed 50+g), token t's
      row = perm[t] (seed 500+g), rows grouped per expert in ascending token order.

The benchmark data is synthetic and seeded; no external dataset is used.  Generators
live in libgfd_workload.so (xoshiro256** seeded by splitmix64, independent 1 MiB
blocks so results do not depend on the thread count).
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass
from typing import Optional

import numpy as np

from . import SG_ENTRY_DTYPE, entries_array

_PKG = os.path.dirname(os.path.abspath(__file__))
_WL = None


def use_generator_library(path: str):
    """Takes the generators from another library that exports the same gfdw_* functions
    (the benchmark's reference arm uses the copy linked into the reference harness, so
    it loads no library of this package).  Call before the first generator use."""
    global _WL
    _WL = _bind(ctypes.CDLL(path))


def wl():
    global _WL
    if _WL is None:
        p = os.path.join(_PKG, "libgfd_workload.so")
        if not os.path.exists(p):
            raise RuntimeError(f"{p} missing: run `python -m gfd_b200.build`")
        _WL = _bind(ctypes.CDLL(p))
    return _WL


def _bind(lib):
    lib.gfdw_fill_bytes.argtypes = [ctypes.c_void_p, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_int]
    lib.gfdw_fill_bf16_normal.argtypes = [ctypes.c_void_p, ctypes.c_uint64, ctypes.c_uint64,
                                          ctypes.c_double, ctypes.c_double, ctypes.c_int]
    lib.gfdw_fill_f32_normal.argtypes = [ctypes.c_void_p, ctypes.c_uint64, ctypes.c_uint64,
                                         ctypes.c_double, ctypes.c_double, ctypes.c_int]
    lib.gfdw_permutation.argtypes = [ctypes.c_void_p, ctypes.c_uint32, ctypes.c_uint64]
    for f in ("gfdw_fill_bytes", "gfdw_fill_bf16_normal", "gfdw_fill_f32_normal", "gfdw_permutation"):
        getattr(lib, f).restype = None
    return lib


def default_threads() -> int:
    n = os.cpu_count() or 1
    local = int(os.environ.get("LOCAL_WORLD_SIZE", "1"))
    return max(1, n // max(1, local))


def fill_bytes(ptr: int, nbytes: int, seed: int, threads: Optional[int] = None):
    wl().gfdw_fill_bytes(ctypes.c_void_p(ptr), nbytes, seed, threads or default_threads())


def fill_bf16_normal(ptr: int, count: int, seed: int, mean: float = 0.0, std: float = 1.0,
                     threads: Optional[int] = None):
    wl().gfdw_fill_bf16_normal(ctypes.c_void_p(ptr), count, seed, mean, std,
                               threads or default_threads())


def fill_f32_normal(ptr: int, count: int, seed: int, mean: float = 0.0, std: float = 1.0,
                    threads: Optional[int] = None):
    wl().gfdw_fill_f32_normal(ctypes.c_void_p(ptr), count, seed, mean, std,
                              threads or default_threads())


def permutation(n: int, seed: int) -> np.ndarray:
    out = np.empty(n, dtype=np.uint32)
    wl().gfdw_permutation(out.ctypes.data_as(ctypes.c_void_p), n, seed)
    return out


def fill_array_bytes(a: np.ndarray, seed: int):
    fill_bytes(a.ctypes.data, a.nbytes, seed)


# ---------------------------------------------------------------------------
# Configurations: each returns the pool size and a function that builds entries
# from the pool's base address and the destination base address.
# ---------------------------------------------------------------------------
@dataclass
class Workload:
    name: str
    pool_bytes: int
    dst_bytes: int
    num_tokens: int
    token_size: int
    kind: str  # "bytes" or "bf16"
    seed: int
    stride: int = 0             # 2x-stride layouts: bytes between token starts
    block_ids: Optional[np.ndarray] = None

    def fill_pool(self, pool_ptr: int, threads: Optional[int] = None):
        if self.kind == "bytes":
            fill_bytes(pool_ptr, self.pool_bytes, self.seed, threads)
        else:
            fill_bf16_normal(pool_ptr, self.pool_bytes // 2, self.seed, 0.0, 1.0, threads)

    def src_offsets(self) -> np.ndarray:
        if self.block_ids is not None:
            return self.block_ids.astype(np.uint64) * np.uint64(self.token_size)
        return np.arange(self.num_tokens, dtype=np.uint64) * np.uint64(self.stride)

    def entries(self, pool_ptr: int, dst_ptr: int) -> np.ndarray:
        src = np.uint64(pool_ptr) + self.src_offsets()
        dst = np.uint64(dst_ptr) + np.arange(self.num_tokens, dtype=np.uint64) * np.uint64(self.token_size)
        return entries_array(dst, src, self.token_size)

    @property
    def total_bytes(self) -> int:
        return self.num_tokens * self.token_size


def cfg1() -> Workload:
    return Workload("cfg1_256x4KiB_stride2", pool_bytes=512 * 4096, dst_bytes=256 * 4096,
                    num_tokens=256, token_size=4096, kind="bytes", seed=1, stride=2 * 4096)


def cfg2(num_blocks: int = 2048, pool_blocks: int = 65536, seed: int = 2) -> Workload:
    perm = permutation(pool_blocks, seed)
    return Workload("cfg2_kv_2048x64KiB_4GiB_pool", pool_bytes=pool_blocks * 65536,
                    dst_bytes=num_blocks * 65536, num_tokens=num_blocks, token_size=65536,
                    kind="bf16", seed=seed, block_ids=perm[:num_blocks].copy())


def cfg3(num_tokens: int, token_size: int, seed: int = 3) -> Workload:
    return Workload(f"cfg3_{num_tokens}x{token_size}B_stride2", pool_bytes=2 * num_tokens * token_size,
                    dst_bytes=num_tokens * token_size, num_tokens=num_tokens, token_size=token_size,
                    kind="bytes", seed=seed, stride=2 * token_size)


CFG3_SIZES = [512, 1024, 2048, 4096, 8192, 16384, 32768, 65536]
CFG3_COUNTS = [16, 64, 256, 1024, 2048, 4096, 8192]


# ---------------------------------------------------------------------------
# cfg4: layer pipeline (page-table fetch + RMS scale)
# ---------------------------------------------------------------------------
CFG4_LAYERS = 32
CFG4_BLOCKS_PER_LAYER = 1024
CFG4_BLOCK_BYTES = 65536
CFG4_POOL_BLOCKS = 65536


def cfg4_table(layers: int = CFG4_LAYERS, per_layer: int = CFG4_BLOCKS_PER_LAYER,
               pool_blocks: int = CFG4_POOL_BLOCKS, seed: int = 4) -> np.ndarray:
    """Page table of the whole pass: layer l's blocks are the first `per_layer` ids of a
    permutation of the pool seeded seed + l (distinct within a layer)."""
    return np.concatenate([permutation(pool_blocks, seed + l)[:per_layer] for l in range(layers)])


def cfg4_fill_pool(pool_ptr: int, pool_blocks: int = CFG4_POOL_BLOCKS, block_bytes: int = CFG4_BLOCK_BYTES,
                   seed: int = 4, threads: Optional[int] = None):
    fill_bf16_normal(pool_ptr, pool_blocks * block_bytes // 2, seed, 0.0, 1.0, threads)


# ---------------------------------------------------------------------------
# cfg5: MoE routing + per-expert gather, one independent shard per GPU
# ---------------------------------------------------------------------------
CFG5_TOKENS = 4096
CFG5_EXPERTS = 64
CFG5_TOPK = 8
CFG5_ROW_BYTES = 7168 * 2
CFG5_POOL_ROWS = 262144


@dataclass
class MoEShard:
    gpu: int
    tokens: int = CFG5_TOKENS
    experts: int = CFG5_EXPERTS
    k: int = CFG5_TOPK
    row_bytes: int = CFG5_ROW_BYTES
    pool_rows: int = CFG5_POOL_ROWS

    @property
    def pool_bytes(self) -> int:
        return self.pool_rows * self.row_bytes

    @property
    def dst_bytes(self) -> int:
        return self.tokens * self.k * self.row_bytes

    def logits(self) -> np.ndarray:
        out = np.empty((self.tokens, self.experts), np.float32)
        fill_f32_normal(out.ctypes.data, out.size, 5 + self.gpu, 0.0, 1.0)
        return out

    def fill_pool(self, pool_ptr: int, threads: Optional[int] = None):
        fill_bf16_normal(pool_ptr, self.pool_bytes // 2, 50 + self.gpu, 0.0, 0.02, threads)

    def token_rows(self) -> np.ndarray:
        """Pool row of each token: the first `tokens` ids of a permutation seeded 500 + gpu."""
        return permutation(self.pool_rows, 500 + self.gpu)[:self.tokens].copy()

    def token_src(self, pool_ptr: int) -> np.ndarray:
        return np.uint64(pool_ptr) + self.token_rows().astype(np.uint64) * np.uint64(self.row_bytes)
