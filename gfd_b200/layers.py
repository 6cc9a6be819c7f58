"""Layer pipeline: page-table KV fetch with dependent compute (libgfd_layers.so).

One pass covers every layer: block g of the pass is read from pool block table[g] by
the producer warps of a WarpSpecSession kernel and, in mode RMS, scaled in place by the
compute warps of the same CTAs (per-block fp32 sum of squares, x * 1/sqrt(ss/n + eps),
bf16 round to nearest even).  The library is a client of libgfd_b200.so through the
C++ session API in include/gfd/warp_spec_session.h.
"""
from __future__ import annotations

import ctypes
import os

from . import load

_PKG = os.path.dirname(os.path.abspath(__file__))
LAYERS_PATH = os.path.join(_PKG, "libgfd_layers.so")
_VP = ctypes.c_void_p
_lib = None

TRANSFER = 0  # producers only
RMS = 1       # producers + RmsScale compute warps


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LAYERS_PATH):
            raise RuntimeError(f"{LAYERS_PATH} missing: run `python -m gfd_b200.build`")
        load()  # libgfd_b200.so first, from its own path
        l = ctypes.CDLL(LAYERS_PATH)
        l.gfd_layers_create.argtypes = [_VP, ctypes.c_uint64, _VP, ctypes.c_uint32, ctypes.c_uint32, _VP, _VP, ctypes.c_uint32,
                                        ctypes.c_int, ctypes.c_int, ctypes.c_uint64, ctypes.POINTER(_VP)]
        l.gfd_layers_create.restype = ctypes.c_int
        l.gfd_layers_run.argtypes = [_VP, ctypes.c_int, _VP]
        l.gfd_layers_run.restype = ctypes.c_int
        l.gfd_layers_sync.argtypes = [_VP] + [ctypes.POINTER(ctypes.c_uint64)] * 3
        l.gfd_layers_sync.restype = ctypes.c_int
        l.gfd_layers_block_threads.argtypes = [_VP]
        l.gfd_layers_block_threads.restype = ctypes.c_int
        l.gfd_layers_destroy.argtypes = [_VP]
        l.gfd_layers_destroy.restype = None
        _lib = l
    return _lib


class LayerPipeline:
    def __init__(self, pool_ptr: int, pool_bytes: int, d_table: int, total_blocks: int, block_bytes: int,
                 d_dst: int, d_ss: int = 0, tokens_per_tile: int = 32, producer_warps: int = 0,
                 double_buffer: bool = False, wait_timeout_ms: int = 0):
        self.lib = lib()
        h = _VP()
        rc = self.lib.gfd_layers_create(_VP(pool_ptr), pool_bytes, _VP(d_table), total_blocks, block_bytes, _VP(d_dst),
                                        _VP(d_ss or None), tokens_per_tile, producer_warps, int(double_buffer),
                                        wait_timeout_ms, ctypes.byref(h))
        if rc != 0 or not h.value:
            raise RuntimeError("gfd_layers_create failed (see stderr)")
        self.handle = h
        self.total_blocks = total_blocks
        self.block_bytes = block_bytes

    @property
    def block_threads(self) -> int:
        return self.lib.gfd_layers_block_threads(self.handle)

    def run(self, mode: int = RMS, stream: int = 0):
        if self.lib.gfd_layers_run(self.handle, mode, _VP(stream)) != 0:
            raise RuntimeError("gfd_layers_run: launch failed")

    def sync(self):
        """Waits for the pass; returns (rejected tokens, timed-out waits, bytes landed)."""
        r, t, b = ctypes.c_uint64(), ctypes.c_uint64(), ctypes.c_uint64()
        self.lib.gfd_layers_sync(self.handle, ctypes.byref(r), ctypes.byref(t), ctypes.byref(b))
        return r.value, t.value, b.value

    def close(self):
        if self.handle:
            self.lib.gfd_layers_destroy(self.handle)
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()
