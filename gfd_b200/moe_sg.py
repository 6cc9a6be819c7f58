"""MoE gather through SGWarpSpecSession with GPU-submitted lists (libgfd_moe_sg.so).

Routing runs first (Context.moe_route_gather(..., route_only=True) writes the
per-expert entry list, counts and offsets on the device); then one SG-framework kernel
pulls the lists while a submitter warp in the same kernel feeds them through the
session's task queue, one list per expert in ascending expert order.
"""
from __future__ import annotations

import ctypes
import os

from . import GFD_OK, load

_PKG = os.path.dirname(os.path.abspath(__file__))
MOE_SG_PATH = os.path.join(_PKG, "libgfd_moe_sg.so")
_VP = ctypes.c_void_p
_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(MOE_SG_PATH):
            raise RuntimeError(f"{MOE_SG_PATH} missing: run `python -m gfd_b200.build`")
        load()
        l = ctypes.CDLL(MOE_SG_PATH)
        l.gfd_moe_sg_create.argtypes = [ctypes.c_int, ctypes.c_uint64, ctypes.c_int, ctypes.POINTER(_VP)]
        l.gfd_moe_sg_prepare.argtypes = [_VP]
        l.gfd_moe_sg_run.argtypes = [_VP, _VP, _VP, _VP, ctypes.c_uint32, ctypes.c_uint32, _VP]
        l.gfd_moe_sg_sync.argtypes = [_VP, ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(ctypes.c_uint64)]
        l.gfd_moe_sg_destroy.argtypes = [_VP]
        for f in ("gfd_moe_sg_create", "gfd_moe_sg_prepare", "gfd_moe_sg_run", "gfd_moe_sg_sync"):
            getattr(l, f).restype = ctypes.c_int
        l.gfd_moe_sg_destroy.restype = None
        _lib = l
    return _lib


class MoESG:
    def __init__(self, producer_warps: int = 0, wait_timeout_ms: int = 0, num_blocks: int = 0):
        """num_blocks: CTAs of the SG kernel (0: one per SM)."""
        self.lib = lib()
        h = _VP()
        if self.lib.gfd_moe_sg_create(producer_warps, wait_timeout_ms, num_blocks, ctypes.byref(h)) != GFD_OK:
            raise RuntimeError("gfd_moe_sg_create failed (see stderr)")
        self.handle = h

    def prepare(self):
        if self.lib.gfd_moe_sg_prepare(self.handle) != GFD_OK:
            raise RuntimeError("gfd_moe_sg_prepare failed")

    def run(self, d_entries: int, d_counts: int, d_offsets: int, experts: int, stream: int = 0,
            rows_per_list: int = 0):
        """rows_per_list: split each expert into lists of at most this many rows (0: one list
        per expert)."""
        rc = self.lib.gfd_moe_sg_run(self.handle, _VP(d_entries), _VP(d_counts), _VP(d_offsets), experts,
                                     rows_per_list, _VP(stream))
        if rc != GFD_OK:
            raise RuntimeError(f"gfd_moe_sg_run: {rc}")

    def sync(self):
        """Waits for the pass; returns (timed-out waits, payload bytes moved)."""
        t, b = ctypes.c_uint64(), ctypes.c_uint64()
        rc = self.lib.gfd_moe_sg_sync(self.handle, ctypes.byref(t), ctypes.byref(b))
        return rc, t.value, b.value

    def close(self):
        if self.handle:
            self.lib.gfd_moe_sg_destroy(self.handle)
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()
