"""Python binding of libgfd_b200 (the C ABI in include/gfd_b200.h) via ctypes.

The data path is the CUDA library; this module only marshals arguments.  Importing
it does not need a GPU; creating a Context does.  If the shared library has not been
built, load() raises -- there is no CPU fallback.
"""
from __future__ import annotations

import ctypes
import os
from typing import Optional, Sequence

import numpy as np

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "libgfd_b200.so")

GFD_OK = 0
GFD_ERR_INVALID = 1
GFD_ERR_TIMEOUT = 2
GFD_ERR_CUDA = 3
GFD_ERR_NOMEM = 4
GFD_ERR_UNSUPPORTED = 5
GFD_ERR_STATE = 6

GATHER_DEFAULT = 0
GATHER_FORCE_CE = 1
GATHER_AUTO_CE = 2
GATHER_TRUSTED = 4
GATHER_FORCE_PULL = 8
GATHER_BULK_STAGE = 16
GATHER_PEER_DST = 32
GATHER_PAGEABLE = 64  # gfd_gather(_sync): pageable sources go to the copy engine
MOE_ROUTE_ONLY = 1  # gfd_moe_route_gather flag

# numpy view of gfd_sg_entry / gfd::SGEntry: {uint64 dst; const void* src; size_t size}
SG_ENTRY_DTYPE = np.dtype([("dst", "<u8"), ("src", "<u8"), ("size", "<u8")])
assert SG_ENTRY_DTYPE.itemsize == 24


class GfdError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"gfd error {code}: {msg}")
        self.code = code


class _Stats(ctypes.Structure):
    _fields_ = [(n, ctypes.c_uint64) for n in
                ("calls", "entries", "bytes", "pull_launches", "ce_copies", "rejected", "prep_ns",
                 "launch_ns", "wait_ns")]


_lib = None

# exported C symbols and their signatures (argtypes, restype)
_VP = ctypes.c_void_p
_SIGS = {
    "gfd_ctx_create": ([ctypes.c_int, ctypes.POINTER(_VP)], ctypes.c_int),
    "gfd_ctx_destroy": ([_VP], ctypes.c_int),
    "gfd_ctx_device": ([_VP], ctypes.c_int),
    "gfd_last_error": ([_VP], ctypes.c_char_p),
    "gfd_set_timeout_ns": ([_VP, ctypes.c_uint64], ctypes.c_int),
    "gfd_set_ce_threshold": ([_VP, ctypes.c_uint64], ctypes.c_int),
    "gfd_get_stats": ([_VP, ctypes.POINTER(_Stats)], ctypes.c_int),
    "gfd_pool_alloc": ([_VP, ctypes.c_size_t, ctypes.c_int, ctypes.POINTER(_VP)], ctypes.c_int),
    "gfd_pool_free": ([_VP, _VP], ctypes.c_int),
    "gfd_pool_register": ([_VP, _VP, ctypes.c_size_t], ctypes.c_int),
    "gfd_pool_unregister": ([_VP, _VP], ctypes.c_int),
    "gfd_pool_numa_node": ([_VP, _VP, ctypes.POINTER(ctypes.c_int)], ctypes.c_int),
    "gfd_gather": ([_VP, _VP, ctypes.c_int64, _VP, ctypes.c_uint32], ctypes.c_int),
    "gfd_gather_sync": ([_VP, _VP, ctypes.c_int64, ctypes.c_uint32,
                         ctypes.POINTER(ctypes.c_double)], ctypes.c_int),
    "gfd_scatter": ([_VP, _VP, ctypes.c_int64, _VP, ctypes.c_uint32], ctypes.c_int),
    "gfd_scatter_sync": ([_VP, _VP, ctypes.c_int64, ctypes.c_uint32,
                          ctypes.POINTER(ctypes.c_double)], ctypes.c_int),
    "gfd_gather_device": ([_VP, _VP, ctypes.c_int64, _VP, ctypes.c_size_t, _VP, ctypes.c_uint32],
                          ctypes.c_int),
    "gfd_gather_device_status": ([_VP, ctypes.POINTER(ctypes.c_int64)], ctypes.c_int),
    "gfd_gather_device_noalloc": ([_VP, ctypes.c_int64, _VP, ctypes.c_size_t, _VP, ctypes.c_size_t, _VP,
                                   _VP], ctypes.c_int),
    "gfd_moe_route_gather": ([_VP, _VP, ctypes.c_int64, ctypes.c_int, ctypes.c_int, _VP, ctypes.c_size_t,
                              _VP, ctypes.c_size_t, _VP, _VP, _VP, _VP, ctypes.c_uint32], ctypes.c_int),
    "gfd_ring_create": ([_VP, _VP, _VP, _VP, ctypes.POINTER(_VP)], ctypes.c_int),
    "gfd_ring_destroy": ([_VP], ctypes.c_int),
    "gfd_ring_start": ([_VP], ctypes.c_int),
    "gfd_ring_stop": ([_VP], ctypes.c_int),
    "gfd_ring_poll": ([_VP, ctypes.POINTER(ctypes.c_int)], ctypes.c_int),
    "gfd_ring_wait": ([_VP, ctypes.c_uint64], ctypes.c_int),
    "gfd_ring_counters": ([_VP, ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(ctypes.c_uint64),
                           ctypes.POINTER(ctypes.c_uint64)], ctypes.c_int),
    "gfd_ring_configure": ([_VP, ctypes.c_uint32, ctypes.c_uint64, ctypes.c_int], ctypes.c_int),
    "gfd_ring_allow": ([_VP, _VP, ctypes.c_size_t], ctypes.c_int),
    "gfd_ring_agent_stats": ([_VP, ctypes.POINTER(ctypes.c_uint64 * 11)], ctypes.c_int),
}


def load(path: Optional[str] = None) -> ctypes.CDLL:
    """Loads libgfd_b200.so (raises if it is missing: build it with gfd_b200.build)."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = path or LIB_PATH
    if not os.path.exists(p):
        raise RuntimeError(f"{p} not found: run `python -m gfd_b200.build` (no CPU fallback exists)")
    lib = ctypes.CDLL(p)  # RTLD_LOCAL: its C++ symbols must not interpose on other libraries
    for name, (args, res) in _SIGS.items():
        fn = getattr(lib, name, None)
        if fn is None:
            continue
        fn.argtypes = args
        fn.restype = res
    if path is None:
        _lib = lib
    return lib


def entries_array(dst, src, size) -> np.ndarray:
    """Builds a gfd_sg_entry array from three integer sequences / arrays."""
    dst = np.asarray(dst, dtype=np.uint64)
    n = dst.shape[0]
    e = np.empty(n, dtype=SG_ENTRY_DTYPE)
    e["dst"] = dst
    e["src"] = np.broadcast_to(np.asarray(src, dtype=np.uint64), (n,))
    e["size"] = np.broadcast_to(np.asarray(size, dtype=np.uint64), (n,))
    return e


class HostPool:
    """Pinned, device-mapped, NUMA-bound host memory owned by a Context."""

    def __init__(self, ctx: "Context", nbytes: int, numa_node: int = -1):
        self.ctx = ctx
        self.nbytes = int(nbytes)
        p = _VP()
        ctx._check(ctx.lib.gfd_pool_alloc(ctx.handle, self.nbytes, numa_node, ctypes.byref(p)))
        self.ptr = int(p.value)

    def array(self, dtype=np.uint8) -> np.ndarray:
        buf = (ctypes.c_uint8 * self.nbytes).from_address(self.ptr)
        return np.frombuffer(buf, dtype=np.uint8).view(dtype)

    @property
    def numa_node(self) -> int:
        """NUMA node the pool is bound to (-1: not bound)."""
        n = ctypes.c_int(-2)
        self.ctx._check(self.ctx.lib.gfd_pool_numa_node(self.ctx.handle, _VP(self.ptr), ctypes.byref(n)))
        return n.value

    def free(self):
        if self.ptr:
            self.ctx._check(self.ctx.lib.gfd_pool_free(self.ctx.handle, _VP(self.ptr)))
            self.ptr = 0


class Context:
    """One GPU.  Thin wrapper over gfd_ctx_* / gfd_gather*."""

    def __init__(self, device: int = 0):
        self.lib = load()
        h = _VP()
        rc = self.lib.gfd_ctx_create(device, ctypes.byref(h))
        if rc != GFD_OK:
            raise GfdError(rc, f"gfd_ctx_create({device}) failed")
        self.handle = h
        self.device = device

    def close(self):
        if self.handle:
            self.lib.gfd_ctx_destroy(self.handle)
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def last_error(self) -> str:
        return self.lib.gfd_last_error(self.handle).decode()

    def _check(self, rc: int):
        if rc != GFD_OK:
            raise GfdError(rc, self.last_error())

    def pool(self, nbytes: int, numa_node: int = -1) -> HostPool:
        return HostPool(self, nbytes, numa_node)

    def register(self, ptr: int, nbytes: int):
        self._check(self.lib.gfd_pool_register(self.handle, _VP(ptr), nbytes))

    def unregister(self, ptr: int):
        self._check(self.lib.gfd_pool_unregister(self.handle, _VP(ptr)))

    def set_timeout_ns(self, ns: int):
        self._check(self.lib.gfd_set_timeout_ns(self.handle, ns))

    def set_ce_threshold(self, nbytes: int):
        self._check(self.lib.gfd_set_ce_threshold(self.handle, nbytes))

    def gather(self, entries: np.ndarray, stream: int = 0, flags: int = 0) -> int:
        """Asynchronous gather on `stream` (0: the context's stream). Returns the raw code."""
        e = np.ascontiguousarray(entries, dtype=SG_ENTRY_DTYPE)
        return self.lib.gfd_gather(self.handle, e.ctypes.data_as(_VP), e.shape[0], _VP(stream), flags)

    def gather_sync(self, entries: np.ndarray, flags: int = 0) -> float:
        """Gathers and waits; returns host latency in microseconds (raises on error)."""
        e = np.ascontiguousarray(entries, dtype=SG_ENTRY_DTYPE)
        us = ctypes.c_double(0.0)
        self._check(self.lib.gfd_gather_sync(self.handle, e.ctypes.data_as(_VP), e.shape[0], flags,
                                             ctypes.byref(us)))
        return us.value

    def gather_sync_rc(self, entries: np.ndarray, flags: int = 0) -> int:
        e = np.ascontiguousarray(entries, dtype=SG_ENTRY_DTYPE)
        us = ctypes.c_double(0.0)
        return self.lib.gfd_gather_sync(self.handle, e.ctypes.data_as(_VP), e.shape[0], flags,
                                        ctypes.byref(us))

    def scatter(self, entries: np.ndarray, stream: int = 0, flags: int = 0) -> int:
        """Asynchronous device -> host scatter on `stream`. Returns the raw code."""
        e = np.ascontiguousarray(entries, dtype=SG_ENTRY_DTYPE)
        return self.lib.gfd_scatter(self.handle, e.ctypes.data_as(_VP), e.shape[0], _VP(stream), flags)

    def scatter_sync(self, entries: np.ndarray, flags: int = 0) -> float:
        """Scatters device bytes into pinned host memory and waits; returns microseconds."""
        e = np.ascontiguousarray(entries, dtype=SG_ENTRY_DTYPE)
        us = ctypes.c_double(0.0)
        self._check(self.lib.gfd_scatter_sync(self.handle, e.ctypes.data_as(_VP), e.shape[0], flags,
                                              ctypes.byref(us)))
        return us.value

    def scatter_sync_rc(self, entries: np.ndarray, flags: int = 0) -> int:
        e = np.ascontiguousarray(entries, dtype=SG_ENTRY_DTYPE)
        us = ctypes.c_double(0.0)
        return self.lib.gfd_scatter_sync(self.handle, e.ctypes.data_as(_VP), e.shape[0], flags,
                                         ctypes.byref(us))

    def gather_device(self, d_entries: int, n: int, dst_base: int, dst_bytes: int,
                      stream: int = 0, flags: int = 0):
        self._check(self.lib.gfd_gather_device(self.handle, _VP(d_entries), n, _VP(dst_base),
                                               dst_bytes, _VP(stream), flags))

    def moe_route_gather(self, d_logits: int, tokens: int, experts: int, k: int, d_token_src: int,
                         row_bytes: int, dst_base: int, dst_bytes: int, d_counts: int, d_offsets: int,
                         d_entries: int, stream: int = 0, route_only: bool = False):
        """Top-k routing over device fp32 logits, then the per-expert gather (all on
        `stream`).  See gfd_moe_route_gather in include/gfd_b200.h."""
        self._check(self.lib.gfd_moe_route_gather(
            self.handle, _VP(d_logits), tokens, experts, k, _VP(d_token_src), row_bytes, _VP(dst_base),
            dst_bytes, _VP(d_counts), _VP(d_offsets), _VP(d_entries), _VP(stream),
            MOE_ROUTE_ONLY if route_only else 0))

    def gather_device_status(self) -> int:
        bad = ctypes.c_int64(-1)
        rc = self.lib.gfd_gather_device_status(self.handle, ctypes.byref(bad))
        return rc, bad.value

    def stats(self) -> dict:
        s = _Stats()
        self._check(self.lib.gfd_get_stats(self.handle, ctypes.byref(s)))
        return {n: getattr(s, n) for n, _ in _Stats._fields_}


# Descriptor ring (include/gfd/descriptor_queue.h): 16384 slots of 64 bytes, then the
# write / read / done indices.
QUEUE_SIZE = 16384
QUEUE_BYTES = QUEUE_SIZE * 64 + 64
FLAG_LAST_IN_BATCH = 1
FLAG_URGENT = 2
DESCRIPTOR_DTYPE = np.dtype([("src", "<u8"), ("dst", "<u8"), ("size", "<u4"), ("flags", "<u4"),
                             ("user", "<u8"), ("seq", "<u8"), ("_pad", "V24")])
assert DESCRIPTOR_DTYPE.itemsize == 64


class DescriptorRing:
    """A descriptor ring in pinned host memory (a HostPool of QUEUE_BYTES) seen from the
    host: `entries` (DESCRIPTOR_DTYPE view) and the three indices.  A host-side producer
    writes a slot's fields, then its `seq` = slot + 1 (the commit marker)."""

    def __init__(self, pool: HostPool):
        if pool.nbytes < QUEUE_BYTES:
            raise ValueError("pool smaller than a DescriptorQueue")
        self.pool = pool
        self.ptr = pool.ptr
        raw = pool.array()[:QUEUE_BYTES]
        raw[:] = 0
        self.entries = raw[:QUEUE_SIZE * 64].view(DESCRIPTOR_DTYPE)
        self._idx = raw[QUEUE_SIZE * 64:QUEUE_SIZE * 64 + 24].view(np.uint64)

    @property
    def write_idx(self) -> int:
        return int(self._idx[0])

    @property
    def read_idx(self) -> int:
        return int(self._idx[1])

    @property
    def done_idx(self) -> int:
        return int(self._idx[2])

    def produce(self, base: int, src, dst, size, flags=None, user=None):
        """Writes descriptors for slots [base, base + n) and commits them in slot order."""
        src = np.asarray(src, dtype=np.uint64)
        n = src.shape[0]
        slots = (base + np.arange(n)) % QUEUE_SIZE
        e = self.entries
        e["src"][slots] = src
        e["dst"][slots] = np.broadcast_to(np.asarray(dst, dtype=np.uint64), (n,))
        e["size"][slots] = np.broadcast_to(np.asarray(size, dtype=np.uint32), (n,))
        e["flags"][slots] = 0 if flags is None else np.broadcast_to(np.asarray(flags, dtype=np.uint32), (n,))
        e["user"][slots] = 0 if user is None else np.broadcast_to(np.asarray(user, dtype=np.uint64), (n,))
        e["seq"][slots] = base + np.arange(n, dtype=np.uint64) + 1


class Ring:
    """This library's consumer of a descriptor ring (gfd_ring_*).  Started, a
    device-resident kernel (the ring agent) consumes the ring; stopped, poll() drains
    what is committed from the calling thread (one pull kernel per run).  `tiled` / `sg`:
    TiledQueue / SGTaskQueue addresses for per-tile / per-list completion (0: none)."""

    def __init__(self, ctx: Context, queue_ptr: int, tiled_ptr: int = 0, sg_ptr: int = 0):
        self.ctx = ctx
        h = _VP()
        ctx._check(ctx.lib.gfd_ring_create(ctx.handle, _VP(queue_ptr), _VP(tiled_ptr or None),
                                           _VP(sg_ptr or None), ctypes.byref(h)))
        self.handle = h

    def configure(self, movers: int = 0, linger_ns: int = 20000, resident: bool = False):
        self.ctx._check(self.ctx.lib.gfd_ring_configure(self.handle, movers, linger_ns, 1 if resident else 0))

    def allow(self, ptr: int, nbytes: int = 0):
        self.ctx._check(self.ctx.lib.gfd_ring_allow(self.handle, _VP(ptr), nbytes))

    def agent_stats(self) -> dict:
        v = (ctypes.c_uint64 * 11)()
        self.ctx._check(self.ctx.lib.gfd_ring_agent_stats(self.handle, ctypes.byref(v)))
        return dict(zip(("launches", "queries", "rejected", "timeouts", "idle_exits", "stop_exits", "error_exits",
                         "resident", "last_first_batch_ns", "last_done_ns", "last_exit_ns"), list(v)))

    def start(self):
        self.ctx._check(self.ctx.lib.gfd_ring_start(self.handle))

    def stop(self):
        self.ctx._check(self.ctx.lib.gfd_ring_stop(self.handle))

    def poll(self) -> int:
        """Drains whatever is committed now; returns the number of drains launched."""
        n = ctypes.c_int(0)
        self.ctx._check(self.ctx.lib.gfd_ring_poll(self.handle, ctypes.byref(n)))
        return n.value

    def wait(self, target: int):
        """Waits (bounded) until done_idx >= target."""
        self.ctx._check(self.ctx.lib.gfd_ring_wait(self.handle, target))

    def counters(self) -> dict:
        c, d, b = ctypes.c_uint64(), ctypes.c_uint64(), ctypes.c_uint64()
        self.ctx._check(self.ctx.lib.gfd_ring_counters(self.handle, ctypes.byref(c), ctypes.byref(d),
                                                       ctypes.byref(b)))
        return {"consumed": c.value, "drains": d.value, "bytes": b.value}

    def close(self):
        if self.handle:
            self.ctx.lib.gfd_ring_destroy(self.handle)
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


def declared_symbols(header: Optional[str] = None) -> Sequence[str]:
    """Names of the functions include/gfd_b200.h declares."""
    import re
    h = header or os.path.join(os.path.dirname(_PKG), "include", "gfd_b200.h")
    text = open(h).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(gfd_[a-z0-9_]+)\s*\(", text)))
