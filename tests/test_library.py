"""libgfd_b200.so loads without a GPU and exports every symbol gfd_b200.h declares."""
import ctypes
import os

import gfd_b200


def test_library_exports_declared_symbols():
    lib = gfd_b200.load()
    declared = gfd_b200.declared_symbols()
    assert len(declared) >= 20
    missing = [s for s in declared if not hasattr(lib, s)]
    assert missing == []


def test_python_signatures_cover_header():
    declared = set(gfd_b200.declared_symbols())
    assert declared == set(gfd_b200._SIGS)


def test_ctx_create_fails_cleanly_without_gpu():
    import torch
    if torch.cuda.is_available():
        return
    lib = gfd_b200.load()
    h = ctypes.c_void_p()
    rc = lib.gfd_ctx_create(0, ctypes.byref(h))
    assert rc == gfd_b200.GFD_ERR_CUDA
    assert not h.value


def test_null_arguments_rejected():
    lib = gfd_b200.load()
    assert lib.gfd_ctx_create(0, None) == gfd_b200.GFD_ERR_INVALID
    assert lib.gfd_gather(None, None, 0, None, 0) == gfd_b200.GFD_ERR_INVALID
    assert lib.gfd_ctx_destroy(None) == gfd_b200.GFD_OK
    assert lib.gfd_ctx_device(None) == -1


def test_workload_generators_deterministic():
    import numpy as np
    from gfd_b200 import workloads as wl
    a = np.zeros(3 << 20, np.uint8)
    b = np.zeros(3 << 20, np.uint8)
    wl.fill_bytes(a.ctypes.data, a.nbytes, 7, threads=1)
    wl.fill_bytes(b.ctypes.data, b.nbytes, 7, threads=5)
    assert np.array_equal(a, b) and a.any()
    p = wl.permutation(1000, 3)
    assert sorted(p.tolist()) == list(range(1000)) and not np.array_equal(p, np.arange(1000))
    x = np.zeros(1 << 20, np.uint16)
    wl.fill_bf16_normal(x.ctypes.data, x.size, 2)
    f = (x.astype(np.uint32) << 16).view(np.float32)
    assert abs(float(f.mean())) < 0.01 and abs(float(f.std()) - 1.0) < 0.01


def test_python_constants_match_header():
    """The binding's status codes and gather flags carry the values gfd_b200.h defines."""
    import re
    hdr = open(os.path.join(os.path.dirname(gfd_b200.LIB_PATH), "..", "include", "gfd_b200.h")).read()
    flags = {m.group(1): int(m.group(2)) for m in re.finditer(r"#define GFD_GATHER_(\w+) (\d+)u", hdr)}
    assert {"DEFAULT", "FORCE_CE", "AUTO_CE", "TRUSTED", "FORCE_PULL", "BULK_STAGE", "PEER_DST",
            "PAGEABLE"} <= set(flags)
    for name, value in flags.items():
        assert getattr(gfd_b200, "GATHER_" + name) == value, name
    codes = {m.group(1): int(m.group(2)) for m in re.finditer(r"GFD_(OK|ERR_\w+) = (\d+)", hdr)}
    assert len(codes) == 7
    for name, value in codes.items():
        assert getattr(gfd_b200, "GFD_" + name) == value, name
