"""The CPU oracle agrees with the reference's own gather on every golden case."""
import json
import os

import numpy as np
import pytest

from tests.golden.cases import (CASES, ODD_CASES, aligned_zeros, build_case, checksum,
                                checksum_py, oracle_gather)

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLD = json.load(open(os.path.join(ROOT, "tests", "golden", "gather_cases.json")))["cases"]
REF_CPU = os.path.join(ROOT, "oracle", "_ref", "libgfd_ref_cpu.so")


def test_checksum_c_matches_python():
    rng = np.random.default_rng(0)
    for n in (0, 1, 7, 8, 9, 63, 64, 1000):
        b = rng.integers(0, 256, n, dtype=np.uint8)
        assert checksum(b) == checksum_py(b.tobytes())


@pytest.mark.parametrize("rec", GOLD, ids=[r["name"] for r in GOLD])
def test_oracle_matches_reference_golden(rec):
    spec = next(c for c in CASES if c["name"] == rec["name"])
    pool, entries, out_len = build_case(spec)
    assert out_len == rec["out_len"]
    out = aligned_zeros(out_len)
    e = entries.copy()
    e["dst"] += np.uint64(out.ctypes.data)
    assert oracle_gather(out, out.ctypes.data, e) == -1
    assert "%016x" % checksum(out) == rec["checksum"]
    per = ["%016x" % checksum(out[int(d):int(d) + int(s)]) for d, s in zip(entries["dst"], entries["size"])]
    assert per == rec["token_checksums"]
    if "bytes_hex" in rec:
        assert out.tobytes().hex() == rec["bytes_hex"]


def test_reference_patterns_known_answers():
    # examples/02_direct_transfer.cu:117-129: token i must be all bytes i & 0xFF
    spec = CASES[0]
    pool, entries, out_len = build_case(spec)
    out = np.zeros(out_len, np.uint8)
    e = entries.copy()
    e["dst"] += np.uint64(out.ctypes.data)
    oracle_gather(out, out.ctypes.data, e)
    tok = out.reshape(spec["n"], spec["size"])
    assert np.all(tok == (np.arange(spec["n"]) & 0xFF)[:, None])
    # test/test_sg_e2e.cu:129-140: output floats are i + 1
    spec = CASES[1]
    pool, entries, out_len = build_case(spec)
    out = np.zeros(out_len, np.uint8)
    e = entries.copy()
    e["dst"] += np.uint64(out.ctypes.data)
    oracle_gather(out, out.ctypes.data, e)
    assert np.array_equal(out.view(np.float32), np.arange(1, out_len // 4 + 1, dtype=np.float32))


def test_oracle_rejects_entries_outside_window():
    pool = np.arange(256, dtype=np.uint8)
    out = np.zeros(64, np.uint8)
    from gfd_b200 import entries_array
    e = entries_array([out.ctypes.data + 32], [pool.ctypes.data], 64)  # runs 32 bytes past the end
    assert oracle_gather(out, out.ctypes.data, e) == 0
    assert not out.any()


@pytest.mark.parametrize("spec", ODD_CASES, ids=[c["name"] for c in ODD_CASES])
def test_oracle_odd_sizes_are_memcpy(spec):
    pool, entries, out_len = build_case(spec)
    out = np.zeros(out_len, np.uint8)
    e = entries.copy()
    e["dst"] += np.uint64(out.ctypes.data)
    assert oracle_gather(out, out.ctypes.data, e) == -1
    for d, s, src in zip(entries["dst"], entries["size"], entries["src"]):
        off = int(src) - pool.ctypes.data
        assert np.array_equal(out[int(d):int(d) + int(s)], pool[off:off + int(s)])


@pytest.mark.skipif(not os.path.exists(REF_CPU), reason="reference not built here (make -C oracle)")
def test_reference_gather_live_matches_oracle():
    """Runs the reference's parallel_gather (compiled from its sources) right now."""
    import ctypes
    lib = ctypes.CDLL(REF_CPU)
    lib.ref_parallel_gather.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p,
                                        ctypes.c_uint64, ctypes.c_int]
    for spec in CASES:
        pool, entries, out_len = build_case(spec)
        a, b = aligned_zeros(out_len), aligned_zeros(out_len)
        ea, eb = entries.copy(), entries.copy()
        ea["dst"] += np.uint64(a.ctypes.data)
        eb["dst"] += np.uint64(b.ctypes.data)
        assert lib.ref_parallel_gather(ea.ctypes.data, len(ea), a.ctypes.data, a.ctypes.data, 15) == 0
        oracle_gather(b, b.ctypes.data, eb)
        assert np.array_equal(a, b), spec["name"]


@pytest.mark.skipif(not os.path.exists(REF_CPU), reason="reference not built here (make -C oracle)")
def test_reference_harness_generators_match_the_package():
    """The benchmark's reference arm draws its inputs from the generators linked into the
    reference harness; they must produce the package's bytes and permutations."""
    from gfd_b200 import workloads as wl
    want_perm = wl.permutation(65536, 2)
    want_bf16 = np.zeros(3 << 19, np.uint16)
    wl.fill_bf16_normal(want_bf16.ctypes.data, want_bf16.size, 2)
    want_bytes = np.zeros(3 << 20, np.uint8)
    wl.fill_bytes(want_bytes.ctypes.data, want_bytes.nbytes, 3)
    saved = wl._WL
    try:
        wl.use_generator_library(REF_CPU)
        got_bf16 = np.zeros_like(want_bf16)
        wl.fill_bf16_normal(got_bf16.ctypes.data, got_bf16.size, 2)
        got_bytes = np.zeros_like(want_bytes)
        wl.fill_bytes(got_bytes.ctypes.data, got_bytes.nbytes, 3)
        assert np.array_equal(wl.permutation(65536, 2), want_perm)
        assert np.array_equal(got_bf16, want_bf16) and np.array_equal(got_bytes, want_bytes)
    finally:
        wl._WL = saved
