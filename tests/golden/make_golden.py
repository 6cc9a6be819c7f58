"""Regenerates the golden fixtures in tests/golden/ from the reference itself.

Run in a container where the reference checkout is present (its location is REF below,
overridable with GFD_REFERENCE):

    make -C oracle                 # builds oracle/_ref/libgfd_ref_cpu.so from the reference sources
    python tests/golden/make_golden.py

Outputs
  abi_layout.json   sizes / offsets / constants of the reference wire structs, printed by
                    abi_probe.cpp compiled against the reference headers.
  gather_cases.json one record per case: the seeded input recipe, the reference
                    output's checksum, per-token checksums and (small cases) the
                    output bytes in hex.  The outputs come from the reference's own
                    CpuPollingThread::parallel_gather (src/parallel_gather.cpp),
                    i.e. the bytes its GFD Direct path DMAs to the GPU.
"""
from __future__ import annotations

import ctypes
import json
import os
import subprocess
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from tests.golden.cases import CASES, aligned_zeros, build_case, checksum  # noqa: E402

# the reference checkout: $GFD_REFERENCE, else a directory named `reference` beside this repository
REF = os.environ.get("GFD_REFERENCE") or os.path.join(os.path.dirname(ROOT), "reference")


def abi_layout():
    with tempfile.TemporaryDirectory() as td:
        exe = os.path.join(td, "abi_ref")
        subprocess.check_call(["g++", "-std=c++17", "-I", os.path.join(REF, "include"),
                               "-I", "/usr/local/cuda/include",
                               os.path.join(HERE, "abi_probe.cpp"), "-o", exe])
        out = subprocess.check_output([exe], text=True)
    return json.loads(out)


def main():
    layout = abi_layout()
    with open(os.path.join(HERE, "abi_layout.json"), "w") as f:
        json.dump(layout, f, indent=1, sort_keys=True)

    lib = ctypes.CDLL(os.path.join(ROOT, "oracle", "_ref", "libgfd_ref_cpu.so"))
    lib.ref_parallel_gather.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p,
                                        ctypes.c_uint64, ctypes.c_int]
    lib.ref_parallel_gather.restype = ctypes.c_int
    records = []
    for spec in CASES:
        pool, entries, out_len = build_case(spec)
        out = aligned_zeros(out_len)  # page-aligned, like the reference's staging buffers
        base = out.ctypes.data
        # the reference gathers into staging at (dst - min_dst); dst offsets are relative
        e = entries.copy()
        e["dst"] += np.uint64(base)
        rc = lib.ref_parallel_gather(e.ctypes.data, len(e), out.ctypes.data, base, spec["workers"])
        assert rc == 0
        per = [checksum(out[d:d + s]) for d, s in zip(entries["dst"].astype(np.int64),
                                                       entries["size"].astype(np.int64))]
        rec = dict(spec)
        rec["out_len"] = int(out_len)
        rec["checksum"] = "%016x" % checksum(out)
        rec["token_checksums"] = ["%016x" % c for c in per]
        if out_len <= 16384:
            rec["bytes_hex"] = out.tobytes().hex()
        records.append(rec)
        print(spec["name"], rec["checksum"], len(entries), "entries")
    with open(os.path.join(HERE, "gather_cases.json"), "w") as f:
        json.dump({"generator": "tests/golden/make_golden.py",
                   "reference_function": "CpuPollingThread::parallel_gather (src/parallel_gather.cpp:74-116)",
                   "cases": records}, f, indent=1)


if __name__ == "__main__":
    main()
