"""Builds the C++ API test programs in tests/cpp/ against include/gfd and
libgfd_b200.so (nvcc, sm_100a).  Binaries go to tests/cpp/bin/ (git-ignored; they
travel to the GPU box with the snapshot).

    python -m tests.cpp_build
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
SRC = os.path.join(HERE, "cpp")
BIN = os.path.join(SRC, "bin")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
LIBDIR = os.path.join(ROOT, "gfd_b200")

PROGRAMS = ["queue_mode", "warp_spec", "sg_session", "ring_modes", "timeouts", "copy_engine", "agent"]

# The reference's own test programs and examples, compiled unmodified against
# include/gfd + libgfd_b200.so (drop-in check).  Built only where the reference
# checkout exists; the binaries go to oracle/_ref/dropin/ (git-ignored, they travel
# to the GPU box).  Not built: examples/04 (calls a copy-engine batch API that is
# closed on this pool) and 05/06/08 (need libnuma, absent here).
# the reference checkout: $GFD_REFERENCE, else a directory named `reference` beside this repository
REFERENCE = os.environ.get("GFD_REFERENCE") or os.path.join(os.path.dirname(ROOT), "reference")
DROPIN_DIR = os.path.join(ROOT, "oracle", "_ref", "dropin")
DROPIN = {
    "test_db_small_tiles": "test/test_db_small_tiles.cu",
    "test_sg_e2e": "test/test_sg_e2e.cu",
    "test_sg_gpu_submit": "test/test_sg_gpu_submit.cu",
    "ex01_basic_transfer": "examples/01_basic_transfer.cu",
    "ex02_direct_transfer": "examples/02_direct_transfer.cu",
    "ex03_gpu_planned_transfer": "examples/03_gpu_planned_transfer.cu",
    "ex07_warp_spec_simple": "examples/07_warp_spec_simple.cu",
    "ex09_sg_warp_spec": "examples/09_sg_warp_spec.cu",
}


def nvcc_cmd(src, out, extra_inc=()):
    cmd = [NVCC, "-std=c++17", "-O2", "-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo",
           "-I", os.path.join(ROOT, "include")]
    for inc in extra_inc:
        cmd += ["-I", inc]
    cmd += [src, "-o", out, "-L", LIBDIR, "-lgfd_b200", "-Xlinker", "-rpath=" + LIBDIR,
            "-L/usr/local/cuda/lib64/stubs", "-lcuda"]
    return cmd


def _stale(out, deps):
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    return any(os.path.getmtime(d) > t for d in deps)


def _deps():
    deps = [os.path.join(LIBDIR, "libgfd_b200.so"), os.path.join(SRC, "common.h")]
    inc = os.path.join(ROOT, "include", "gfd")
    deps += [os.path.join(inc, f) for f in os.listdir(inc)]
    return deps


def build_all(verbose=False):
    os.makedirs(BIN, exist_ok=True)
    deps = _deps()
    outs = []
    for p in PROGRAMS:
        src = os.path.join(SRC, p + ".cu")
        out = os.path.join(BIN, p)
        if _stale(out, deps + [src]):
            cmd = nvcc_cmd(src, out)
            if verbose:
                print(" ".join(cmd))
            r = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
            if r.returncode != 0:
                sys.stderr.write(r.stdout)
                raise RuntimeError(f"building {p} failed")
        outs.append(out)
    return outs


def build_dropin(verbose=False):
    """Compiles the reference programs in DROPIN against this library (if present)."""
    if not os.path.isdir(os.path.join(REFERENCE, "examples")):
        return []
    os.makedirs(DROPIN_DIR, exist_ok=True)
    deps = _deps()
    outs = []
    for name, rel in DROPIN.items():
        src = os.path.join(REFERENCE, rel)
        out = os.path.join(DROPIN_DIR, name)
        if _stale(out, deps + [src]):
            cmd = nvcc_cmd(src, out)
            if verbose:
                print(" ".join(cmd))
            r = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
            if r.returncode != 0:
                sys.stderr.write(r.stdout)
                raise RuntimeError(f"building reference program {rel} against gfd_b200 failed")
        outs.append(out)
    return outs


if __name__ == "__main__":
    for o in build_all(verbose="-v" in sys.argv):
        print(o)
    for o in build_dropin(verbose="-v" in sys.argv):
        print(o)
