"""Builds libgfd_b200.so (sm_100a) in-tree with nvcc.

    python -m gfd_b200.build            # incremental
    python -m gfd_b200.build --clean

Objects go to gfd_b200/_build/, the shared library to gfd_b200/libgfd_b200.so.  The
CUDA runtime is linked statically and the driver is reached through
cudaGetDriverEntryPoint, so the library loads (and its symbols can be inspected)
on machines without a GPU driver.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libgfd_b200.so")
WORKLOAD_LIB = os.path.join(PKG, "libgfd_workload.so")
LAYERS_LIB = os.path.join(PKG, "libgfd_layers.so")
QUEUE_CLIENT_LIB = os.path.join(PKG, "libgfd_queue_client.so")
MOE_SG_LIB = os.path.join(PKG, "libgfd_moe_sg.so")

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-std=c++17", "-O3", "-lineinfo", "-Xcompiler", "-fPIC,-Wall,-Wno-unused-function",
          "-I", INCLUDE, "-I", CSRC]

SOURCES = [
    "gather.cu",
    "context.cpp",
    "noalloc.cu",
    "moe.cu",
    "ring.cu",
    "agent.cu",
    "copy_engine.cpp",
    "cpu_polling.cpp",
    "sessions.cpp",
]


def _headers():
    out = []
    for base in (CSRC, os.path.join(INCLUDE, "gfd")):
        for f in os.listdir(base):
            if f.endswith((".h", ".cuh")):
                out.append(os.path.join(base, f))
    out.append(os.path.join(INCLUDE, "gfd_b200.h"))
    return out


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd, verbose):
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout)
        raise RuntimeError("build step failed: " + " ".join(cmd[:4]) + " ...")
    if verbose and r.stdout.strip():
        print(r.stdout)


def build(verbose: bool = False, ptxas_info: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    headers = _headers()
    objs = []
    for src in SOURCES:
        path = os.path.join(CSRC, src)
        obj = os.path.join(BUILD, src + ".o")
        objs.append(obj)
        if _stale(obj, [path, __file__] + headers) or ptxas_info:
            cmd = [NVCC] + ARCH + COMMON + ["-c", path, "-o", obj]
            if ptxas_info and src.endswith(".cu"):
                cmd += ["-Xptxas", "-v"]
            _run(cmd, verbose or ptxas_info)
    if _stale(LIB, objs):
        _run([NVCC] + ARCH + ["-shared", "-cudart", "static", "-Xlinker", "-Bsymbolic", "-o", LIB] + objs +
             ["-lpthread", "-ldl", "-lrt"], verbose)
    # layer pipeline: a client of libgfd_b200.so through the C++ session API
    lsrc = os.path.join(CSRC, "layers.cu")
    if _stale(LAYERS_LIB, [lsrc, LIB, __file__] + headers):
        _run([NVCC] + ARCH + COMMON + ["-shared", "-cudart", "static", "-Xlinker", "-Bsymbolic", "-o", LAYERS_LIB,
                                       lsrc, "-L", PKG, "-lgfd_b200", "-Xlinker", "-rpath=$ORIGIN"], verbose)
    # GPU-queued submit client (device producer API + this library's ring consumer)
    qsrc = os.path.join(CSRC, "queue_client.cu")
    if _stale(QUEUE_CLIENT_LIB, [qsrc, LIB, __file__] + headers):
        _run([NVCC] + ARCH + COMMON + ["-shared", "-cudart", "static", "-Xlinker", "-Bsymbolic", "-o",
                                       QUEUE_CLIENT_LIB, qsrc, "-L", PKG, "-lgfd_b200", "-Xlinker", "-rpath=$ORIGIN"],
             verbose)
    # MoE gather through SGWarpSpecSession with GPU-submitted lists
    msrc = os.path.join(CSRC, "moe_sg.cu")
    if _stale(MOE_SG_LIB, [msrc, LIB, __file__] + headers):
        _run([NVCC] + ARCH + COMMON + ["-shared", "-cudart", "static", "-Xlinker", "-Bsymbolic", "-o", MOE_SG_LIB,
                                       msrc, "-L", PKG, "-lgfd_b200", "-Xlinker", "-rpath=$ORIGIN"], verbose)
    wsrc = os.path.join(CSRC, "workload.c")
    if _stale(WORKLOAD_LIB, [wsrc, __file__]):
        _run(["gcc", "-O3", "-fPIC", "-shared", "-Wall", "-o", WORKLOAD_LIB, wsrc, "-lm",
              "-lpthread"], verbose)
    return LIB


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--clean", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="print registers / spills / smem")
    a = ap.parse_args()
    if a.clean and os.path.isdir(BUILD):
        shutil.rmtree(BUILD)
        if os.path.exists(LIB):
            os.remove(LIB)
    print(build(verbose=a.verbose, ptxas_info=a.ptxas_info))


if __name__ == "__main__":
    main()
