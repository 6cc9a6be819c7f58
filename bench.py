#!/usr/bin/env python3
"""Benchmark: scattered host->device gather (KV block fetch).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step = one gather of 2048 x 64 KiB KV blocks, chosen by a seeded permutation from
a 4 GiB pinned, NUMA-local host pool (65,536 blocks of bf16 ~ N(0,1)), into a
contiguous 128 MiB HBM buffer.  Under torchrun each rank drives its own GPU with
its own pool and shard (independent replicas, weak scaling, no data-path collective;
NCCL only carries the barrier and the max-over-ranks timing reduction).

value   device time (CUDA events on the launching stream) of gfd_gather_device, the
        entry list already resident in HBM; L2 is flushed (256 MiB memset) before
        every timed step; aggregate GB/s = ranks x bytes / sum over steps of the
        slowest rank's step time.
e2e     the same workload through the public C ABI from HOST entries
        (gfd_gather_sync: entry copy + validation + pull + completion word read back),
        host wall clock per call, L2 flushed between calls.
roofline  bound = PCIe H2D: peak = contiguous pinned cudaMemcpyAsync H2D of 256 MiB
        measured in this run on this GPU (median of 10).
cpu_baseline  the reference's GFD Direct path (CpuPollingThread::submit_direct: AVX-512
        gather workers + copy engine), compiled from the reference sources into
        oracle/_ref/, timed on this box's host cores on the same workload.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "scattered H2D GB/s (per GPU and 8-GPU aggregate) and % of measured PCIe peak"
REF_LIB = os.path.join(ROOT, "oracle", "_ref", "libgfd_ref.so")
ORACLE_LIB = os.path.join(ROOT, "oracle", "_build", "libgfd_oracle.so")
REF_QUEUE_LIB = os.path.join(ROOT, "oracle", "_ref", "libgfd_ref_queue.so")
QUEUE_CLIENT_LIB = os.path.join(ROOT, "gfd_b200", "libgfd_queue_client.so")


# ---------------------------------------------------------------------------
def dist_env():
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("LOCAL_RANK", "0")),
            int(os.environ.get("WORLD_SIZE", "1")))


class Dist:
    """Process-group plumbing for the multi-GPU bench: a barrier and an elementwise
    max over ranks.  NCCL on GPUs; gloo (CPU tensors) is what the CPU tests use."""

    def __init__(self, world, backend="nccl", timeout_s=120):
        self.world = world
        self.pg = None
        self.device = "cuda" if backend == "nccl" else "cpu"
        if world > 1:
            import datetime
            import torch.distributed as dist
            # bounded: a rank that died or never arrives ends the others' next collective
            # with an error instead of a hang
            dist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s))
            self.pg = dist

    def barrier(self):
        if self.pg:
            import torch
            t = torch.zeros(1, device=self.device)
            self.pg.all_reduce(t)
            if self.device == "cuda":
                torch.cuda.synchronize()

    def max_vec(self, v):
        if not self.pg:
            return list(v)
        import torch
        t = torch.tensor(v, dtype=torch.float64, device=self.device)
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return t.cpu().tolist()

    def all_values(self, x):
        """[x of rank 0, x of rank 1, ...] on every rank."""
        if not self.pg:
            return [x]
        import torch
        t = torch.tensor([x], dtype=torch.float64, device=self.device)
        out = [torch.zeros_like(t) for _ in range(self.world)]
        self.pg.all_gather(out, t)
        return [float(o.item()) for o in out]

    def all_bytes(self, b: bytes):
        """[b of rank 0, b of rank 1, ...] on every rank (every rank's b has the same length)."""
        if not self.pg:
            return [bytes(b)]
        import torch
        t = torch.tensor(list(b), dtype=torch.uint8, device=self.device)
        out = [torch.zeros_like(t) for _ in range(self.world)]
        self.pg.all_gather(out, t)
        return [bytes(o.cpu().tolist()) for o in out]

    def sum_vec(self, v):
        if not self.pg:
            return list(v)
        import torch
        t = torch.tensor(v, dtype=torch.float64, device=self.device)
        self.pg.all_reduce(t)
        return t.cpu().tolist()

    def close(self):
        if self.pg:
            self.pg.destroy_process_group()
            self.pg = None


def aggregate_gbs(bytes_per_rank, world, slowest_step_seconds):
    """Whole-job GB/s: every rank moves bytes_per_rank per step; a step lasts as long as
    its slowest rank."""
    return world * bytes_per_rank * len(slowest_step_seconds) / sum(slowest_step_seconds) / 1e9


class ClockSampler:
    """SM clock and clock-event reasons sampled every 5 ms through NVML (read-only queries)
    while the timed region runs; nvidia-smi every 50 ms where NVML is not importable."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    NAMES = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.thread = None
        self.samples = []
        self.path = os.path.join("/tmp", f"gfd_clocks_{os.getpid()}.csv")

    def _nvml_loop(self, nv, h, bits, ready):
        while True:
            try:
                sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                r = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                self.samples.append((float(sm), tuple(n for n, b in bits if r & b)))
            except Exception:
                pass
            ready.set()
            if self._stop.wait(0.005):
                return

    def start(self):
        import threading
        try:
            import pynvml as nv
            nv.nvmlInit()
            h = nv.nvmlDeviceGetHandleByIndex(self.gpu)
            self.max_mhz = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))
            bits = list(zip(self.NAMES, (nv.nvmlClocksEventReasonHwSlowdown, nv.nvmlClocksEventReasonHwThermalSlowdown,
                                         nv.nvmlClocksEventReasonSwThermalSlowdown, nv.nvmlClocksEventReasonSwPowerCap)))
            self._stop = threading.Event()
            ready = threading.Event()
            self.thread = threading.Thread(target=self._nvml_loop, args=(nv, h, bits, ready), daemon=True)
            self.thread.start()
            ready.wait(1.0)  # the first sample precedes the timed region
            return
        except Exception:
            self.thread = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), "--query-gpu=" + self.FIELDS, "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.thread is not None:
            self._stop.set()
            self.thread.join()
            sm = [x[0] for x in self.samples]
            reasons = sorted({n for x in self.samples for n in x[1]})
            if not sm:
                return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["no samples"]}
            return {"sm_mhz": statistics.median(sm), "sm_min_mhz": min(sm), "sm_max_mhz": self.max_mhz,
                    "reasons": reasons, "samples": len(sm), "source": "NVML, 5 ms"}
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        self.proc.wait()
        rows = []
        for line in open(self.path):
            p = [x.strip() for x in line.split(",")]
            if len(p) >= 9:
                rows.append(p)
        try:
            os.remove(self.path)
        except OSError:
            pass
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        reasons = sorted({self.NAMES[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows), "source": "nvidia-smi, 50 ms"}


# ---------------------------------------------------------------------------
def measure_pcie_peak(ctx, pool_ptr, nbytes, stream, iters=10):
    """Contiguous pinned H2D cudaMemcpyAsync (the roofline denominator)."""
    import torch
    dst = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    src = torch.from_numpy(np.ctypeslib.as_array((ctypes.c_uint8 * nbytes).from_address(pool_ptr)))
    times = []
    with torch.cuda.stream(stream):
        for i in range(iters + 3):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            dst.copy_(src, non_blocking=True)
            b.record(stream)
            b.synchronize()
            if i >= 3:
                times.append(a.elapsed_time(b) / 1e3)
    del dst
    return nbytes / statistics.median(times) / 1e9


def reference_direct(w, pool_ptr, dst_ptr, device, warmup, steps, entries, before=None):
    """Times the reference's GFD Direct (compiled from its sources) on `entries`;
    `before` (untimed) runs before every call, e.g. an L2 flush."""
    if not os.path.exists(REF_LIB):
        return None
    total = int(entries["size"].sum())
    try:
        ref = RefLib(device, dst_ptr, pool_ptr, total)
    except RuntimeError:
        return None
    e = np.ascontiguousarray(entries)
    before = before or (lambda: None)

    def timed(fn):
        before()
        return fn()
    for _ in range(warmup):
        timed(lambda: ref.direct_us(e))
    us = [timed(lambda: ref.direct_us(e)) for _ in range(steps)]
    import torch
    s = torch.cuda.Stream()
    for _ in range(min(warmup, 3)):
        timed(lambda: ref.memcpy_n_us(e, s.cuda_stream))
    mus = [timed(lambda: ref.memcpy_n_us(e, s.cuda_stream)) for _ in range(max(3, steps // 4))]
    workers = ref.workers
    ref.close()
    return {"direct_us": us, "memcpy_n_us": mus, "workers": workers, "bytes": total}


def oracle_port_baseline(pool_ptr, entries, seconds=1.0):
    """CPU restatement timed on one core (used only when the reference is not built)."""
    lib = ctypes.CDLL(ORACLE_LIB)
    lib.gfd_oracle_gather.argtypes = [ctypes.c_void_p, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_void_p,
                                      ctypes.c_int64]
    lib.gfd_oracle_gather.restype = ctypes.c_int64
    total = int(entries["size"].sum())
    out = np.empty(total, np.uint8)
    e = entries.copy()
    e["dst"] = np.uint64(out.ctypes.data) + (e["dst"] - e["dst"][0])
    n, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < seconds:
        lib.gfd_oracle_gather(out.ctypes.data, out.ctypes.data, total, e.ctypes.data, len(e))
        n += 1
    dt = time.perf_counter() - t0
    return total * n / dt / 1e9


def load_profile_traffic(config="cfg2"):
    """Per-launch traffic figures of a configuration's dominant kernel from the committed
    ncu summary (profiles/kernel_traffic.txt)."""
    p = os.path.join(ROOT, "profiles", "kernel_traffic.txt")
    out = {}
    try:
        for line in open(p):
            if ":" in line and not line.startswith("#") and line.startswith(config + "."):
                k, v = line.split(":", 1)
                k = k.strip()[len(config) + 1:]
                v = v.strip()
                out[k] = int(v) if v.isdigit() else v
    except OSError:
        return None
    return out or None


# ---------------------------------------------------------------------------
def run_ours(args, rank, local_rank, world, dist):
    import torch
    import gfd_b200
    from gfd_b200 import workloads as wl

    torch.cuda.set_device(local_rank)
    ctx = gfd_b200.Context(local_rank)
    w = wl.cfg2()
    # N > 1: each rank's pool is a memfd segment, so ranks with faster links can map the
    # pools of slower ones and pull part of their blocks for them (ForwardedJob)
    forwarding = world > 1 and not args.equal_shards
    pool = _SegmentPool(ctx, w.pool_bytes) if forwarding else ctx.pool(w.pool_bytes)
    w.fill_pool(pool.ptr)
    if forwarding:
        pool.register()
    dst = torch.empty(w.total_bytes, dtype=torch.uint8, device="cuda")
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    entries = w.entries(pool.ptr, dst.data_ptr())
    d_entries = torch.from_numpy(entries.view(np.uint8).copy()).cuda()
    stream = torch.cuda.Stream()
    st = stream.cuda_stream
    nbytes = w.total_bytes

    def step_device():
        ctx.gather_device(d_entries.data_ptr(), w.num_tokens, dst.data_ptr(), nbytes, stream=st)

    # warm-up (also checks the result once)
    for _ in range(max(args.warmup, 1)):
        step_device()
    stream.synchronize()
    rc, bad = ctx.gather_device_status()
    if rc != gfd_b200.GFD_OK:
        raise RuntimeError(f"warm-up gather failed: {ctx.last_error()}")
    got = dst[:65536].cpu().numpy()
    first = np.ctypeslib.as_array((ctypes.c_uint8 * 65536).from_address(int(entries["src"][0])))
    if not np.array_equal(got, first):
        raise RuntimeError("warm-up gather produced wrong bytes")

    dist.barrier()  # every rank measures its link at the same time
    peak = measure_pcie_peak(ctx, pool.ptr, 256 << 20, stream)
    peak_sum = dist.sum_vec([peak])[0]
    peaks = dist.all_values(peak)

    # ---- value: device-timed, entries resident in HBM ----
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    clocks = ClockSampler(int(vis.split(",")[local_rank]) if vis else local_rank)
    clocks.start()
    step_times = []
    for _ in range(args.steps):
        with torch.cuda.stream(stream):
            flush.zero_()
        stream.synchronize()
        dist.barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        step_device()
        b.record(stream)
        b.synchronize()
        step_times.append(a.elapsed_time(b) / 1e3)
    clk = clocks.stop()
    rc, _ = ctx.gather_device_status()
    if rc != gfd_b200.GFD_OK:
        raise RuntimeError(ctx.last_error())
    max_steps = dist.max_vec(step_times)
    total_t = sum(max_steps)
    value = aggregate_gbs(nbytes, world, max_steps)
    my_t = sum(step_times)

    # ---- e2e: host entries through the public C ABI ----
    e2e_us = []
    for i in range(args.warmup + args.steps):
        flush.zero_()
        torch.cuda.synchronize()
        dist.barrier()
        us = ctx.gather_sync(entries)
        if i >= args.warmup:
            e2e_us.append(us)
    max_e2e = dist.max_vec(e2e_us)
    e2e_value = aggregate_gbs(nbytes, world, [u / 1e6 for u in max_e2e])

    # ---- the two SM-pull movers side by side (host entries, same call, same flush) ----
    variants = {}
    for name, fl in (("pull_16B_loads", gfd_b200.GATHER_FORCE_PULL), ("bulk_stage", gfd_b200.GATHER_BULK_STAGE)):
        us = []
        for i in range(args.warmup + args.steps):
            flush.zero_()
            torch.cuda.synchronize()
            dist.barrier()
            t_us = ctx.gather_sync(entries, flags=fl)
            if i >= args.warmup:
                us.append(t_us)
        variants[name] = aggregate_gbs(nbytes, world, [u / 1e6 for u in dist.max_vec(us)])

    out = {
        "value": value, "ms_per_step": total_t / args.steps * 1e3, "per_rank_gbs": nbytes * args.steps / my_t / 1e9,
        "rank_gbs": dist.all_values(nbytes * args.steps / my_t / 1e9), "rank_peaks": peaks,
        "peak": peak, "peak_sum": peak_sum, "clocks": clk, "e2e_value": e2e_value, "e2e_p50_us": statistics.median(max_e2e),
        "bytes": nbytes, "entries_bytes": entries.nbytes, "pull_variants": variants,
        "launches_per_step": 2, "d2h_bytes": 8,
    }

    # ---- N > 1: the same job pulled by link rate, slower ranks' tails forwarded over NVLink ----
    if forwarding:
        fwd = None
        try:
            fwd = ForwardedJob(ctx, w, rank, world, dist, pool.seg, dst.data_ptr(), stream, flush)
            calib = fwd.calibrate(args, peaks)
            if max(abs(a - b) for a, b in zip(fwd.shares, fwd.need)) <= kForwardMinShift * w.num_tokens:
                # links within a few percent of one another: nothing worth moving
                raise _EqualLinks(calib)
            clocks = ClockSampler(int(vis.split(",")[local_rank]) if vis else local_rank)
            clocks.start()
            t = fwd.timed(args, args.steps)
            clk_f = clocks.stop()
            slowest = dist.max_vec(t)
            dist.barrier()  # every donor's stores into this rank's buffer have landed
            pool_np = np.frombuffer(pool.seg.map, dtype=np.uint8)
            bad = fwd.check(dst.cpu().numpy(), pool_np)
            del pool_np
            if dist.sum_vec([float(bad)])[0] > 0:
                raise RuntimeError("forwarded job: checked blocks differ from the pools")
            e2e_t = dist.max_vec(fwd.e2e(args))
            mine = fwd.pulled_bytes * len(t) / sum(t) / 1e9
            out["equal_shards"] = {"value": value, "ms_per_step": out["ms_per_step"], "rank_gbs": out["rank_gbs"],
                                   "e2e_value": e2e_value, "clocks": clk}
            out.update({
                "value": aggregate_gbs(nbytes, world, slowest), "ms_per_step": sum(slowest) / len(slowest) * 1e3,
                "per_rank_gbs": mine, "rank_gbs": dist.all_values(mine), "clocks": clk_f,
                "e2e_value": aggregate_gbs(nbytes, world, e2e_t), "e2e_p50_us": statistics.median(e2e_t) * 1e6,
                "entries_bytes": sum(c[0].numel() for c in fwd.calls), "bytes": fwd.pulled_bytes,
                "launches_per_step": sum(1 if c[2] <= 512 else 2 for c in fwd.calls), "d2h_bytes": 56,
            })
            out["forwarding"] = {"used": True, "blocks_pulled_per_rank": fwd.shares,
                                 "transfers": [list(x) for x in fwd.transfers], "calibration": calib,
                                 "note": "every rank receives its own 2048 blocks from its own pool; ranks "
                                         "with faster host links also pull the tail of a slower rank's list "
                                         "from that rank's pool and store it into its buffer over NVLink"}
        except _EqualLinks as eq:
            out["forwarding"] = {"used": False, "calibration": eq.calib,
                                 "reason": "every rank's rate-proportional share is within %d%% of its own "
                                           "blocks: equal shards" % round(100 * kForwardMinShift)}
        except (RuntimeError, OSError, ValueError) as exc:
            out["forwarding"] = {"used": False, "unavailable": str(exc), "value_is": "equal shards"}
        finally:
            if fwd is not None:
                fwd.close()

    # ---- second target: 2048 x 4 KiB at 2x stride, every rank ----
    out["cfg3_4k"] = measure_cfg3_4k(ctx, args, local_rank, world, dist, stream, flush, peak)

    # ---- N > 1: one shared pool, equal and link-rate-proportional shards ----
    if world > 1 and not args.no_shared_pool:
        pool.free()
        pool = None
        try:
            out["shared_pool"] = measure_shared_pool(ctx, args, rank, world, dist, stream, flush, peaks)
        except (RuntimeError, OSError, ValueError) as exc:
            out["shared_pool"] = {"unavailable": str(exc)}

    # ---- cpu baseline (rank 0, N = 1 only) ----
    if world == 1 and not args.no_cpu_baseline:
        ref = reference_direct(w, pool.ptr, dst.data_ptr(), local_rank, warmup=15, steps=50, entries=entries)
        if ref is not None:
            p50 = statistics.median(ref["direct_us"])
            out["cpu_baseline"] = {
                "value": nbytes / (p50 / 1e6) / 1e9, "unit": "GB/s", "cores": ref["workers"] + 1,
                "kind": "reference",
                "sample": f"full workload (2048 x 64 KiB from the 4 GiB pool), reference "
                          f"CpuPollingThread::submit_direct, {ref['workers']} gather workers + caller, "
                          f"p50 of 50 calls after 15 warm-up (reference method, examples/04_benchmark.cu)",
                "memcpy_n_gbs": nbytes / (statistics.median(ref["memcpy_n_us"]) / 1e6) / 1e9,
            }
        else:
            gbs = oracle_port_baseline(pool.ptr, entries)
            out["cpu_baseline"] = {"value": gbs, "unit": "GB/s", "cores": 1, "kind": "port",
                                   "sample": "CPU restatement (memcpy per entry into host memory), 1 s of calls"}
    if pool is not None:
        pool.free()
    ctx.close()
    return out


def measure_cfg3_4k(ctx, args, local_rank, world, dist, stream, flush, peak):
    """The second north_star target on every rank: 2048 x 4 KiB tokens at 2x stride
    (BASELINE config 3's 4 KiB point), device-timed through gfd_gather_device (entries in
    HBM) and end to end through gfd_gather_sync from host entries, L2 flushed before every
    call; at N = 1 the reference's GFD Direct and Memcpy(N) on the same tokens beside it."""
    import torch
    import gfd_b200
    from gfd_b200 import workloads as wl

    w = wl.cfg3(2048, 4096)
    nbytes = w.total_bytes
    pool = ctx.pool(w.pool_bytes)
    w.fill_pool(pool.ptr)
    dst = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    e = w.entries(pool.ptr, dst.data_ptr())
    d_e = torch.from_numpy(e.view(np.uint8).copy()).cuda()
    st = stream.cuda_stream
    want = pool.array()[:w.pool_bytes].reshape(w.num_tokens, 2, w.token_size)[:, 0, :].reshape(-1)
    for _ in range(args.warmup):
        ctx.gather_sync(e)
    if not np.array_equal(dst.cpu().numpy(), want):
        raise RuntimeError("cfg3_4k: gfd_gather_sync produced wrong bytes")
    dst.zero_()
    for _ in range(args.warmup):
        ctx.gather_device(d_e.data_ptr(), w.num_tokens, dst.data_ptr(), nbytes, stream=st)
    stream.synchronize()
    if ctx.gather_device_status() != (gfd_b200.GFD_OK, -1) or not np.array_equal(dst.cpu().numpy(), want):
        raise RuntimeError("cfg3_4k: gfd_gather_device produced wrong bytes")
    dev_t = _timed_steps(args, stream, flush, dist,
                         lambda: ctx.gather_device(d_e.data_ptr(), w.num_tokens, dst.data_ptr(), nbytes, stream=st))
    e2e_t = []
    for _ in range(args.steps):
        flush.zero_()
        torch.cuda.synchronize()
        dist.barrier()
        e2e_t.append(ctx.gather_sync(e) / 1e6)
    m_dev, m_e2e = dist.max_vec(dev_t), dist.max_vec(e2e_t)
    value, e2e = aggregate_gbs(nbytes, world, m_dev), aggregate_gbs(nbytes, world, m_e2e)
    out = {"workload": "cfg3_2048x4KiB_stride2", "tokens": 2048, "token_bytes": 4096,
           "l2": "flushed (256 MiB memset) before every call", "unit": "GB/s",
           "value": value, "ms_per_step": sum(m_dev) / len(m_dev) * 1e3,
           "e2e": {"value": e2e, "unit": "GB/s", "p50_us": statistics.median(m_e2e) * 1e6,
                   "h2d_bytes_per_step": nbytes + e.nbytes, "d2h_bytes_per_step": 8},
           "roofline": {"bound": "pcie", "peak": peak, "unit": "GB/s",
                        "achieved": value / world, "frac": value / world / peak,
                        "e2e_achieved": e2e / world, "e2e_frac": e2e / world / peak,
                        "target_frac": 0.70,
                        "kernel": "gfdb::pull_kernel (+ gfdb::plan_kernel for device entries)"},
           "per_rank_e2e_gbs": dist.all_values(nbytes * len(e2e_t) / sum(e2e_t) / 1e9),
           "per_rank_device_gbs": dist.all_values(nbytes * len(dev_t) / sum(dev_t) / 1e9)}
    if world == 1 and not args.no_cpu_baseline:
        ref = reference_direct(w, pool.ptr, dst.data_ptr(), local_rank, warmup=15, steps=50, entries=e,
                               before=lambda: (flush.zero_(), torch.cuda.synchronize()))
        if ref is not None:
            out["reference_direct_gbs"] = nbytes / (statistics.median(ref["direct_us"]) / 1e6) / 1e9
            out["reference_memcpy_n_gbs"] = nbytes / (statistics.median(ref["memcpy_n_us"]) / 1e6) / 1e9
            out["reference_note"] = (f"GFD Direct with {ref['workers']} gather workers + caller, p50 of 50 calls "
                                     "after 15 warm-up; Memcpy(N) = one cudaMemcpyAsync per token; L2 flushed "
                                     "before every call")
    pool.free()
    return out


def measure_shared_pool(ctx, args, rank, world, dist, stream, flush, peaks, calibration_rounds=2):
    """Config 2's blocks fetched by every rank from ONE 4 GiB pool in shared host memory
    (gfd_b200.shared_pool: a memfd segment created by rank 0, attached and registered by
    every rank), in two splits of the same job of world x 2048 blocks:

    equal              2048 blocks per rank;
    rate_proportional  blocks in proportion to each rank's link rate: first the concurrent
                       contiguous-copy peaks measured in this run (`peaks`), then
                       `calibration_rounds` times the rates the ranks reached pulling
                       their previous shares together (the host fabric is shared, so a
                       rank's rate depends on what the others pull), then timed.

    Ranks take disjoint slices of one permutation of the pool's blocks.  Device-timed like
    the headline (entries in HBM, L2 flushed, ranks aligned before every step); the
    aggregate is the job's bytes over the slowest rank's time."""
    import types
    import torch
    import gfd_b200
    from gfd_b200 import workloads as wl
    from gfd_b200.shared_pool import SharedSegment, rate_shares

    base = wl.cfg2()
    bs = base.token_size
    seg = SharedSegment.create(base.pool_bytes) if rank == 0 else None
    pid, fd = (seg.pid_fd() if seg is not None else (0, 0))
    pids, fds = dist.all_values(float(pid)), dist.all_values(float(fd))
    if rank == 0:
        base.fill_pool(seg.ptr)
    dist.barrier()
    if rank != 0:
        seg = SharedSegment.attach(int(pids[0]), int(fds[0]), base.pool_bytes)
    ctx.register(seg.ptr, seg.nbytes)
    pool_view = np.frombuffer(seg.map, dtype=np.uint8)
    perm = wl.permutation(base.pool_bytes // bs, base.seed)
    total = world * base.num_tokens
    st = stream.cuda_stream
    out = {"pool": "one 4 GiB pool in shared host memory (memfd), registered by every rank",
           "job_blocks": total, "unit": "GB/s", "concurrent_peak_gbs": peaks}

    def run_split(shares, steps, label):
        """Every rank pulls its share; returns (slowest-rank step times, this rank's GB/s)."""
        n, off = shares[rank], sum(shares[:rank])
        ids = perm[off:off + n].astype(np.uint64)
        dst = torch.empty(max(n, 1) * bs, dtype=torch.uint8, device="cuda")
        e = gfd_b200.entries_array(np.uint64(dst.data_ptr()) + np.arange(n, dtype=np.uint64) * np.uint64(bs),
                                   np.uint64(seg.ptr) + ids * np.uint64(bs), bs)
        d_e = torch.from_numpy(e.view(np.uint8).copy()).cuda()

        def step():
            if n > 0:
                ctx.gather_device(d_e.data_ptr(), n, dst.data_ptr(), n * bs, stream=st)

        for _ in range(args.warmup):
            step()
        stream.synchronize()
        if ctx.gather_device_status()[0] != gfd_b200.GFD_OK:
            raise RuntimeError(ctx.last_error())
        if n > 0:  # first and last block against the shared pool
            got = dst.cpu().numpy()
            for k in (0, n - 1):
                o = int(ids[k]) * bs
                if not np.array_equal(got[k * bs:(k + 1) * bs], pool_view[o:o + bs]):
                    raise RuntimeError(f"shared pool ({label}): block {k} differs from the pool")
        times = _timed_steps(types.SimpleNamespace(steps=steps), stream, flush, dist, step)
        if ctx.gather_device_status()[0] != gfd_b200.GFD_OK:
            raise RuntimeError(ctx.last_error())
        return dist.max_vec(times), n * bs * len(times) / sum(times) / 1e9

    try:
        shares = [base.num_tokens] * world
        slowest, mine = run_split(shares, args.steps, "equal")
        out["equal"] = {"value": total * bs * len(slowest) / sum(slowest) / 1e9, "blocks_per_rank": shares,
                        "rank_gbs": dist.all_values(mine)}
        rates = list(peaks)
        calib = []
        for r in range(calibration_rounds):
            shares = rate_shares(rates, total)
            _, mine = run_split(shares, 3, f"calibration {r}")
            rates = dist.all_values(mine)
            calib.append({"blocks_per_rank": shares, "rank_gbs": rates})
        shares = rate_shares(rates, total)
        slowest, mine = run_split(shares, args.steps, "rate_proportional")
        out["rate_proportional"] = {"value": total * bs * len(slowest) / sum(slowest) / 1e9,
                                    "blocks_per_rank": shares, "rank_gbs": dist.all_values(mine),
                                    "calibration": calib}
        for mode in ("equal", "rate_proportional"):
            out[mode]["fraction_of_concurrent_peak_sum"] = out[mode]["value"] / sum(peaks)
        if world > 1:
            try:
                out["forwarded"] = measure_forwarded(ctx, args, rank, world, dist, stream, flush, seg, pool_view,
                                                     perm, [base.num_tokens] * world, shares, bs)
                out["forwarded"]["fraction_of_concurrent_peak_sum"] = out["forwarded"]["value"] / sum(peaks)
            except (RuntimeError, OSError, ValueError) as exc:
                out["forwarded"] = {"unavailable": str(exc)}
    finally:
        del pool_view
        torch.cuda.synchronize()
        ctx.unregister(seg.ptr)
        dist.barrier()  # nobody closes the segment while another rank still uses it
        seg.close()
    return out


def ipc_export(ptr):
    """CUDA IPC handle (64 bytes) of the allocation holding device pointer `ptr`, plus the
    pointer's offset in it (8 bytes, little endian)."""
    from cuda.bindings import driver as drv, runtime as rt
    err, base, _size = drv.cuMemGetAddressRange(ptr)
    if int(err) != 0:
        raise RuntimeError(f"cuMemGetAddressRange: {err}")
    err, h = rt.cudaIpcGetMemHandle(int(base))
    if int(err) != 0:
        raise RuntimeError(f"cudaIpcGetMemHandle: {err}")
    return bytes(h.reserved) + int(ptr - int(base)).to_bytes(8, "little")


def ipc_open(blob):
    """Maps another process's allocation (ipc_export's blob) into this one; returns
    (pointer inside it, base to close with cudaIpcCloseMemHandle) or raises."""
    from cuda.bindings import runtime as rt
    h = rt.cudaIpcMemHandle_t()
    h.reserved = blob[:64]
    err, base = rt.cudaIpcOpenMemHandle(h, rt.cudaIpcMemLazyEnablePeerAccess)
    if int(err) != 0:
        raise RuntimeError(f"cudaIpcOpenMemHandle: {err}")
    return int(base) + int.from_bytes(blob[64:72], "little"), int(base)


# Forward over NVLink only when some rank's rate-proportional share differs from its own
# block count by more than this fraction (each forwarded range costs one more launch).
kForwardMinShift = 0.03


class _EqualLinks(Exception):
    def __init__(self, calib):
        super().__init__("equal links")
        self.calib = calib


class _SegmentPool:
    """A pool in a memfd segment registered with the context (gfd_pool_register), so other
    rank processes can map it too; same .ptr / .free() as gfd_b200.HostPool."""

    def __init__(self, ctx, nbytes):
        from gfd_b200.shared_pool import SharedSegment
        self.ctx = ctx
        self.seg = SharedSegment.create(nbytes)
        self.ptr = self.seg.ptr
        self.registered = False

    def register(self):
        self.ctx.register(self.ptr, self.seg.nbytes)
        self.registered = True

    def free(self):
        if self.registered:
            self.ctx.unregister(self.ptr)
            self.registered = False
        self.seg.close()


class ForwardedJob:
    """N > 1, config 2 as the benchmark defines it (every rank receives its own 2048 blocks
    from its own 4 GiB pool), pulled by link rate: ranks whose host link is faster also
    pull the tail of a slower rank's list, from that rank's pool, into that rank's buffer
    over NVLink (gfd_gather_device with GFD_GATHER_PEER_DST).  The pools are memfd segments
    (gfd_b200.shared_pool) so a donor can map and register a receiver's pool; receivers'
    buffers are mapped through CUDA IPC.  Shares start from the concurrent copy peaks and
    are recalibrated from the rates the ranks reach together."""

    def __init__(self, ctx, w, rank, world, dist, seg, dst_ptr, stream, flush):
        import torch
        self.ctx, self.w, self.rank, self.world, self.dist = ctx, w, rank, world, dist
        self.seg, self.dst_ptr, self.stream, self.flush = seg, dst_ptr, stream, flush
        self.need = [w.num_tokens] * world
        self.offsets = w.src_offsets()
        pid, fd = seg.pid_fd()
        self.pids, self.fds = dist.all_values(float(pid)), dist.all_values(float(fd))
        self.dst_blobs = dist.all_bytes(ipc_export(dst_ptr))
        self.pools = {}   # receiver -> attached, registered SharedSegment
        self.opened = {}  # receiver -> (peer dst pointer, base)
        self.calls = []
        self.torch = torch

    def _serve(self, r):
        from gfd_b200.shared_pool import SharedSegment
        if r not in self.pools:
            sg = SharedSegment.attach(int(self.pids[r]), int(self.fds[r]), self.w.pool_bytes)
            try:
                self.ctx.register(sg.ptr, sg.nbytes)
            except BaseException:
                sg.close()
                raise
            self.pools[r] = sg
        if r not in self.opened:
            self.opened[r] = ipc_open(self.dst_blobs[r])

    def build(self, shares):
        """Entry lists of this rank for `shares` (collective: every rank must call it)."""
        import gfd_b200
        from gfd_b200.shared_pool import forward_plan
        torch = self.torch
        own, transfers = forward_plan(shares, self.need)
        failed = ""
        for d, r, first, count in transfers:
            if d == self.rank and not failed:
                try:
                    self._serve(r)
                except (RuntimeError, OSError, ValueError) as exc:
                    failed = str(exc)
        if self.dist.sum_vec([1.0 if failed else 0.0])[0] > 0:
            raise RuntimeError(failed or "another rank could not map a receiver's pool or buffer")
        bs = self.w.token_size
        nbytes = self.need[self.rank] * bs

        def entries(pool_ptr, dst_base, first, count):
            e = gfd_b200.entries_array(
                np.uint64(dst_base) + (np.arange(count, dtype=np.uint64) + np.uint64(first)) * np.uint64(bs),
                np.uint64(pool_ptr) + self.offsets[first:first + count], bs)
            return e, torch.from_numpy(e.view(np.uint8).copy()).pin_memory()

        calls = []
        if own[self.rank] > 0:
            e, h = entries(self.seg.ptr, self.dst_ptr, 0, own[self.rank])
            calls.append((h, own[self.rank], self.dst_ptr, nbytes, 0))
        for d, r, first, count in transfers:
            if d == self.rank:
                e, h = entries(self.pools[r].ptr, self.opened[r][0], first, count)
                calls.append((h, count, self.opened[r][0], self.need[r] * bs, gfd_b200.GATHER_PEER_DST))
        self.calls = [(h, h.cuda(), n, base, size, fl) for h, n, base, size, fl in calls]
        self.shares, self.own, self.transfers = list(shares), own, transfers
        self.pulled_bytes = shares[self.rank] * bs
        return self

    def step(self, copy_entries=False):
        st = self.stream.cuda_stream
        for h, d_e, n, base, size, fl in self.calls:
            if copy_entries:
                with self.torch.cuda.stream(self.stream):
                    d_e.copy_(h, non_blocking=True)
            self.ctx.gather_device(d_e.data_ptr(), n, base, size, stream=st, flags=fl)

    def timed(self, args, steps):
        import types
        import gfd_b200
        for _ in range(args.warmup):
            self.step()
        self.stream.synchronize()
        if self.ctx.gather_device_status()[0] != gfd_b200.GFD_OK:
            raise RuntimeError(self.ctx.last_error())
        times = _timed_steps(types.SimpleNamespace(steps=steps), self.stream, self.flush, self.dist, self.step)
        if self.ctx.gather_device_status()[0] != gfd_b200.GFD_OK:
            raise RuntimeError(self.ctx.last_error())
        return times

    def calibrate(self, args, peaks, rounds=2):
        from gfd_b200.shared_pool import rate_shares
        total = sum(self.need)
        rates, calib = list(peaks), []
        for _ in range(rounds):
            self.build(rate_shares(rates, total))
            t = self.timed(args, 3)
            rates = self.dist.all_values(self.pulled_bytes * len(t) / sum(t) / 1e9)
            calib.append({"blocks_pulled_per_rank": self.shares, "rank_pull_gbs": rates})
        self.build(rate_shares(rates, total))
        return calib

    def e2e(self, args):
        """Per step, host wall clock: the entry lists copied in from pinned host memory,
        the gathers, a stream synchronise (max over ranks; every rank's step ends when its
        own pulls, forwarded ones included, have landed)."""
        torch = self.torch
        t = []
        for i in range(args.warmup + args.steps):
            with torch.cuda.stream(self.stream):
                self.flush.zero_()
            self.stream.synchronize()
            self.dist.barrier()
            t0 = time.perf_counter()
            self.step(copy_entries=True)
            rc, _ = self.ctx.gather_device_status()  # synchronises; reads the status back
            if i >= args.warmup:
                t.append(time.perf_counter() - t0)
            if rc != 0:
                raise RuntimeError(self.ctx.last_error())
        return t

    def check(self, dst_np, pool_np):
        """Head and tail of every part of this rank's buffer against its own pool (after
        a barrier, so donors' stores have landed).  Returns the number of bad blocks."""
        bs = self.w.token_size
        marks = [0, self.own[self.rank] - 1] if self.own[self.rank] > 0 else []
        for d, r, first, count in self.transfers:
            if r == self.rank:
                marks += [first, first + count - 1]
        bad = 0
        for k in marks:
            o = int(self.offsets[k])
            bad += 0 if np.array_equal(dst_np[k * bs:(k + 1) * bs], pool_np[o:o + bs]) else 1
        return bad

    def close(self):
        from cuda.bindings import runtime as rt
        self.torch.cuda.synchronize()
        for _, base in self.opened.values():
            rt.cudaIpcCloseMemHandle(base)
        self.opened = {}
        for sg in self.pools.values():
            try:
                self.ctx.unregister(sg.ptr)
            finally:
                sg.close()
        self.pools = {}
        self.dist.barrier()  # no rank still maps another's pool or buffer


def measure_forwarded(ctx, args, rank, world, dist, stream, flush, seg, pool_view, perm, need, shares, bs):
    """The equal job (every rank receives its own `need` blocks from the shared pool in its
    own HBM), pulled in the link-rate-proportional `shares`: ranks with a faster host link
    also pull the tail of a slower rank's list and store it into that rank's buffer over
    NVLink (gfd_gather_device with GFD_GATHER_PEER_DST into a CUDA IPC mapping of the
    receiver's buffer).  Each rank checks the head and tail of its own part and of every
    forwarded part it received."""
    import torch
    from cuda.bindings import runtime as rt
    import gfd_b200
    from gfd_b200.shared_pool import forward_plan

    def ck(res, what):
        err = res[0] if isinstance(res, tuple) else res
        if int(err) != 0:
            raise RuntimeError(f"{what}: {err}")
        return res[1] if isinstance(res, tuple) and len(res) > 1 else None

    own, transfers = forward_plan(shares, need)
    dev = torch.cuda.current_device()
    ck(rt.cudaSetDevice(dev), "cudaSetDevice")
    nbytes = need[rank] * bs
    buf = ck(rt.cudaMalloc(nbytes), "cudaMalloc")  # a whole allocation: its IPC handle maps it exactly
    opened = {}
    st = stream.cuda_stream
    try:
        handle = ck(rt.cudaIpcGetMemHandle(buf), "cudaIpcGetMemHandle")
        handles = dist.all_bytes(bytes(handle.reserved))
        failed = ""
        for d, r, first, count in transfers:
            if d == rank and r not in opened and not failed:
                h = rt.cudaIpcMemHandle_t()
                h.reserved = handles[r]
                err, p = rt.cudaIpcOpenMemHandle(h, rt.cudaIpcMemLazyEnablePeerAccess)
                if int(err) != 0:
                    failed = f"cudaIpcOpenMemHandle(rank {r}): {err}"
                else:
                    opened[r] = p
        # every rank learns whether all mappings opened before anyone launches into them
        if dist.sum_vec([1.0 if failed else 0.0])[0] > 0:
            raise RuntimeError(failed or "a peer rank could not map a receiver's buffer")
        # entry lists: own head, then one list per forwarded range
        calls = []

        def entries_for(owner, first, count, dst_base):
            off = sum(need[:owner]) + first
            ids = perm[off:off + count].astype(np.uint64)
            e = gfd_b200.entries_array(np.uint64(dst_base) + (np.arange(count, dtype=np.uint64) + np.uint64(first)) *
                                       np.uint64(bs), np.uint64(seg.ptr) + ids * np.uint64(bs), bs)
            return torch.from_numpy(e.view(np.uint8).copy()).cuda()

        if own[rank] > 0:
            calls.append((entries_for(rank, 0, own[rank], int(buf)), own[rank], int(buf), nbytes, 0))
        for d, r, first, count in transfers:
            if d == rank:
                calls.append((entries_for(r, first, count, int(opened[r])), count, int(opened[r]),
                              need[r] * bs, gfd_b200.GATHER_PEER_DST))

        def step():
            for d_e, n, base, size, fl in calls:
                ctx.gather_device(d_e.data_ptr(), n, base, size, stream=st, flags=fl)

        for _ in range(args.warmup):
            step()
        stream.synchronize()
        if ctx.gather_device_status()[0] != gfd_b200.GFD_OK:
            raise RuntimeError(ctx.last_error())
        times = _timed_steps(args, stream, flush, dist, step)
        if ctx.gather_device_status()[0] != gfd_b200.GFD_OK:
            raise RuntimeError(ctx.last_error())
        slowest = dist.max_vec(times)
        dist.barrier()  # every donor's stores into this rank's buffer have landed
        # check: head and tail of the own part and of each range a donor forwarded here
        got = np.empty(nbytes, np.uint8)
        ck(rt.cudaMemcpy(got.ctypes.data, buf, nbytes, rt.cudaMemcpyKind.cudaMemcpyDeviceToHost), "cudaMemcpy")
        marks = [0, own[rank] - 1] if own[rank] > 0 else []
        for d, r, first, count in transfers:
            if r == rank:
                marks += [first, first + count - 1]
        bad = 0
        for k in marks:
            o = int(perm[sum(need[:rank]) + k]) * bs
            bad += 0 if np.array_equal(got[k * bs:(k + 1) * bs], pool_view[o:o + bs]) else 1
        bad_all = dist.sum_vec([float(bad)])[0]
        if bad_all:
            raise RuntimeError(f"forwarded split: {int(bad_all)} checked blocks differ from the pool")
        mine = shares[rank] * bs * len(times) / sum(times) / 1e9
        return {"value": sum(need) * bs * len(slowest) / sum(slowest) / 1e9, "blocks_pulled_per_rank": shares,
                "blocks_received_per_rank": need, "transfers": [list(t) for t in transfers],
                "rank_pull_gbs": dist.all_values(mine),
                "note": "every rank receives its own 2048 blocks; donors pull part of a slower rank's "
                        "list and store it into that rank's buffer over NVLink"}
    finally:
        torch.cuda.synchronize()
        for p in opened.values():
            rt.cudaIpcCloseMemHandle(p)
        dist.barrier()  # no donor still maps this rank's buffer
        rt.cudaFree(buf)


# ---------------------------------------------------------------------------
def _timed_steps(args, stream, flush, dist, launch, after=None):
    """K device-timed steps on `stream` (CUDA events), L2 flushed and ranks aligned
    before each; returns the per-step seconds of this rank."""
    import torch
    times = []
    for _ in range(args.steps):
        with torch.cuda.stream(stream):
            flush.zero_()
        stream.synchronize()
        dist.barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        launch()
        b.record(stream)
        b.synchronize()
        if after is not None:
            after()
        times.append(a.elapsed_time(b) / 1e3)
    return times


def run_cfg4(args, rank, local_rank, world, dist):
    """Layer pipeline: 32 layers x 1024 page-table-selected 64 KiB bf16 blocks per pass,
    pulled by the producer warps of a WarpSpecSession kernel while its compute warps
    RMS-scale the blocks already landed (one launch per pass)."""
    import torch
    import gfd_b200
    from gfd_b200 import layers
    from gfd_b200 import workloads as wl

    torch.cuda.set_device(local_rank)
    ctx = gfd_b200.Context(local_rank)
    bb = wl.CFG4_BLOCK_BYTES
    pool = ctx.pool(wl.CFG4_POOL_BLOCKS * bb)
    wl.cfg4_fill_pool(pool.ptr, seed=4 + 100 * rank)
    table = wl.cfg4_table(seed=4 + 100 * rank)
    n = len(table)
    nbytes = n * bb
    d_table = torch.from_numpy(table.astype(np.int32)).cuda()
    dst = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    ss = torch.zeros(n, dtype=torch.float32, device="cuda")
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    stream = torch.cuda.Stream()
    st = stream.cuda_stream
    lp = layers.LayerPipeline(pool.ptr, pool.nbytes, d_table.data_ptr(), n, bb, dst.data_ptr(), ss.data_ptr(),
                              tokens_per_tile=32)

    def check(mode):
        rj, to, moved = lp.sync()
        if rj or to or moved != nbytes:
            raise RuntimeError(f"layer pipeline: rejected {rj}, timeouts {to}, bytes {moved}")

    for mode in (layers.RMS, layers.TRANSFER):
        for _ in range(args.warmup):
            lp.run(mode, st)
            check(mode)
    # warm-up check (transfer mode ran last): block 0 holds pool block table[0]
    first = np.ctypeslib.as_array((ctypes.c_uint8 * bb).from_address(pool.ptr + int(table[0]) * bb))
    if not np.array_equal(dst[:bb].cpu().numpy(), first):
        raise RuntimeError("layer pipeline warm-up produced wrong bytes")
    dist.barrier()  # every rank measures its link at the same time
    peak = measure_pcie_peak(ctx, pool.ptr, 256 << 20, stream)
    peak_sum = dist.sum_vec([peak])[0]
    peaks = dist.all_values(peak)

    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    clocks = ClockSampler(int(vis.split(",")[local_rank]) if vis else local_rank)
    clocks.start()
    t_rms = _timed_steps(args, stream, flush, dist, lambda: lp.run(layers.RMS, st), lambda: check(layers.RMS))
    clk = clocks.stop()
    t_xfer = _timed_steps(args, stream, flush, dist, lambda: lp.run(layers.TRANSFER, st),
                          lambda: check(layers.TRANSFER))
    m_rms, m_xfer = dist.max_vec(t_rms), dist.max_vec(t_xfer)

    # e2e: page table from pinned host memory in, sums of squares back out, every step
    h_table = torch.from_numpy(table.astype(np.int32)).pin_memory()
    h_ss = torch.empty(n, dtype=torch.float32).pin_memory()
    e2e = []
    for i in range(args.warmup + args.steps):
        flush.zero_()
        torch.cuda.synchronize()
        dist.barrier()
        t0 = time.perf_counter()
        with torch.cuda.stream(stream):
            d_table.copy_(h_table, non_blocking=True)
            lp.run(layers.RMS, st)
            h_ss.copy_(ss, non_blocking=True)
        stream.synchronize()
        dt = time.perf_counter() - t0
        check(layers.RMS)
        if i >= args.warmup:
            e2e.append(dt)
    m_e2e = dist.max_vec(e2e)

    out = {"value": aggregate_gbs(nbytes, world, m_rms), "ms_per_step": sum(m_rms) / len(m_rms) * 1e3,
           "transfer_only_gbs": aggregate_gbs(nbytes, world, m_xfer),
           "transfer_only_ms": sum(m_xfer) / len(m_xfer) * 1e3, "peak": peak, "peak_sum": peak_sum, "clocks": clk,
           "rank_gbs": dist.all_values(nbytes * len(t_rms) / sum(t_rms) / 1e9), "rank_peaks": peaks,
           "e2e_value": aggregate_gbs(nbytes, world, m_e2e), "bytes": nbytes,
           "h2d": table.nbytes, "d2h": n * 4, "block_threads": lp.block_threads}
    if world == 1 and not args.no_cpu_baseline:
        from tests.golden.cases import oracle_layer_pipeline
        pool_u16 = pool.array(np.uint16)
        sample = table[:1024]
        k, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < 10.0:
            oracle_layer_pipeline(pool_u16, sample, bb)
            k += 1
        dt = time.perf_counter() - t0
        out["cpu_baseline"] = {"value": k * len(sample) * bb / dt / 1e9, "unit": "GB/s", "cores": 1, "kind": "port",
                               "sample": f"layer 0 (1024 blocks) through the C restatement (gather + RMS scale, "
                                         f"one core), {k} passes in {dt:.1f} s"}
    lp.close()
    pool.free()
    ctx.close()
    return out


def run_cfg5(args, rank, local_rank, world, dist):
    """MoE: top-8 routing of 4096 tokens over 64 experts, then the gather of the 32,768
    selected 14,336-byte rows into per-expert segments; one independent shard per GPU."""
    import torch
    import gfd_b200
    from gfd_b200 import workloads as wl

    torch.cuda.set_device(local_rank)
    ctx = gfd_b200.Context(local_rank)
    shard = wl.MoEShard(rank)
    pool = ctx.pool(shard.pool_bytes)
    shard.fill_pool(pool.ptr)
    logits = shard.logits()
    rows = shard.tokens * shard.k
    nbytes = shard.dst_bytes
    d_logits = torch.from_numpy(logits).cuda()
    d_src = torch.from_numpy(shard.token_src(pool.ptr).view(np.int64)).cuda()
    dst = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    d_counts = torch.zeros(shard.experts, dtype=torch.int32, device="cuda")
    d_offsets = torch.zeros(shard.experts, dtype=torch.int32, device="cuda")
    d_entries = torch.empty(rows * 24, dtype=torch.uint8, device="cuda")
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    stream = torch.cuda.Stream()
    st = stream.cuda_stream

    def step():
        ctx.moe_route_gather(d_logits.data_ptr(), shard.tokens, shard.experts, shard.k, d_src.data_ptr(),
                             shard.row_bytes, dst.data_ptr(), nbytes, d_counts.data_ptr(), d_offsets.data_ptr(),
                             d_entries.data_ptr(), stream=st)

    for _ in range(args.warmup):
        step()
    stream.synchronize()
    if ctx.gather_device_status()[0] != gfd_b200.GFD_OK:
        raise RuntimeError(ctx.last_error())
    # warm-up check: every row routed, and row 0 holds the bytes its list entry names
    if int(d_counts.sum()) != rows:
        raise RuntimeError("routing lost rows")
    e0 = d_entries[:24].cpu().numpy().view(gfd_b200.SG_ENTRY_DTYPE)[0]
    first = np.ctypeslib.as_array((ctypes.c_uint8 * shard.row_bytes).from_address(int(e0["src"])))
    if not np.array_equal(dst[:shard.row_bytes].cpu().numpy(), first):
        raise RuntimeError("MoE gather produced wrong bytes")
    dist.barrier()  # every rank measures its link at the same time
    peak = measure_pcie_peak(ctx, pool.ptr, 256 << 20, stream)
    peak_sum = dist.sum_vec([peak])[0]
    peaks = dist.all_values(peak)

    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    clocks = ClockSampler(int(vis.split(",")[local_rank]) if vis else local_rank)
    clocks.start()
    t = _timed_steps(args, stream, flush, dist, step)
    clk = clocks.stop()
    if ctx.gather_device_status()[0] != gfd_b200.GFD_OK:
        raise RuntimeError(ctx.last_error())
    m = dist.max_vec(t)

    # the same shard through SGWarpSpecSession: GPU routing, then one SG-framework kernel
    # whose submitter warp feeds the per-expert lists (device-timed: route + SG kernel)
    sg_out = None
    try:
        from gfd_b200 import moe_sg
        with moe_sg.MoESG() as sg:
            def sg_step(rows_per_list):
                sg.prepare()
                with torch.cuda.stream(stream):
                    flush.zero_()
                stream.synchronize()
                dist.barrier()
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(stream)
                ctx.moe_route_gather(d_logits.data_ptr(), shard.tokens, shard.experts, shard.k, d_src.data_ptr(),
                                     shard.row_bytes, dst.data_ptr(), nbytes, d_counts.data_ptr(),
                                     d_offsets.data_ptr(), d_entries.data_ptr(), stream=st, route_only=True)
                sg.run(d_entries.data_ptr(), d_counts.data_ptr(), d_offsets.data_ptr(), shard.experts, st,
                       rows_per_list=rows_per_list)
                b.record(stream)
                rc, to, moved = sg.sync()
                if rc != gfd_b200.GFD_OK or moved != nbytes:
                    raise RuntimeError(f"SG session pass: rc {rc}, timeouts {to}, bytes {moved}")
                return a.elapsed_time(b) / 1e3

            def sg_measure(rows_per_list):
                for _ in range(args.warmup):
                    sg_step(rows_per_list)
                ts = dist.max_vec([sg_step(rows_per_list) for _ in range(args.steps)])
                return {"value": aggregate_gbs(nbytes, world, ts), "unit": "GB/s",
                        "ms_per_step": sum(ts) / len(ts) * 1e3}
            sg_out = sg_measure(256)
            sg_out["path"] = ("SGWarpSpecSession; a warp of the SG kernel submits each expert's rows as lists of "
                              "at most 256 entries; timed: route + SG kernel")
            sg_out["lists_of_128"] = sg_measure(128)
            sg_out["one_list_per_expert"] = sg_measure(0)
    except (RuntimeError, OSError) as exc:
        sg_out = {"unavailable": str(exc)}

    h_logits = torch.from_numpy(logits).pin_memory()
    h_counts = torch.empty(shard.experts, dtype=torch.int32).pin_memory()
    e2e = []
    for i in range(args.warmup + args.steps):
        flush.zero_()
        torch.cuda.synchronize()
        dist.barrier()
        t0 = time.perf_counter()
        with torch.cuda.stream(stream):
            d_logits.copy_(h_logits, non_blocking=True)
            step()
            h_counts.copy_(d_counts, non_blocking=True)
        stream.synchronize()
        dt = time.perf_counter() - t0
        if i >= args.warmup:
            e2e.append(dt)
    m_e2e = dist.max_vec(e2e)
    out = {"value": aggregate_gbs(nbytes, world, m), "ms_per_step": sum(m) / len(m) * 1e3, "peak": peak,
           "peak_sum": peak_sum, "clocks": clk, "e2e_value": aggregate_gbs(nbytes, world, m_e2e), "bytes": nbytes,
           "rank_gbs": dist.all_values(nbytes * len(t) / sum(t) / 1e9), "rank_peaks": peaks,
           "h2d": logits.nbytes, "d2h": shard.experts * 4, "sg_session": sg_out}
    if world == 1 and not args.no_cpu_baseline:
        from tests.golden.cases import oracle, oracle_moe_route as route
        lib = oracle()
        token_src = shard.token_src(pool.ptr)
        out_buf = np.empty(512 * shard.row_bytes, np.uint8)
        k, t0, moved = 0, time.perf_counter(), 0
        while time.perf_counter() - t0 < 10.0:
            _, _, _, rt = route(logits, shard.k)
            e = gfd_b200.entries_array(np.uint64(out_buf.ctypes.data) +
                                       (np.arange(512, dtype=np.uint64) * np.uint64(shard.row_bytes)),
                                       token_src[rt[:512]], shard.row_bytes)
            lib.gfd_oracle_gather(out_buf.ctypes.data, out_buf.ctypes.data, out_buf.nbytes, e.ctypes.data, len(e))
            moved += out_buf.nbytes
            k += 1
        dt = time.perf_counter() - t0
        out["cpu_baseline"] = {"value": moved / dt / 1e9, "unit": "GB/s", "cores": 1, "kind": "port",
                               "sample": f"full routing of the 4096 x 64 logits + gather of the first 512 routed "
                                         f"rows through the C restatement (one core), {k} passes in {dt:.1f} s"}
    pool.free()
    ctx.close()
    return out


def measure_d2h_peak(pool_ptr, nbytes, stream, iters=10):
    """Contiguous device -> pinned host cudaMemcpyAsync (the scatter's roofline)."""
    import torch
    src = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    dst = torch.from_numpy(np.ctypeslib.as_array((ctypes.c_uint8 * nbytes).from_address(pool_ptr)))
    times = []
    with torch.cuda.stream(stream):
        for i in range(iters + 3):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            dst.copy_(src, non_blocking=True)
            b.record(stream)
            b.synchronize()
            if i >= 3:
                times.append(a.elapsed_time(b) / 1e3)
    del src
    return nbytes / statistics.median(times) / 1e9


def run_d2h(args, rank, local_rank, world, dist):
    """Reverse path: 2048 x 64 KiB HBM blocks scattered into their (cfg2-permuted) slots
    of a 4 GiB pinned pool (KV offload)."""
    import torch
    import gfd_b200
    from gfd_b200 import workloads as wl

    torch.cuda.set_device(local_rank)
    ctx = gfd_b200.Context(local_rank)
    w = wl.cfg2(seed=2 + 100 * rank)
    pool = ctx.pool(w.pool_bytes)
    src = torch.empty(w.total_bytes, dtype=torch.uint8, device="cuda")
    wl.fill_bytes(pool.ptr, w.total_bytes, 7)
    src.copy_(torch.from_numpy(pool.array()[:w.total_bytes].copy()))
    e = w.entries(pool.ptr, src.data_ptr())
    e["dst"], e["src"] = e["src"].copy(), e["dst"].copy()
    nbytes = w.total_bytes
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    stream = torch.cuda.Stream()
    st = stream.cuda_stream

    def step():
        rc = ctx.scatter(e, stream=st)
        if rc != gfd_b200.GFD_OK:
            raise RuntimeError(ctx.last_error())

    for _ in range(args.warmup):
        step()
    stream.synchronize()
    blk = int(w.block_ids[0])
    if not np.array_equal(pool.array()[blk * 65536:(blk + 1) * 65536], src[:65536].cpu().numpy()):
        raise RuntimeError("scatter warm-up produced wrong bytes")
    dist.barrier()
    peak = measure_d2h_peak(pool.ptr + w.total_bytes, 256 << 20, stream)
    peak_sum = dist.sum_vec([peak])[0]
    peaks = dist.all_values(peak)
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    clocks = ClockSampler(int(vis.split(",")[local_rank]) if vis else local_rank)
    clocks.start()
    t = _timed_steps(args, stream, flush, dist, step)
    clk = clocks.stop()
    m = dist.max_vec(t)
    e2e = []
    for i in range(args.warmup + args.steps):
        flush.zero_()
        torch.cuda.synchronize()
        dist.barrier()
        us = ctx.scatter_sync(e)
        if i >= args.warmup:
            e2e.append(us / 1e6)
    m_e2e = dist.max_vec(e2e)
    out = {"value": aggregate_gbs(nbytes, world, m), "ms_per_step": sum(m) / len(m) * 1e3, "peak": peak,
           "peak_sum": peak_sum, "clocks": clk, "e2e_value": aggregate_gbs(nbytes, world, m_e2e), "bytes": nbytes,
           "rank_gbs": dist.all_values(nbytes * len(t) / sum(t) / 1e9), "rank_peaks": peaks,
           "h2d": e.nbytes, "d2h": nbytes}
    pool.free()
    ctx.close()
    return out


class QueueClientLib:
    """GPU-queued submit timed the reference's way (submit kernel + wait kernel + device
    sync, host wall clock): gfd_b200/csrc/queue_client.cu built against this library
    (libgfd_queue_client.so) or against the reference (oracle/_ref/libgfd_ref_queue.so)."""

    def __init__(self, path, device, gpu_ptr, cpu_ptr, total, exclusive_cores=32):
        if path != QUEUE_CLIENT_LIB:
            import gfd_b200  # noqa: F401  (keeps this library's classes local, loaded first)
        lib = ctypes.CDLL(path)
        lib.qc_create.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int]
        lib.qc_create.restype = ctypes.c_void_p
        lib.qc_run.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_uint32, ctypes.c_int,
                               ctypes.c_int, ctypes.c_void_p]
        lib.qc_run.restype = ctypes.c_int
        lib.qc_destroy.argtypes = [ctypes.c_void_p]
        lib.qc_destroy.restype = None
        self.lib = lib
        self.h = lib.qc_create(device, gpu_ptr, cpu_ptr, total, exclusive_cores)
        if not self.h:
            raise RuntimeError(f"qc_create failed ({os.path.basename(path)})")

    def run_us(self, addrs, token_size):
        a = np.ascontiguousarray(addrs, dtype=np.uint64)
        us = np.zeros(1, np.float64)
        rc = self.lib.qc_run(self.h, a.ctypes.data, len(a), token_size, 0, 1, us.ctypes.data)
        if rc != 0:
            raise RuntimeError(f"queue client: rc {rc}")
        return float(us[0])

    def close(self):
        if self.h:
            self.lib.qc_destroy(self.h)
            self.h = None


_REF = None


def ref_lib():
    """oracle/_ref/libgfd_ref.so with its argument types (the reference's own sources plus
    the harness: GFD Direct, Memcpy(N), allocation, L2 flush, verification, generators)."""
    global _REF
    if _REF is None:
        lib = ctypes.CDLL(REF_LIB)
        vp = ctypes.c_void_p
        lib.ref_direct_create.argtypes = [ctypes.c_int, vp, vp, ctypes.c_size_t, ctypes.c_int, ctypes.c_int]
        lib.ref_direct_create.restype = vp
        lib.ref_direct_submit.argtypes = [vp, vp, ctypes.c_int]
        lib.ref_direct_submit.restype = ctypes.c_double
        lib.ref_direct_destroy.argtypes = [vp]
        lib.ref_direct_workers.argtypes = [vp]
        lib.ref_direct_workers.restype = ctypes.c_int
        lib.ref_memcpy_n.argtypes = [vp, ctypes.c_int, vp]
        lib.ref_memcpy_n.restype = ctypes.c_double
        lib.ref_set_device.argtypes = [ctypes.c_int]
        lib.ref_set_device.restype = ctypes.c_int
        for f in ("ref_host_alloc", "ref_dev_alloc"):
            getattr(lib, f).argtypes = [ctypes.c_size_t]
            getattr(lib, f).restype = vp
        for f in ("ref_host_free", "ref_dev_free"):
            getattr(lib, f).argtypes = [vp]
            getattr(lib, f).restype = None
        lib.ref_l2_flush.argtypes = [vp, ctypes.c_size_t]
        lib.ref_l2_flush.restype = ctypes.c_int
        lib.ref_verify.argtypes = [vp, ctypes.c_int, vp, ctypes.c_size_t]
        lib.ref_verify.restype = ctypes.c_longlong
        _REF = lib
    return _REF


class RefLib:
    """The reference's GFD Direct and Memcpy(N) (oracle/_ref/libgfd_ref.so), one instance."""

    def __init__(self, device, dst_ptr, pool_ptr, staging_bytes):
        lib = ref_lib()
        self.lib = lib
        self.h = lib.ref_direct_create(device, ctypes.c_void_p(dst_ptr), ctypes.c_void_p(pool_ptr),
                                       staging_bytes, 0, 32)
        if not self.h:
            raise RuntimeError("reference GFD Direct failed to initialise")
        self.workers = lib.ref_direct_workers(self.h)

    def direct_us(self, e):
        return self.lib.ref_direct_submit(self.h, e.ctypes.data, len(e))

    def memcpy_n_us(self, e, stream):
        return self.lib.ref_memcpy_n(e.ctypes.data, len(e), ctypes.c_void_p(stream))

    def close(self):
        if self.h:
            self.lib.ref_direct_destroy(self.h)
            self.h = None


def run_sweep(args, local_rank):
    """Config 1 and config 3 sweeps: p50 latency -> GB/s for every method (the reference's
    own methodology, examples/04_benchmark.cu: warm-up, then p50 of the calls), L2
    flushed before every call.  Prints one JSON line per point and a markdown table."""
    import torch
    import gfd_b200
    from gfd_b200 import workloads as wl

    torch.cuda.set_device(local_rank)
    ctx = gfd_b200.Context(local_rank)
    points = [(256, 4096)] + [(2048, s) for s in wl.CFG3_SIZES] + [(n, 4096) for n in wl.CFG3_COUNTS]
    max_total = max(n * s for n, s in points)
    max_pool = max(2 * n * s for n, s in points)
    pool = ctx.pool(max_pool)
    wl.fill_bytes(pool.ptr, max_pool, 3)
    dst = torch.empty(max_total, dtype=torch.uint8, device="cuda")
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    stream = torch.cuda.Stream()
    ref = RefLib(local_rank, dst.data_ptr(), pool.ptr, max_total) if os.path.exists(REF_LIB) else None
    W, K = 5, args.steps

    def p50(fn):
        ts = []
        for i in range(W + K):
            flush.zero_()
            torch.cuda.synchronize()
            t = fn()
            if i >= W:
                ts.append(t)
        return statistics.median(ts)

    rows = []
    for n, size in points:
        w = wl.Workload(f"{n}x{size}", pool_bytes=2 * n * size, dst_bytes=n * size, num_tokens=n,
                        token_size=size, kind="bytes", seed=3, stride=2 * size)
        e = w.entries(pool.ptr, dst.data_ptr())
        nbytes = n * size
        d_e = torch.from_numpy(e.view(np.uint8).copy()).cuda()

        def dev_us():
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            ctx.gather_device(d_e.data_ptr(), n, dst.data_ptr(), nbytes, stream=stream.cuda_stream)
            b.record(stream)
            b.synchronize()
            return a.elapsed_time(b) * 1e3

        r = {"tokens": n, "token_bytes": size, "bytes": nbytes,
             "default_e2e_us": p50(lambda: ctx.gather_sync(e)),
             "pull_e2e_us": p50(lambda: ctx.gather_sync(e, flags=gfd_b200.GATHER_FORCE_PULL)),
             "pull_device_us": p50(dev_us),
             "ce_e2e_us": p50(lambda: ctx.gather_sync(e, flags=gfd_b200.GATHER_FORCE_CE))}
        if ref is not None:
            r["ref_direct_us"] = p50(lambda: ref.direct_us(e))
            r["ref_memcpy_n_us"] = p50(lambda: ref.memcpy_n_us(e, stream.cuda_stream))
        for k in [k for k in r if k.endswith("_us")]:
            r[k.replace("_us", "_gbs")] = nbytes / (r[k] / 1e6) / 1e9
        rows.append(r)
        print(json.dumps(r), flush=True)
    if ref is not None:
        ref.close()
    # GPU-queued submit (descriptor ring), ours then the reference's, one client each
    # for the whole pass so only one consumer runs at a time
    for key, path in (("queue", QUEUE_CLIENT_LIB), ("ref_queue", REF_QUEUE_LIB)):
        if not os.path.exists(path):
            continue
        qc = QueueClientLib(path, local_rank, dst.data_ptr(), pool.ptr, max_pool)
        try:
            for r in rows:
                n, size = r["tokens"], r["token_bytes"]
                addrs = np.uint64(pool.ptr) + np.arange(n, dtype=np.uint64) * np.uint64(2 * size)
                r[key + "_us"] = p50(lambda: qc.run_us(addrs, size))
                r[key + "_gbs"] = r["bytes"] / (r[key + "_us"] / 1e6) / 1e9
        except RuntimeError as exc:
            print(json.dumps({"path": key, "error": str(exc)}), flush=True)
        finally:
            qc.close()
    for r in rows:
        if "queue_us" in r or "ref_queue_us" in r:
            print(json.dumps({k: r[k] for k in ("tokens", "token_bytes", "queue_gbs", "ref_queue_gbs") if k in r}))
    pool.free()
    ctx.close()
    cols = ["default_e2e_gbs", "pull_e2e_gbs", "pull_device_gbs", "ce_e2e_gbs", "queue_gbs", "ref_direct_gbs",
            "ref_memcpy_n_gbs", "ref_queue_gbs"]
    print("\n| tokens x size | total | " + " | ".join(cols) + " |")
    print("|---|---|" + "---|" * len(cols))
    for r in rows:
        print(f"| {r['tokens']} x {r['token_bytes']} | {r['bytes'] >> 10} KiB | " +
              " | ".join(f"{r.get(c, float('nan')):.2f}" for c in cols) + " |")


def run_profile_target(local_rank, config="cfg2"):
    """A short, untimed run of a benchmark workload for ncu (no JSON line).

    cfg2  5 device-entry gathers (plan + pull); the kernels of interest are launches 3..5
    cfg4  a 4-layer pass (4 x 1024 page-table blocks of 64 KiB from a 4 GiB pool) run
          4 times through the layer pipeline (RMS-scale compute); launches 2..4
    cfg5  5 MoE steps (topk, emit, plan, pull) on the full shard; steps 3..5
    d2h   5 scatters of cfg2's blocks back into the pool (pull kernel, host destinations)
    cfg3_4k  5 calls of 2048 x 4 KiB at 2x stride through gfd_gather_sync with the SM pull
          forced (one pull launch each, host-built table), then 5 through
          gfd_gather_device (plan_kernel + pull_kernel, table in HBM)
    cfg5_sg  3 passes of half a config 5 shard (2048 tokens, 16,384 rows) through
          SGWarpSpecSession with 128-row lists (one moe_sg_kernel launch each)
    cfg2_bulk  config 2 through gfd_gather_sync: 5 calls with the 16-byte-load pull
          (pull_kernel), then 5 with the cp.async.bulk pull (pull_bulk_kernel); the two
          results are compared byte for byte
    cfg1  config 1 (256 x 4 KiB at 2x stride, 1 MiB): 5 calls through gfd_gather_sync
          (pull_kernel, host-built table), then 5 through gfd_gather_device
          (list_pull_kernel), each compared with the pool
    """
    import torch
    import gfd_b200
    from gfd_b200 import workloads as wl

    torch.cuda.set_device(local_rank)
    ctx = gfd_b200.Context(local_rank)
    ok = True
    if config == "cfg4":
        from gfd_b200 import layers
        bb = wl.CFG4_BLOCK_BYTES
        pool = ctx.pool(wl.CFG4_POOL_BLOCKS * bb)
        wl.cfg4_fill_pool(pool.ptr)
        table = wl.cfg4_table(layers=4)
        d_table = torch.from_numpy(table.astype(np.int32)).cuda()
        dst = torch.empty(len(table) * bb, dtype=torch.uint8, device="cuda")
        ss = torch.zeros(len(table), dtype=torch.float32, device="cuda")
        with layers.LayerPipeline(pool.ptr, pool.nbytes, d_table.data_ptr(), len(table), bb, dst.data_ptr(),
                                  ss.data_ptr(), tokens_per_tile=32) as lp:
            for _ in range(4):
                lp.run(layers.RMS)
                ok = ok and lp.sync()[:2] == (0, 0)
    elif config == "cfg5":
        shard = wl.MoEShard(0)
        pool = ctx.pool(shard.pool_bytes)
        shard.fill_pool(pool.ptr)
        d_logits = torch.from_numpy(shard.logits()).cuda()
        d_src = torch.from_numpy(shard.token_src(pool.ptr).view(np.int64)).cuda()
        dst = torch.empty(shard.dst_bytes, dtype=torch.uint8, device="cuda")
        cnt = torch.zeros(2 * shard.experts, dtype=torch.int32, device="cuda")
        ent = torch.empty(shard.tokens * shard.k * 24, dtype=torch.uint8, device="cuda")
        for _ in range(5):
            ctx.moe_route_gather(d_logits.data_ptr(), shard.tokens, shard.experts, shard.k, d_src.data_ptr(),
                                 shard.row_bytes, dst.data_ptr(), shard.dst_bytes, cnt.data_ptr(),
                                 cnt.data_ptr() + 4 * shard.experts, ent.data_ptr())
        ok = ctx.gather_device_status()[0] == gfd_b200.GFD_OK
    elif config == "cfg5_sg":
        from gfd_b200 import moe_sg
        shard = wl.MoEShard(0, tokens=2048)  # half the benchmark shard: 16,384 rows, 235 MB
        pool = ctx.pool(shard.pool_bytes)
        shard.fill_pool(pool.ptr)
        d_logits = torch.from_numpy(shard.logits()).cuda()
        d_src = torch.from_numpy(shard.token_src(pool.ptr).view(np.int64)).cuda()
        dst = torch.empty(shard.dst_bytes, dtype=torch.uint8, device="cuda")
        cnt = torch.zeros(2 * shard.experts, dtype=torch.int32, device="cuda")
        ent = torch.empty(shard.tokens * shard.k * 24, dtype=torch.uint8, device="cuda")
        stream = torch.cuda.Stream()
        with moe_sg.MoESG() as sg:
            for _ in range(3):
                sg.prepare()
                ctx.moe_route_gather(d_logits.data_ptr(), shard.tokens, shard.experts, shard.k, d_src.data_ptr(),
                                     shard.row_bytes, dst.data_ptr(), shard.dst_bytes, cnt.data_ptr(),
                                     cnt.data_ptr() + 4 * shard.experts, ent.data_ptr(), stream=stream.cuda_stream,
                                     route_only=True)
                sg.run(ent.data_ptr(), cnt.data_ptr(), cnt.data_ptr() + 4 * shard.experts, shard.experts,
                       stream.cuda_stream, rows_per_list=128)
                rc, to, moved = sg.sync()
                ok = ok and rc == gfd_b200.GFD_OK and moved == shard.dst_bytes
    elif config == "cfg1":
        w = wl.cfg1()
        pool = ctx.pool(w.pool_bytes)
        w.fill_pool(pool.ptr)
        dst = torch.zeros(w.total_bytes, dtype=torch.uint8, device="cuda")
        torch.cuda.synchronize()
        entries = w.entries(pool.ptr, dst.data_ptr())
        want = pool.array()[:w.pool_bytes].reshape(w.num_tokens, 2, w.token_size)[:, 0, :].reshape(-1)
        for _ in range(5):
            ok = ok and ctx.gather_sync_rc(entries) == gfd_b200.GFD_OK
        ok = ok and np.array_equal(dst.cpu().numpy(), want)
        dst.zero_()
        torch.cuda.synchronize()
        d_entries = torch.from_numpy(entries.view(np.uint8).copy()).cuda()
        for _ in range(5):
            ctx.gather_device(d_entries.data_ptr(), w.num_tokens, dst.data_ptr(), w.total_bytes)
        ok = ok and ctx.gather_device_status() == (gfd_b200.GFD_OK, -1)
        ok = ok and np.array_equal(dst.cpu().numpy(), want)
    elif config == "cfg3_4k":
        w = wl.cfg3(2048, 4096)
        pool = ctx.pool(w.pool_bytes)
        w.fill_pool(pool.ptr)
        dst = torch.empty(w.total_bytes, dtype=torch.uint8, device="cuda")
        entries = w.entries(pool.ptr, dst.data_ptr())
        for _ in range(5):
            ok = ok and ctx.gather_sync_rc(entries, gfd_b200.GATHER_FORCE_PULL) == gfd_b200.GFD_OK
        # then the benchmarked device-entry path (plan + pull, table in HBM), 5 calls
        d_entries = torch.from_numpy(entries.view(np.uint8).copy()).cuda()
        for _ in range(5):
            ctx.gather_device(d_entries.data_ptr(), w.num_tokens, dst.data_ptr(), w.total_bytes)
        ok = ok and ctx.gather_device_status()[0] == gfd_b200.GFD_OK
    else:
        w = wl.cfg2()
        pool = ctx.pool(w.pool_bytes)
        w.fill_pool(pool.ptr)
        dst = torch.empty(w.total_bytes, dtype=torch.uint8, device="cuda")
        entries = w.entries(pool.ptr, dst.data_ptr())
        if config == "d2h":
            entries["dst"], entries["src"] = entries["src"].copy(), entries["dst"].copy()
            for _ in range(5):
                ok = ok and ctx.scatter_sync_rc(entries) == gfd_b200.GFD_OK
        elif config == "cfg2_bulk":
            for _ in range(5):
                ok = ok and ctx.gather_sync_rc(entries, gfd_b200.GATHER_FORCE_PULL) == gfd_b200.GFD_OK
            first = dst.clone()
            dst.zero_()
            torch.cuda.synchronize()  # the library's stream is not ordered after torch's
            for _ in range(5):
                ok = ok and ctx.gather_sync_rc(entries, gfd_b200.GATHER_BULK_STAGE) == gfd_b200.GFD_OK
            ok = ok and bool(torch.equal(first, dst))
        else:
            d_entries = torch.from_numpy(entries.view(np.uint8).copy()).cuda()
            for _ in range(5):
                ctx.gather_device(d_entries.data_ptr(), w.num_tokens, dst.data_ptr(), w.total_bytes)
            ok = ctx.gather_device_status()[0] == gfd_b200.GFD_OK
    torch.cuda.synchronize()
    pool.free()
    ctx.close()
    if not ok:
        raise SystemExit("profile target: the workload failed")


def run_reference(args, rank, local_rank, world):
    """--impl reference: the reference's own GFD Direct (CpuPollingThread::submit_direct,
    compiled from its sources into oracle/_ref/libgfd_ref.so) on this box's host cores, on
    the headline workload.  This arm loads no library of this repository: the source pool
    comes from cudaMallocHost and the destination from cudaMalloc, as the reference's
    benchmark allocates them (examples/04_benchmark.cu:346-356), through the harness
    linked into libgfd_ref.so, which also carries the seeded generators.  L2 is flushed
    before every call, as in the other arm; every gathered byte is compared with its
    source afterwards."""
    if not os.path.exists(REF_LIB):
        return {"unavailable": "reference library oracle/_ref/libgfd_ref.so was not built (make -C oracle)"}
    from gfd_b200 import workloads as wl
    wl.use_generator_library(REF_LIB)
    lib = ref_lib()
    if lib.ref_set_device(local_rank) != 0:
        return {"unavailable": f"cudaSetDevice({local_rank}) failed"}
    w = wl.cfg2()
    pool = lib.ref_host_alloc(w.pool_bytes)
    dst = lib.ref_dev_alloc(w.total_bytes)
    flush = lib.ref_dev_alloc(256 << 20)
    if not (pool and dst and flush):
        return {"unavailable": "cudaMallocHost / cudaMalloc of the workload failed"}
    try:
        w.fill_pool(pool)
        entries = np.ascontiguousarray(w.entries(pool, dst))
        try:
            ref = RefLib(local_rank, dst, pool, w.total_bytes)
        except RuntimeError:
            return {"unavailable": "reference GFD Direct failed to initialise on this box"}
        try:
            for _ in range(max(args.warmup, 3)):
                lib.ref_l2_flush(ctypes.c_void_p(flush), 256 << 20)
                ref.direct_us(entries)
            direct_us = []
            for _ in range(args.steps):
                lib.ref_l2_flush(ctypes.c_void_p(flush), 256 << 20)
                direct_us.append(ref.direct_us(entries))
            if min(direct_us) < 0:
                return {"unavailable": "reference GFD Direct returned an error on this box"}
            bad = lib.ref_verify(entries.ctypes.data, len(entries), ctypes.c_void_p(dst), w.total_bytes)
            if bad != -1:
                return {"unavailable": f"reference GFD Direct produced wrong bytes on this box (entry {bad})"}
            memcpy_us = []
            for _ in range(3 + max(3, args.steps // 4)):
                lib.ref_l2_flush(ctypes.c_void_p(flush), 256 << 20)
                memcpy_us.append(ref.memcpy_n_us(entries, 0))
            memcpy_us = memcpy_us[3:]
            workers = ref.workers
        finally:
            ref.close()
    finally:
        lib.ref_dev_free(ctypes.c_void_p(flush))
        lib.ref_dev_free(ctypes.c_void_p(dst))
        lib.ref_host_free(ctypes.c_void_p(pool))
    total_s = sum(direct_us) / 1e6
    return {"value": w.total_bytes * args.steps / total_s / 1e9, "ms_per_step": total_s / args.steps * 1e3,
            "workers": workers, "p50_us": statistics.median(direct_us),
            "memcpy_n_gbs": w.total_bytes / (statistics.median(memcpy_us) / 1e6) / 1e9}


def run_secondary(args, rank, local_rank, world):
    """cfg4 / cfg5 lines (same contract as the headline line)."""
    dist = Dist(world)
    try:
        if args.config == "cfg4":
            r = run_cfg4(args, rank, local_rank, world, dist)
            config = {"workload": "cfg4_layer_pipeline", "layers": 32, "blocks_per_layer": 1024,
                      "block_bytes": 65536, "pool_bytes": 65536 * 65536,
                      "selection": "page table: layer l = first 1024 ids of a permutation seeded 4 + l",
                      "compute": "per-block fp32 sum of squares + in-place bf16 scale by 1/sqrt(ss/n + 1e-6)",
                      "launch": f"one WarpSpecSession launch per pass, {r['block_threads']} threads/CTA "
                                "(4 producer + 8 compute warps), tokens_per_tile 32",
                      "l2": "flushed (256 MiB memset) before every timed step; 2 GiB per pass",
                      "parallelism": f"independent replica per GPU x{world} (no data-path collective)"}
            dtype, kernel, launches = "bf16", "layers_rms_kernel (WarpSpec page-table mode)", 1
        elif args.config == "d2h":
            r = run_d2h(args, rank, local_rank, world, dist)
            config = {"workload": "d2h_kv_block_offload", "blocks": 2048, "block_bytes": 65536,
                      "pool_bytes": 65536 * 65536,
                      "selection": "cfg2 permutation: HBM block j -> pool slot perm[j]",
                      "l2": "flushed (256 MiB memset) before every timed step",
                      "parallelism": f"independent replica per GPU x{world} (no data-path collective)"}
            dtype, kernel, launches = "u8", "gfdb::pull_kernel (device -> host roles)", 1
        else:
            r = run_cfg5(args, rank, local_rank, world, dist)
            config = {"workload": "cfg5_moe_route_gather", "tokens": 4096, "experts": 64, "top_k": 8,
                      "row_bytes": 14336, "pool_rows": 262144,
                      "routing": "top-8 over fp32 N(0,1) logits (seed 5+rank), ties to the lower id",
                      "l2": "flushed (256 MiB memset) before every timed step",
                      "parallelism": f"independent shard per GPU x{world} (no data-path collective)"}
            dtype, kernel, launches = "u8", "gfdb::pull_kernel (after topk, emit and the plan kernels)", 6
        if rank == 0:
            achieved = r["bytes"] / (r["ms_per_step"] / 1e3) / 1e9
            line = {"metric": METRIC, "value": r["value"], "unit": "GB/s", "n_gpus": world, "steps": args.steps,
                    "warmup": args.warmup, "ms_per_step": r["ms_per_step"], "higher_is_better": True,
                    "scaling": "weak", "vs_baseline": None, "dtype": dtype, "data": "synthetic (seeded)",
                    "config": config, "per_gpu_gbs": r["value"] / world,
                    "fraction_of_pcie_peak": (r["value"] / world) / r["peak"],
                    "aggregate_peak_concurrent": r["peak_sum"],
                    "fraction_of_aggregate_peak": r["value"] / r["peak_sum"],
                    "roofline": {"bound": "pcie", "achieved": achieved, "peak": r["peak"], "unit": "GB/s",
                                 "frac": achieved / r["peak"], "kernel": kernel,
                                 "traffic": (load_profile_traffic(args.config) or {}).get("dram_bytes_per_launch"),
                                 "traffic_note": "DRAM read+write bytes per launch of the kernel (ncu, "
                                                 "profiles/kernel_traffic.txt); the bound is PCIe",
                                 "peak_source": "contiguous pinned cudaMemcpyAsync %s, 256 MiB, median of 10, "
                                                "measured in this run" % ("D2H" if args.config == "d2h" else "H2D")},
                    "e2e": {"value": r["e2e_value"], "unit": "GB/s", "h2d_bytes_per_step": r["h2d"],
                            "d2h_bytes_per_step": r["d2h"]},
                    "gpu_launches": launches * args.steps, "clocks": r["clocks"]}
            line["gpus_active"] = world
            if world > 1:
                line["per_rank"] = {"gbs": r["rank_gbs"], "concurrent_peak_gbs": r["rank_peaks"],
                                    "note": "value is bound by the slowest rank (max over ranks per step)"}
            if "transfer_only_gbs" in r:
                line["transfer_only"] = {"value": r["transfer_only_gbs"], "unit": "GB/s",
                                         "ms_per_step": r["transfer_only_ms"]}
            if r.get("sg_session") is not None:
                line["sg_session"] = r["sg_session"]
            if "cpu_baseline" in r:
                line["cpu_baseline"] = r["cpu_baseline"]
            print(json.dumps(line))
    finally:
        dist.close()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--equal-shards", action="store_true",
                    help="N > 1: every rank pulls its own 2048 blocks (no link-rate forwarding over NVLink)")
    ap.add_argument("--no-shared-pool", action="store_true",
                    help="N > 1: skip the shared-pool measurement (equal and rate-proportional shards)")
    ap.add_argument("--sweep", action="store_true",
                    help="config 1 + config 3 sweeps (ours, copy-engine path, reference paths); table output")
    ap.add_argument("--config", choices=["cfg2", "cfg4", "cfg5", "d2h", "cfg1", "cfg3_4k", "cfg5_sg", "cfg2_bulk"],
                    default="cfg2",
                    help="cfg2 KV block fetch (headline); cfg4 layer pipeline with RMS-scale compute; "
                         "cfg5 MoE routing + per-expert gather; d2h the reverse scatter of cfg2's blocks; "
                         "cfg1 (with --profile only) 256 x 4 KiB at 2x stride, host and device entries; "
                         "cfg3_4k (with --profile only) 2048 x 4 KiB at 2x stride through the C ABI; "
                         "cfg5_sg (with --profile only) half a config 5 shard through SGWarpSpecSession; "
                         "cfg2_bulk (with --profile only) config 2 with the 16-byte-load and the bulk-copy pull")
    ap.add_argument("--profile", action="store_true",
                    help="profiling target: a few untimed steps of --config's workload, no JSON line")
    args = ap.parse_args()
    if args.config in ("cfg1", "cfg3_4k", "cfg5_sg", "cfg2_bulk") and not args.profile:
        ap.error(f"--config {args.config} is a profiling target (use it with --profile)")
    args.warmup = max(args.warmup, 3)
    rank, local_rank, world = dist_env()

    config = {"workload": "cfg2_kv_block_fetch", "blocks": 2048, "block_bytes": 65536,
              "pool_bytes": 65536 * 65536, "block_layout": "bf16[16 tok][8 heads][128 dim][K,V]",
              "selection": "seeded Fisher-Yates permutation, first 2048 of 65536",
              "l2": "flushed (256 MiB memset) before every timed step; 4 GiB source pool",
              "parallelism": f"independent replica per GPU x{world} (no data-path collective)"}

    if args.impl == "reference":
        if rank != 0:
            return
        r = run_reference(args, rank, local_rank, world)
        line = {"metric": METRIC, "impl": "reference", "unit": "GB/s", "n_gpus": world, "ranks_timed": 1,
                "ranks_note": (f"launched on {world} GPU(s); rank 0 alone runs the reference's CPU path (one "
                               "GPU's replica) and the other ranks exit without work"),
                "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "u8", "data": "synthetic (seeded)", "config": config}
        if "unavailable" in r:
            print(json.dumps({"impl": "reference", "unavailable": r["unavailable"]}))
            return
        line.update({"value": r["value"], "ms_per_step": r["ms_per_step"],
                     "cpu_baseline": {"value": r["value"], "unit": "GB/s", "cores": r["workers"] + 1,
                                      "kind": "reference",
                                      "sample": "full workload per step via CpuPollingThread::submit_direct "
                                                f"({r['workers']} gather workers + caller; CPU gather + copy engine); "
                                                "pool from cudaMallocHost, destination from cudaMalloc, every "
                                                "byte verified after the timed calls"},
                     "e2e": {"value": r["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
                     "reference_memcpy_n_gbs": r["memcpy_n_gbs"]})
        print(json.dumps(line))
        return

    if args.profile:
        run_profile_target(local_rank, args.config)
        return
    if args.sweep:
        if rank == 0:
            run_sweep(args, local_rank)
        return

    if args.config in ("cfg4", "cfg5", "d2h"):
        run_secondary(args, rank, local_rank, world)
        return

    dist = Dist(world)
    try:
        r = run_ours(args, rank, local_rank, world, dist)
        if rank == 0:
            traffic = load_profile_traffic()
            achieved = r["bytes"] * world / (r["ms_per_step"] / 1e3) / 1e9 / world
            line = {
                "metric": METRIC, "value": r["value"], "unit": "GB/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": r["ms_per_step"], "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "u8", "data": "synthetic (seeded)",
                "config": config,
                "per_gpu_gbs": r["value"] / world,
                "fraction_of_pcie_peak": (r["value"] / world) / r["peak"],
                "aggregate_peak_concurrent": r["peak_sum"],
                "fraction_of_aggregate_peak": r["value"] / r["peak_sum"],
                "roofline": {"bound": "pcie", "achieved": achieved, "peak": r["peak"], "unit": "GB/s",
                             "frac": achieved / r["peak"],
                             "peak_source": "contiguous pinned cudaMemcpyAsync H2D, 256 MiB, median of 10, "
                                            "measured in this run (MEASURED_PEAKS.json has no PCIe figure)",
                             "kernel": "gfdb::pull_kernel (+ gfdb::plan_kernel, <1% of the step)",
                             "traffic": traffic.get("dram_bytes_per_launch") if traffic else None,
                             "traffic_note": "DRAM read+write bytes per launch (ncu); the bound is PCIe: "
                                             "pcie read bytes per launch = %s for %s payload bytes"
                                             % ((traffic or {}).get("pcie_read_bytes_per_launch"),
                                                (traffic or {}).get("payload_bytes_per_launch"))},
                "e2e": {"value": r["e2e_value"], "unit": "GB/s", "p50_us": r["e2e_p50_us"],
                        "h2d_bytes_per_step": r["bytes"] + r["entries_bytes"], "d2h_bytes_per_step": r["d2h_bytes"]},
                "gpu_launches": r["launches_per_step"] * args.steps,
                "clocks": r["clocks"],
                "gpus_active": world,
            }
            if world > 1:
                line["per_rank"] = {"gbs": r["rank_gbs"], "concurrent_peak_gbs": r["rank_peaks"],
                                    "note": "GB/s each rank pulled over its own host link; value is the job's "
                                            "bytes over the slowest rank's time per step (max over ranks)"}
                for k in ("forwarding", "equal_shards", "shared_pool"):
                    if k in r:
                        line[k] = r[k]
            if "cpu_baseline" in r:
                line["cpu_baseline"] = r["cpu_baseline"]
            line["cfg3_4k"] = r["cfg3_4k"]
            line["pull_variants_e2e"] = dict(r["pull_variants"], unit="GB/s",
                                             note="gfd_gather_sync on host entries (table build, pull, completion "
                                                  "word), one call per step with the 16-byte-load pull and with "
                                                  "the cp.async.bulk pull (GFD_GATHER_BULK_STAGE)")
            print(json.dumps(line))
    finally:
        dist.close()


if __name__ == "__main__":
    main()
