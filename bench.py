#!/usr/bin/env python
"""Benchmark of the KernelIntrinsics B200 primitives (one JSON line on rank 0).

Headline workload: the vectorised byte copy (copyto!) of 2^28 bytes.  One step copies 2^28 bytes
once for each of the 256 (src_offset, dst_offset) pairs in 0..15 x 0..15, so every step exercises
every relative misalignment.  Every rank copies its own buffers (weak scaling, no collective).

The same line carries, under "kernels", the other device-wide primitives on their own workloads:
  reduce   Float32 sum, n = 2^24 (L2 flushed between steps; inputs are smaller than L2)
  scan     Int64 inclusive scan, n = 2^30, range-sharded over the ranks + NCCL all-gather of totals
  scan_f32 Float32 cumsum (generic scan, Float64 accumulation), n = 2^28 per rank
  compact  filter/findall of x > 0.5 over 2^28 N(0,1) Float32, range-sharded + all-gather of counts
  gemm     fp8 e4m3 GEMM 8192^3 with Float32 output (replicas at N > 1)

--impl reference times the reference semantics' CPU implementation (the C oracle, all host
threads) on the headline workload, rank 0 only.

Launch: python bench.py [--gpus N --steps K --warmup W]; N > 1 under torch.distributed.run.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO / "kernelintrinsics.jl_b200"))

COPY_BYTES = 1 << 28
REDUCE_N = 1 << 24
SCAN_N = 1 << 30
SCAN_F32_N = 1 << 28
COMPACT_N = 1 << 28
GEMM_MNK = 8192
L2_FLUSH_BYTES = 256 << 20

FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0

# Per-launch DRAM traffic (dram__bytes_read.sum + dram__bytes_write.sum) from one ncu capture of the
# headline kernel (ncu flushes L2 before the capture, so ~50 MB of the launch's writes are still in
# L2 when it ends); the capture and its command are summarised in profiles/.
NCU_TRAFFIC_PER_LAUNCH = {
    "vcopy_kernel": 486_999_808,
}


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--no-extra", action="store_true", help="headline copy only")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--cpu-seconds", type=float, default=10.0)
    p.add_argument("--only", default="", help="comma list of kernels to run under 'kernels'")
    p.add_argument("--profile", default="", choices=["", "copy", "reduce", "scan", "compact", "gemm", "scan_f32", "scan_u8", "rows", "copy2d",
                            "count"],
                   help="run only this kernel, --profile-launches times, on a small case (for ncu)")
    p.add_argument("--profile-n", type=int, default=0, help="elements (bytes for copy; M=N=K for gemm)")
    p.add_argument("--profile-launches", type=int, default=3)
    return p.parse_args()


def run_profile(args):
    """A small case of one kernel: 2 warm-up launches, then --profile-launches timed launches."""
    import torch

    torch.cuda.set_device(0)
    import kernelintrinsics as KI

    dev = torch.device("cuda", 0)
    k = args.profile
    n = args.profile_n
    if k == "copy":
        n = n or COPY_BYTES
        src = torch.empty(n + 16, dtype=torch.uint8, device=dev)
        KI.fill_bytes(src, seed=2)
        dst = torch.empty_like(src)
        fn = lambda: KI.vcopy(dst, src, n, dst_offset=3, src_offset=7)
        alg = 2 * n
    elif k == "reduce":
        n = n or REDUCE_N
        x = torch.empty(n, dtype=torch.float32, device=dev)
        KI.fill_uniform(x, seed=1)
        out = torch.empty((), dtype=torch.float64, device=dev)
        fn = lambda: KI.warpfold_reduce(x, out_f64=out)
        alg = 4 * n
    elif k == "scan":
        n = n or (1 << 26)
        x = torch.empty(n, dtype=torch.int64, device=dev)
        KI.fill_int_range(x, seed=3, lo=-1000, hi=1000)
        y = torch.empty_like(x)
        fn = lambda: KI.warpreduce_scan(x, out=y)
        alg = 16 * n
    elif k == "compact":
        n = n or (1 << 26)
        x = torch.empty(n, dtype=torch.float32, device=dev)
        KI.fill_normal(x, seed=4)
        v = torch.empty_like(x)
        i = torch.empty(n, dtype=torch.int32, device=dev)
        c = torch.zeros((), dtype=torch.uint64, device=dev)
        fn = lambda: KI.vote_compact(x, 0.5, out_vals=v, out_idx=i, count=c, trim=False)
        alg = 4 * n + 8 * int(0.30854 * n)
    elif k == "scan_f32":
        n = n or (1 << 26)
        x = torch.empty(n, dtype=torch.float32, device=dev)
        KI.fill_uniform(x, seed=1)
        y = torch.empty_like(x)
        fn = lambda: KI.scan(x, "+", out=y)
        alg = 8 * n
    elif k == "scan_u8":
        n = n or (1 << 26)  # UInt8 cumsum into UInt64
        x = torch.empty(n, dtype=torch.uint8, device=dev)
        KI.fill_bytes(x, seed=2)
        y = torch.empty(n, dtype=torch.uint64, device=dev)
        fn = lambda: KI.scan(x, "+", out=y)
        alg = 9 * n
    elif k == "copy2d":
        n = n or 8192  # rows of 32 KiB between pitches 33000 and 40000, odd offsets
        src = torch.empty(n * 33000 + 16, dtype=torch.uint8, device=dev)
        KI.fill_bytes(src, seed=2)
        dst = torch.empty(n * 40000 + 16, dtype=torch.uint8, device=dev)
        fn = lambda: KI.vcopy_2d(dst, 40000, src, 33000, 32768, n, dst_offset=3, src_offset=11)
        alg = 2 * 32768 * n
    elif k == "count":
        n = n or (1 << 26)  # count(>(0.5), x) over N(0,1) Float32
        x = torch.empty(n, dtype=torch.float32, device=dev)
        KI.fill_normal(x, seed=4)
        c = torch.zeros((), dtype=torch.uint64, device=dev)
        fn = lambda: KI.count(x, ">", 0.5, out=c)
        alg = 4 * n
    elif k == "rows":
        n = n or 8192  # n x n Float32, one sum per row
        x = torch.empty((n, n), dtype=torch.float32, device=dev)
        KI.fill_uniform(x.view(-1), seed=1)
        y = torch.empty(n, dtype=torch.float32, device=dev)
        fn = lambda: KI.reduce_rows(x, "+", out=y)
        alg = 4 * n * n
    else:
        n = n or 4096
        A = torch.empty((n, n), dtype=torch.uint8, device=dev)
        B = torch.empty((n, n), dtype=torch.uint8, device=dev)
        KI.fill_e4m3_uniform(A, seed=5, scale=112.0)
        KI.fill_e4m3_uniform(B, seed=6, scale=112.0)
        C = torch.empty((n, n), dtype=torch.float32, device=dev)
        fn = lambda: KI.fp8_gemm(A, B, C)
        alg = 2 * n ** 3
    for _ in range(2):
        fn()
    torch.cuda.synchronize()
    ts = []
    for _ in range(args.profile_launches):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        ts.append((a, b))
    torch.cuda.synchronize()
    KI.context(0).check()
    ms = statistics.median(a.elapsed_time(b) for a, b in ts)
    unit = "TFLOP/s" if k == "gemm" else "GB/s"
    val = alg / (ms * 1e-3) / (1e12 if k == "gemm" else 1e9)
    print(json.dumps({"profile": k, "n": n, "ms_median": round(ms, 5), "value": round(val, 2), "unit": unit}))
    return 0


# ---------------------------------------------------------------------------------------------
# process group / timing helpers
# ---------------------------------------------------------------------------------------------
class Dist:
    def __init__(self, gpus: int):
        import torch

        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        if self.world != gpus and not (self.world == 1 and gpus == 1):
            raise SystemExit(f"--gpus {gpus} but WORLD_SIZE={self.world}")
        self.dev = self.local
        self.pg = None

    def init(self):
        import datetime

        import torch
        import torch.distributed as dist

        torch.cuda.set_device(self.dev)
        if self.world > 1:
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                    device_id=torch.device("cuda", self.dev))
            self.pg = True

    def barrier(self):
        import torch
        import torch.distributed as dist

        if self.world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max(self, v: float) -> float:
        import torch
        import torch.distributed as dist

        if self.world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def close(self):
        import torch.distributed as dist

        if self.world > 1 and dist.is_initialized():
            dist.destroy_process_group()


class Clocks:
    """nvidia-smi sampler for the timed region (start before, stop after)."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, dev: int):
        self.dev = dev
        self.proc = None
        self.windows = []

    def start(self):
        self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.dev}", f"--query-gpu=timestamp,{self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=self.file, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def mark(self, t0: float, t1: float):
        self.windows.append((t0, t1))

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.file.flush()
        rows = []
        for line in Path(self.file.name).read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 10:
                continue
            try:
                ts = time.mktime(time.strptime(parts[0].split(".")[0], "%Y/%m/%d %H:%M:%S"))
                ts += float("0." + parts[0].split(".")[1]) if "." in parts[0] else 0.0
                rows.append((ts, float(parts[2]), float(parts[3]), parts[6:10]))
            except (ValueError, IndexError):
                continue
        os.unlink(self.file.name)
        inside = [r for r in rows if any(a - 0.15 <= r[0] <= b + 0.15 for a, b in self.windows)]
        use = inside or rows
        if not use:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in use for i, v in enumerate(r[3]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(r[1] for r in use), "sm_max_mhz": max(r[2] for r in use),
                "reasons": reasons, "samples": len(use), "samples_in_timed_region": len(inside)}


def peaks():
    f = REPO / "MEASURED_PEAKS.json"
    if f.exists():
        d = json.loads(f.read_text())
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), "measured"
    return FALLBACK_HBM_GBS, FALLBACK_BF16_TFLOPS, 1400.0, "fallback"


def roofline(bound, achieved, peak, unit, traffic, source):
    return {"bound": bound, "achieved": round(achieved, 2), "peak": peak, "unit": unit,
            "frac": round(achieved / peak, 4), "traffic": traffic, "peak_source": source}


# ---------------------------------------------------------------------------------------------
# headline: byte copy over the 256 (src_offset, dst_offset) pairs
# ---------------------------------------------------------------------------------------------
PAIRS = [(so, do) for do in range(16) for so in range(16)]


def bench_copy(KI, D, steps, warmup, clocks):
    import torch

    dev = torch.device("cuda", D.dev)
    src = torch.empty(COPY_BYTES + 16, dtype=torch.uint8, device=dev)
    dst = torch.empty(COPY_BYTES + 16, dtype=torch.uint8, device=dev)
    KI.fill_bytes(src, seed=2 + D.rank)
    stream = torch.cuda.current_stream(dev)

    def step(ev=None):
        for k, (so, do) in enumerate(PAIRS):
            if ev is not None:
                ev[k][0].record(stream)
            KI.vcopy(dst, src, COPY_BYTES, dst_offset=do, src_offset=so)
            if ev is not None:
                ev[k][1].record(stream)

    for _ in range(warmup):
        step()
    # correctness spot check outside the timed region
    KI.vcopy(dst, src, COPY_BYTES - 5, dst_offset=7, src_offset=3)
    assert torch.equal(dst[7:7 + COPY_BYTES - 5], src[3:3 + COPY_BYTES - 5])
    evs = [[[torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)] for _ in PAIRS]
           for _ in range(steps)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    D.barrier()
    t0 = time.time()
    start.record(stream)
    for s in range(steps):
        step(evs[s])
    end.record(stream)
    torch.cuda.synchronize()
    clocks.mark(t0, time.time())
    ms = D.max(start.elapsed_time(end))
    kern_ms = [e[0].elapsed_time(e[1]) for st in evs for e in st]
    launches = steps * len(PAIRS)
    bytes_total = 2 * COPY_BYTES * launches * D.world
    out = {"ms_total": ms, "ms_per_step": ms / steps, "value_gbs": bytes_total / (ms * 1e-3) / 1e9,
           "kernel_ms_avg": statistics.mean(kern_ms), "kernel_ms_median": statistics.median(kern_ms),
           "launches": launches, "bytes_per_launch": 2 * COPY_BYTES}
    del src, dst
    torch.cuda.empty_cache()
    return out


def bench_copy_e2e(KI, D, steps):
    """Host buffers in pinned memory; every step is one ki_vcopy_host call: the source crosses to the
    device, the copy kernel runs there and the result comes back, chunked so both directions overlap."""
    import torch

    dev = torch.device("cuda", D.dev)
    n = COPY_BYTES
    src_h = torch.empty(n + 16, dtype=torch.uint8, pin_memory=True)
    dst_h = torch.empty(n + 16, dtype=torch.uint8, pin_memory=True)
    tmp = torch.empty(n + 16, dtype=torch.uint8, device=dev)
    KI.fill_bytes(tmp, seed=2 + D.rank)
    src_h.copy_(tmp)
    del tmp
    stream = torch.cuda.current_stream(dev)

    def step(k):
        so, do = PAIRS[(k * 37) % len(PAIRS)]
        KI.vcopy_host(dst_h, src_h, n, dst_offset=do, src_offset=so, device=D.dev, stream=stream)

    for k in range(2):
        step(k)
    torch.cuda.synchronize()
    D.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for k in range(steps):
        step(k)
    b.record(stream)
    torch.cuda.synchronize()
    ms = D.max(a.elapsed_time(b))
    so, do = PAIRS[((steps - 1) * 37) % len(PAIRS)]
    assert torch.equal(dst_h[do:do + n], src_h[so:so + n])
    val = 2 * n * steps * D.world / (ms * 1e-3) / 1e9
    del src_h, dst_h
    torch.cuda.empty_cache()
    return {"value": round(val, 2), "unit": "GB/s", "h2d_bytes_per_step": n, "d2h_bytes_per_step": n,
            "steps": steps, "ms_per_step": ms / steps,
            "path": "ki_vcopy_host: pinned host buffers, 16 MiB chunks over 3 streams (H2D, kernel, D2H overlapped)"}


# ---------------------------------------------------------------------------------------------
# the other primitives
# ---------------------------------------------------------------------------------------------
def _timed_steps(D, stream, step, steps, warmup, between=None):
    """Per-step device times (events around each step only) -> max over ranks of the mean."""
    import torch

    for _ in range(warmup):
        if between:
            between()
        step()
    D.barrier()
    ts = []
    for _ in range(steps):
        if between:
            between()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        step()
        b.record(stream)
        ts.append((a, b))
    torch.cuda.synchronize()
    ms = [a.elapsed_time(b) for a, b in ts]
    return D.max(statistics.mean(ms)), D.max(statistics.median(ms))


def bench_reduce(KI, D, steps, warmup, hbm):
    import torch

    from kernelintrinsics import sharded

    dev = torch.device("cuda", D.dev)
    lo, hi = sharded.shard_range(REDUCE_N, D.world, D.rank)
    # 8 rotating inputs (8 x 64 MiB at N=1, more than L2): each step reads data that is not in L2.
    nbuf = max(8, (1 << 29) // max(4 * (hi - lo), 1))
    xs = [torch.empty(hi - lo, dtype=torch.float32, device=dev) for _ in range(nbuf)]
    for k, x in enumerate(xs):
        KI.fill_uniform(x, seed=1 + k)  # shard-local streams; the parity tests check the global one
    stream = torch.cuda.current_stream(dev)
    out = torch.empty((), dtype=torch.float64, device=dev)
    it = [0]

    def step():
        x = xs[it[0] % nbuf]
        it[0] += 1
        if D.world == 1:
            KI.warpfold_reduce(x, out_f64=out)
        else:
            sharded.reduce_sharded(x)

    if D.world == 1:
        # A ~12 us kernel is shorter than one host launch through Python: replay the steps from a
        # CUDA graph so the device time is measured, not the launch path.
        for _ in range(warmup):
            step()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        cs = torch.cuda.Stream(dev)
        with torch.cuda.stream(cs):
            with torch.cuda.graph(g, stream=cs):
                for _ in range(steps):
                    step()
        g.replay()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        g.replay()
        b.record(stream)
        torch.cuda.synchronize()
        mean_ms = med_ms = a.elapsed_time(b) / steps
        how = f"one CUDA graph of {steps} back-to-back launches"
        del g
    else:
        mean_ms, med_ms = _timed_steps(D, stream, step, steps, warmup)
        how = "per-step events (reduce + NCCL all-gather)"
    gbs = 4 * REDUCE_N / (mean_ms * 1e-3) / 1e9
    per_gpu = gbs / D.world
    del xs
    torch.cuda.empty_cache()
    return {"workload": f"Float32 sum n=2^24 ({D.world} shard(s))", "value": round(gbs, 2), "unit": "GB/s",
            "ms_per_step": round(mean_ms, 5), "ms_median": round(med_ms, 5),
            "frac_of_hbm_per_gpu": round(per_gpu / hbm, 4), "timing": how,
            "l2": f"{nbuf} rotating inputs ({nbuf * 4 * (hi - lo) >> 20} MiB > L2): no step reads cached data",
            "algorithmic_bytes": 4 * REDUCE_N}


def bench_scan(KI, D, steps, warmup, hbm):
    import torch

    from kernelintrinsics import sharded

    dev = torch.device("cuda", D.dev)
    lo, hi = sharded.shard_range(SCAN_N, D.world, D.rank)
    x = torch.empty(hi - lo, dtype=torch.int64, device=dev)
    KI.fill_int_range(x, seed=3 + D.rank, lo=-1000, hi=1000)
    y = torch.empty_like(x)
    stream = torch.cuda.current_stream(dev)
    if D.world == 1:
        step = lambda: KI.warpreduce_scan(x, out=y)
    else:
        step = lambda: sharded.scan_sharded(x, y)
    mean_ms, med_ms = _timed_steps(D, stream, step, steps, warmup)
    KI.context(D.dev).check()
    gbs = 16 * SCAN_N / (mean_ms * 1e-3) / 1e9
    assert y[0].item() == x[0].item() or D.rank > 0
    del x, y
    torch.cuda.empty_cache()
    return {"workload": f"Int64 inclusive scan n=2^30 ({D.world} shard(s))", "value": round(gbs, 2),
            "unit": "GB/s", "elements_per_s": round(SCAN_N / (mean_ms * 1e-3), 1), "ms_per_step": round(mean_ms, 4),
            "frac_of_hbm_per_gpu": round(gbs / D.world / hbm, 4), "algorithmic_bytes": 16 * SCAN_N,
            "bytes_moved_per_elem": 16 if D.world == 1 else 24, "l2": "inputs larger than L2"}


def bench_scan_f32(KI, D, steps, warmup, hbm):
    """Float32 cumsum (ki_scan, Float64 accumulation) of 2^28 uniform[0,1) values per rank; the
    per-rank scans are independent (a replica per rank, weak scaling)."""
    import torch

    n = SCAN_F32_N
    dev = torch.device("cuda", D.dev)
    x = torch.empty(n, dtype=torch.float32, device=dev)
    KI.fill_uniform(x, seed=1 + D.rank)
    y = torch.empty_like(x)
    stream = torch.cuda.current_stream(dev)
    mean_ms, med_ms = _timed_steps(D, stream, lambda: KI.scan(x, "+", out=y), steps, warmup)
    KI.context(D.dev).check()
    gbs = 8 * n * D.world / (mean_ms * 1e-3) / 1e9
    del x, y
    torch.cuda.empty_cache()
    return {"workload": "Float32 inclusive scan (cumsum) n=2^28 per rank, Float64 accumulation", "value": round(gbs, 2),
            "unit": "GB/s", "ms_per_step": round(mean_ms, 4), "frac_of_hbm_per_gpu": round(gbs / D.world / hbm, 4),
            "algorithmic_bytes": 8 * n, "replicas": D.world, "l2": "inputs larger than L2"}


def bench_compact(KI, D, steps, warmup, hbm):
    import torch

    from kernelintrinsics import sharded

    dev = torch.device("cuda", D.dev)
    lo, hi = sharded.shard_range(COMPACT_N, D.world, D.rank)
    x = torch.empty(hi - lo, dtype=torch.float32, device=dev)
    KI.fill_normal(x, seed=4 + D.rank)
    vals = torch.empty_like(x)
    idx = torch.empty(x.numel(), dtype=torch.int32, device=dev)
    cnt = torch.zeros((), dtype=torch.uint64, device=dev)
    stream = torch.cuda.current_stream(dev)
    if D.world == 1:
        step = lambda: KI.vote_compact(x, 0.5, out_vals=vals, out_idx=idx, count=cnt, trim=False)
        k_total = None
    else:
        ops = sharded.cuda_ops()
        ops.compact_gt = lambda xx, thr, base: KI.vote_compact(xx, thr, out_vals=vals, out_idx=idx, count=cnt,
                                                               index_base=base, trim=False)
        step = lambda: sharded.compact_sharded(x, 0.5, lo, ops=ops)
    mean_ms, med_ms = _timed_steps(D, stream, step, steps, warmup)
    KI.context(D.dev).check()
    k = int(cnt.item())
    if D.world > 1:
        import torch.distributed as dist

        t = torch.tensor([k], dtype=torch.int64, device=dev)
        dist.all_reduce(t)
        k = int(t.item())
    alg = 4 * COMPACT_N + 8 * k
    gbs = alg / (mean_ms * 1e-3) / 1e9
    del x, vals, idx
    torch.cuda.empty_cache()
    return {"workload": f"filter/findall x>0.5, n=2^28 N(0,1) ({D.world} shard(s))", "value": round(gbs, 2),
            "unit": "GB/s", "kept": k, "kept_frac": round(k / COMPACT_N, 5), "ms_per_step": round(mean_ms, 4),
            "frac_of_hbm_per_gpu": round(gbs / D.world / hbm, 4), "algorithmic_bytes": alg,
            "l2": "inputs larger than L2"}


def bench_gemm(KI, D, steps, warmup, bf16):
    import torch

    dev = torch.device("cuda", D.dev)
    M = N = K = GEMM_MNK
    A = torch.empty((M, K), dtype=torch.uint8, device=dev)
    B = torch.empty((K, N), dtype=torch.uint8, device=dev)
    KI.fill_e4m3_uniform(A, seed=5, scale=112.0)
    KI.fill_e4m3_uniform(B, seed=6, scale=112.0)
    C = torch.empty((M, N), dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)
    try:
        KI.fp8_gemm(A, B, C)
        torch.cuda.synchronize()
    except KI.KIError as e:
        return {"workload": "fp8 e4m3 GEMM 8192^3", "unavailable": str(e)}
    mean_ms, med_ms = _timed_steps(D, stream, lambda: KI.fp8_gemm(A, B, C), steps, warmup)
    tflops = 2 * M * N * K / (mean_ms * 1e-3) / 1e12
    # measured fp8 reference point on this GPU: torch._scaled_mm (cuBLASLt) on the same shape
    ref = None
    try:
        a8 = A.view(torch.float8_e4m3fn)
        b8 = B.view(torch.float8_e4m3fn).t().contiguous().t()
        one = torch.ones((), dtype=torch.float32, device=dev)
        f = lambda: torch._scaled_mm(a8, b8, scale_a=one, scale_b=one, out_dtype=torch.float32)
        r_ms, _ = _timed_steps(D, stream, f, steps, warmup)
        ref = 2 * M * N * K / (r_ms * 1e-3) / 1e12
    except Exception:  # noqa: BLE001 - the reference point is optional
        ref = None
    del A, B, C
    torch.cuda.empty_cache()
    fp8_peak = 2 * bf16
    return {"workload": "fp8 e4m3 GEMM M=N=K=8192, Float32 out", "value": round(tflops, 2), "unit": "TFLOP/s",
            "ms_per_step": round(mean_ms, 4), "frac_of_2x_bf16_measured": round(tflops / fp8_peak, 4),
            "frac_of_nominal_4500": round(tflops / 4500.0, 4),
            "cublaslt_fp8_same_shape_tflops": None if ref is None else round(ref, 1),
            "replicas": D.world}


# ---------------------------------------------------------------------------------------------
# CPU baseline and the reference arm
# ---------------------------------------------------------------------------------------------
def cpu_copy_baseline(seconds: float):
    """The oracle's multithreaded byte copy (restatement of copyto!) on this host's cores."""
    import numpy as np

    sys.path.insert(0, str(REPO / "oracle"))
    import ki_oracle

    ki_oracle.build()
    th = os.cpu_count() or 1
    src = ki_oracle.gen_bytes(2, COPY_BYTES + 16, th)
    dst = np.empty_like(src)
    reps, moved = 0, 0
    t0 = time.perf_counter()
    while True:
        so, do = PAIRS[(reps * 37) % len(PAIRS)]
        n = COPY_BYTES
        ki_oracle.lib().ko_copy_bytes(dst.ctypes.data + do, src.ctypes.data + so, n, th)
        reps += 1
        moved += 2 * n
        el = time.perf_counter() - t0
        if el >= seconds or reps >= 1000:
            break
    assert np.array_equal(dst[do:do + n], src[so:so + n])
    return {"value": round(moved / el / 1e9, 3), "unit": "GB/s", "cores": th, "kind": "port",
            "sample": f"{reps} copies of 2^28 bytes at cycling (src,dst) offsets, {el:.1f} s"}, reps, el


def run_reference(args, D):
    if D.rank != 0:
        return 0
    import numpy as np

    sys.path.insert(0, str(REPO / "oracle"))
    import ki_oracle

    ki_oracle.build()
    th = os.cpu_count() or 1
    src = ki_oracle.gen_bytes(2, COPY_BYTES + 16, th)
    dst = np.empty_like(src)
    lib = ki_oracle.lib()

    def step(k):
        so, do = PAIRS[(k * 37) % len(PAIRS)]
        lib.ko_copy_bytes(dst.ctypes.data + do, src.ctypes.data + so, COPY_BYTES, th)

    for k in range(args.warmup):
        step(k)
    t0 = time.perf_counter()
    for k in range(args.steps):
        step(k)
    el = time.perf_counter() - t0
    val = 2 * COPY_BYTES * args.steps / el / 1e9
    line = {"metric": "vectorised byte copy bandwidth (copyto!, 2^28 B, all 256 src/dst misalignments)",
            "value": round(val, 3), "unit": "GB/s", "impl": "reference", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(el / args.steps * 1e3, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "u8", "data": "synthetic (splitmix64 bytes, seed 2)",
            "config": {"workload": "copyto! of 2^28 bytes at (src_offset, dst_offset) in 0..15 x 0..15",
                       "bytes_per_copy": COPY_BYTES, "sample_per_step": "one 2^28-byte copy (cycling pairs)"},
            "cpu_baseline": {"value": round(val, 3), "unit": "GB/s", "cores": th, "kind": "port",
                             "sample": f"{args.steps} copies of 2^28 bytes, C oracle memcpy on {th} threads"},
            "e2e": {"value": round(val, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------------------------
def main():
    args = parse()
    if args.profile:
        return run_profile(args)
    D = Dist(args.gpus)
    if args.impl == "reference":
        return run_reference(args, D)
    import torch

    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    D.init()
    import kernelintrinsics as KI

    KI.context(D.dev)
    hbm, bf16, bf16_sus, src = peaks()
    clocks = Clocks(D.dev)
    clocks.start()
    try:
        head = bench_copy(KI, D, args.steps, args.warmup, clocks)
        kernels = {}
        if not args.no_extra:
            only = set(filter(None, args.only.split(",")))
            plan = [("reduce", lambda: bench_reduce(KI, D, 50, 5, hbm)),
                    ("scan", lambda: bench_scan(KI, D, 10, 3, hbm)),
                    ("scan_f32", lambda: bench_scan_f32(KI, D, 10, 3, hbm)),
                    ("compact", lambda: bench_compact(KI, D, 20, 3, hbm)),
                    ("gemm", lambda: bench_gemm(KI, D, 20, 3, bf16))]
            for name, fn in plan:
                if only and name not in only:
                    continue
                t0 = time.time()
                kernels[name] = fn()
                clocks.mark(t0, time.time())
        e2e = bench_copy_e2e(KI, D, 6)
    finally:
        clk = clocks.stop()
    cpu = None
    if D.world == 1 and D.rank == 0 and not args.no_cpu_baseline:
        cpu, _, _ = cpu_copy_baseline(args.cpu_seconds)
    achieved = head["bytes_per_launch"] / (head["kernel_ms_avg"] * 1e-3) / 1e9
    line = {
        "metric": "vectorised byte copy bandwidth (copyto!, 2^28 B, all 256 src/dst misalignments)",
        "value": round(head["value_gbs"], 2), "unit": "GB/s", "n_gpus": D.world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(head["ms_per_step"], 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "u8", "data": "synthetic (splitmix64 bytes, seed 2+rank)",
        "config": {"workload": "copyto! of 2^28 bytes, one step = 256 copies at (src_offset, dst_offset) in 0..15^2",
                   "bytes_per_copy": COPY_BYTES, "copies_per_step": len(PAIRS), "parallelism": f"dp{D.world}",
                   "l2": "inputs larger than L2 (256 MiB source + 256 MiB destination)"},
        "roofline": roofline("hbm", achieved, hbm, "GB/s", NCU_TRAFFIC_PER_LAUNCH["vcopy_kernel"], src),
        "kernel_ms_avg": round(head["kernel_ms_avg"], 5),
        "e2e": e2e,
        "gpu_launches": head["launches"],
        "clocks": clk,
        "kernels": kernels,
    }
    if cpu is not None:
        line["cpu_baseline"] = cpu
    if D.rank == 0:
        print(json.dumps(line), flush=True)
    D.close()
    return 0


if __name__ == "__main__":
    sys.exit(main())
