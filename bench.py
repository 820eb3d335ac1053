#!/usr/bin/env python
"""Benchmark of the KernelIntrinsics B200 primitives (one JSON line on rank 0).

Headline workload: the Int64 inclusive prefix sum (Base.cumsum) of n = 2^30 elements drawn from
U{-1000..1000}, split into contiguous shards over the N GPUs (strong scaling: the total is fixed).
Each rank scans its shard through the libki_b200 communicator (ki_scan_inclusive_i64_sharded):
phase 1 sums the shard, one 8-byte total per rank crosses NVLink (pushed into every peer's exchange
buffer by the exchange kernel), phase 2 scans the shard seeded on the device.  The shards follow
ki_comm_scan_shard_range (the last rank, which skips phase 1, holds 3/2 of a share so every rank
moves the same bytes).  One step is one sharded scan of the whole array.

The same line carries, under "kernels", the other device-wide primitives on their own workloads:
  copy     copyto! of 2^28 bytes, one step = 256 copies at every (src, dst) offset pair (weak
           scaling: each rank copies its own buffers)
  reduce   Float32 sum, n = 2^24 in total, sharded (8 rotating inputs, more than L2)
  scan_f32 Float32 cumsum (generic scan, Float64 accumulation), n = 2^28 per rank (replicas)
  compact  filter/findall of x > 0.5 over 2^28 N(0,1) Float32 in total, sharded
  gemm     fp8 e4m3 GEMM 8192^3 with Float32 output (replicas at N > 1)
Outside every timed region each rank checks its results ("parity"): the scan against the oracle's
cumsum on windows of the global input plus the difference property over the whole shard and the
shard boundaries, the compaction against the oracle's filter/findall on the whole shard, the sum
against the oracle's Float64 sum.  A mismatch makes the run exit non-zero.

--impl reference times the reference semantics' CPU implementation (the C oracle's multithreaded
cumsum, all host threads) on the headline workload, rank 0 only.

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
GOLDEN = 0x9E3779B97F4A7C15  # splitmix64 increment: element i of stream s is mix64(s + (i+1)*GOLDEN)

FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0

# Per-launch DRAM traffic (dram__bytes_read.sum + dram__bytes_write.sum) of the headline kernel,
# scan_i64_kernel: 1,040,247,808 B captured by ncu at n = 2^26 (profiles/scan_i64_kernel_2e26.md),
# scaled by the elements a launch processes (the traffic grows in proportion: one read of the input,
# one write of the output, ~8 B of tile status per 15872 elements).
NCU_TRAFFIC_PER_ELEM = {"scan_i64_kernel": 1_040_247_808 / (1 << 26), "vcopy_kernel": 486_999_808 / (1 << 28)}

SCAN_WORKLOAD = ("Int64 inclusive prefix sum (cumsum) of n=2^30 U{-1000..1000}, contiguous shards over the GPUs "
                 "(ki_comm_scan_shard_range), shard totals exchanged over NVLink")


def window_seed(seed: int, lo: int) -> int:
    """Seed of the stream whose element i is element lo + i of stream ``seed`` (a shard's window)."""
    return (seed + lo * GOLDEN) % (1 << 64)


def wrap64(v: int) -> int:
    v &= (1 << 64) - 1
    return v - (1 << 64) if v >= 1 << 63 else v


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--no-extra", action="store_true", help="headline scan only")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--cpu-seconds", type=float, default=10.0)
    p.add_argument("--only", default="", help="comma list of kernels to run under 'kernels'")
    p.add_argument("--profile", default="", choices=["", "copy", "reduce", "scan", "compact", "gemm", "scan_f32", "scan_u8", "rows", "copy2d",
                            "count", "scan_i8max", "scan_u8or"],
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
    elif k in ("scan_i8max", "scan_u8or"):
        n = n or (1 << 27)  # accumulate(max) over Int8 / accumulate(|) over UInt8, same type out
        x = torch.empty(n, dtype=torch.uint8, device=dev)
        KI.fill_bytes(x, seed=2)
        if k == "scan_i8max":
            x = x.view(torch.int8)
        y = torch.empty_like(x)
        op = "max" if k == "scan_i8max" else "|"
        fn = lambda: KI.scan(x, op, out=y)
        alg = 2 * n
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
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        if self.world != gpus and not (self.world == 1 and gpus == 1):
            raise SystemExit(f"--gpus {gpus} but WORLD_SIZE={self.world}")
        self.dev = self.local

    def init(self):
        import datetime

        import torch
        import torch.distributed as dist

        torch.cuda.set_device(self.dev)
        if self.world > 1:
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                    device_id=torch.device("cuda", self.dev))

    def barrier(self):
        import torch
        import torch.distributed as dist

        if self.world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def gather(self, v) -> list:
        """Every rank's Python number (int64 or float64), in rank order."""
        import torch
        import torch.distributed as dist

        if self.world == 1:
            return [v]
        dt = torch.float64 if isinstance(v, float) else torch.int64
        t = torch.tensor([v], dtype=dt, device="cuda")
        out = torch.empty(self.world, dtype=dt, device="cuda")
        dist.all_gather_into_tensor(out, t)
        return [x.item() for x in out.cpu()]

    def max(self, v: float) -> float:
        return max(self.gather(float(v)))

    def all_ok(self, ok: bool) -> bool:
        return min(self.gather(int(bool(ok)))) == 1

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


def oracle_mod():
    """The oracle (C restatement of the reference semantics): the checker and the CPU baseline only."""
    if str(REPO / "oracle") not in sys.path:
        sys.path.insert(0, str(REPO / "oracle"))
    import ki_oracle

    ki_oracle.build()
    return ki_oracle


def oracle_sum_i64_window(o, seed: int, a: int, b: int) -> int:
    """Wrapping Int64 sum of elements [a, b) of the U{-1000..1000} stream ``seed``, in chunks."""
    tot, chunk = 0, 1 << 26
    for c in range(a, b, chunk):
        m = min(chunk, b - c)
        tot = wrap64(tot + o.sum_i64(o.gen_int_range_i64(window_seed(seed, c), -1000, 1000, m)))
    return tot


# ---------------------------------------------------------------------------------------------
# headline: sharded Int64 scan of 2^30 elements
# ---------------------------------------------------------------------------------------------
def bench_scan(KI, D, comm, steps, warmup, clocks):
    import torch

    dev = torch.device("cuda", D.dev)
    lo, hi = comm.scan_shard_range(SCAN_N)
    n = hi - lo
    x = torch.empty(n, dtype=torch.int64, device=dev)
    KI.fill_int_range(x, seed=window_seed(3, lo), lo=-1000, hi=1000)  # this rank's window of the global input
    y = torch.empty_like(x)
    stream = torch.cuda.current_stream(dev)
    step = lambda: comm.scan(x, out=y)  # noqa: E731
    for _ in range(warmup):
        step()
    comm.check()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    D.barrier()
    t0 = time.time()
    start.record(stream)
    for a, b in evs:
        a.record(stream)
        step()
        b.record(stream)
    end.record(stream)
    torch.cuda.synchronize()
    clocks.mark(t0, time.time())
    comm.check()
    ms = D.max(start.elapsed_time(end))
    step_ms = [a.elapsed_time(b) for a, b in evs]
    if D.world == 1:
        # one step is one launch of scan_i64_kernel (plus the clear of its tile status words)
        kern_ms = statistics.mean(step_ms)
        how = "CUDA events around each of the timed steps (one scan_i64_kernel launch per step)"
    else:
        # the step also holds phase 1 and the exchange: time the phase-2 kernel alone on this shard
        ks = []
        for _ in range(max(steps, 5)):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            KI.warpreduce_scan(x, out=y)
            b.record(stream)
            ks.append((a, b))
        torch.cuda.synchronize()
        kern_ms = statistics.mean(a.elapsed_time(b) for a, b in ks)
        how = ("CUDA events around launches of scan_i64_kernel alone on each rank's shard after the timed steps; "
               "the rank with the lowest achieved bandwidth is reported")
        step()  # leave y holding the sharded result for the parity check
        torch.cuda.synchronize()
        comm.check()
    kernels_per_step = 1 if D.world == 1 else (2 if comm.rank == D.world - 1 else 3)
    launches = sum(D.gather(kernels_per_step * steps))
    # the roofline kernel: each rank's own elements over its own launch time; the lowest rank reported
    achieved = 16 * n / (kern_ms * 1e-3) / 1e9
    ach_all, ms_all, n_all = D.gather(float(achieved)), D.gather(float(kern_ms)), D.gather(int(n))
    worst = min(range(D.world), key=lambda r: ach_all[r])
    parity = parity_scan(D, x, y, lo, hi)
    out = {"ms_total": ms, "ms_per_step": ms / steps, "value_gbs": 16 * SCAN_N * steps / (ms * 1e-3) / 1e9,
           "kernel_ms_avg": ms_all[worst], "achieved_gbs": ach_all[worst], "kernel_rank": worst,
           "kernel_timing": how, "launches": launches, "n_local": n_all[worst], "lo": lo,
           "step_ms_median": D.max(statistics.median(step_ms)), "parity": parity}
    return out, x, y


def parity_scan(D, x, y, lo, hi) -> dict:
    """Checks of this rank's slice of cumsum(global input), outside the timed region:
    (a) y[i] - y[i-1] == x[i] over the whole shard, on the device (chunks);
    (b) y[0] - x[0] == the previous rank's last value (0 on rank 0): with (a) this fixes every value;
    (c) the first and last 2^16 values against the oracle's cumsum of the regenerated global input,
        seeded with the oracle's sum of everything before the window."""
    import numpy as np
    import torch

    o = oracle_mod()
    n = hi - lo
    ok_diff = True
    ch = 1 << 26
    for a in range(1, n, ch):
        b = min(n, a + ch)
        ok_diff = ok_diff and bool(torch.equal(y[a:b] - y[a - 1:b - 1], x[a:b]))
    first = wrap64(int(y[0].item()) - int(x[0].item()))
    lasts = D.gather(int(y[-1].item()))
    ok_edge = first == (0 if D.rank == 0 else lasts[D.rank - 1])
    w = min(1 << 16, n)
    prefix = oracle_sum_i64_window(o, 3, 0, lo)
    xw = o.gen_int_range_i64(window_seed(3, lo), -1000, 1000, w)
    ok_head = bool(np.array_equal(y[:w].cpu().numpy(), o.cumsum_i64(xw, seed=prefix)))
    p2 = wrap64(prefix + oracle_sum_i64_window(o, 3, lo, hi - w))
    xw2 = o.gen_int_range_i64(window_seed(3, hi - w), -1000, 1000, w)
    ok_tail = bool(np.array_equal(y[n - w:].cpu().numpy(), o.cumsum_i64(xw2, seed=p2)))
    ok = D.all_ok(ok_diff and ok_edge and ok_head and ok_tail)
    return {"result": "ok" if ok else "MISMATCH", "checks": "difference property over every shard, shard boundaries, "
            "first and last 2^16 values of every shard vs the oracle's cumsum (bit-exact)",
            "rank0": {"diff": ok_diff, "boundary": ok_edge, "head": ok_head, "tail": ok_tail}}


def bench_scan_e2e(KI, D, comm, x, y, steps):
    """The same sharded scan through the host-buffer entry point: every step each rank's shard goes from
    pinned host memory to the device and its scanned slice comes back (ki_scan_inclusive_i64_sharded_host;
    with one rank the chunked pipeline of ki_scan_inclusive_i64_host, both copy directions overlapped)."""
    import torch

    dev = torch.device("cuda", D.dev)
    n = x.numel()
    xh = torch.empty(n, dtype=torch.int64, pin_memory=True)
    yh = torch.empty(n, dtype=torch.int64, pin_memory=True)
    xh.copy_(x)
    stream = torch.cuda.current_stream(dev)
    D.barrier()  # the ranks pinned their buffers at different speeds: line them up before the first exchange
    comm.scan_host(xh, out=yh)
    torch.cuda.synchronize()
    comm.check()
    D.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(steps):
        comm.scan_host(xh, out=yh)
    b.record(stream)
    torch.cuda.synchronize()
    comm.check()
    ms = D.max(a.elapsed_time(b))
    ok = True
    ch = 1 << 26
    for s0 in range(0, n, ch):
        s1 = min(n, s0 + ch)
        ok = ok and bool(torch.equal(yh[s0:s1], y[s0:s1].cpu()))
    ok = D.all_ok(ok)
    val = 16 * SCAN_N * steps / (ms * 1e-3) / 1e9
    path = ("ki_scan_inclusive_i64_host: 16 MiB chunks over 3 streams (H2D, scan, D2H overlapped)" if D.world == 1 else
            "ki_scan_inclusive_i64_sharded_host: shard to the device in 16 MiB chunks (each summed as it lands), "
            "totals exchanged, chunks scanned in place and sent back as they finish")
    del xh, yh
    return {"value": round(val, 2), "unit": "GB/s", "h2d_bytes_per_step": 8 * SCAN_N, "d2h_bytes_per_step": 8 * SCAN_N,
            "steps": steps, "ms_per_step": round(ms / steps, 3), "path": path,
            "parity": "ok (equal to the device-resident result)" if ok else "MISMATCH"}


# ---------------------------------------------------------------------------------------------
# the other primitives
# ---------------------------------------------------------------------------------------------
PAIRS = [(so, do) for do in range(16) for so in range(16)]


def _timed_steps(D, stream, step, steps, warmup, between=None):
    """Per-step device times (events around each step only) -> max over ranks of the mean and median."""
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


def bench_copy(KI, D, steps, warmup, hbm, src_kind):
    """copyto! of 2^28 bytes: one step = 256 copies, one per (src_offset, dst_offset) in 0..15^2."""
    import torch

    dev = torch.device("cuda", D.dev)
    src = torch.empty(COPY_BYTES + 16, dtype=torch.uint8, device=dev)
    dst = torch.empty(COPY_BYTES + 16, dtype=torch.uint8, device=dev)
    KI.fill_bytes(src, seed=2 + D.rank)
    stream = torch.cuda.current_stream(dev)

    def step():
        for so, do in PAIRS:
            KI.vcopy(dst, src, COPY_BYTES, dst_offset=do, src_offset=so)

    for _ in range(warmup):
        step()
    KI.vcopy(dst, src, COPY_BYTES - 5, dst_offset=7, src_offset=3)
    ok = D.all_ok(bool(torch.equal(dst[7:7 + COPY_BYTES - 5], src[3:3 + COPY_BYTES - 5])))
    # events around whole steps only: an event between two launches would keep the second from
    # overlapping the first's tail (programmatic dependent launch), so a launch's duration is the
    # step's time over its 256 launches
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    D.barrier()
    start.record(stream)
    for _ in range(steps):
        step()
    end.record(stream)
    torch.cuda.synchronize()
    ms = D.max(start.elapsed_time(end))
    kern = ms / (steps * len(PAIRS))
    bytes_total = 2 * COPY_BYTES * steps * len(PAIRS) * D.world
    del src, dst
    torch.cuda.empty_cache()
    achieved = 2 * COPY_BYTES / (kern * 1e-3) / 1e9
    return {"workload": "copyto! of 2^28 bytes, one step = 256 copies at (src_offset, dst_offset) in 0..15^2, "
                        "each rank its own buffers (weak scaling)",
            "value": round(bytes_total / (ms * 1e-3) / 1e9, 2), "unit": "GB/s", "ms_per_step": round(ms / steps, 4),
            "kernel_ms_avg": round(kern, 5), "frac_of_hbm_per_gpu": round(achieved / hbm, 4),
            "kernel_timing": "CUDA events around each step of 256 back-to-back launches; per launch = step / 256",
            "roofline": roofline("hbm", achieved, hbm, "GB/s", int(NCU_TRAFFIC_PER_ELEM["vcopy_kernel"] * COPY_BYTES),
                                 src_kind),
            "launches": steps * len(PAIRS) * D.world, "parity": "ok" if ok else "MISMATCH",
            "l2": "inputs larger than L2 (256 MiB source + 256 MiB destination)"}


def bench_reduce(KI, D, comm, steps, warmup, hbm):
    """Float32 sum of 2^24 elements in total, sharded; steps replayed from one CUDA graph (a ~12 us
    operation is shorter than a launch through Python).  The graph starts right after one sharded
    reduce, whose exchange lines the ranks up, so the timed replays start together."""
    import numpy as np
    import torch

    dev = torch.device("cuda", D.dev)
    lo, hi = comm.shard_range(REDUCE_N)
    n = hi - lo
    nbuf = max(8, (1 << 29) // max(4 * n, 1))  # more bytes than L2 in the rotation
    xs = [torch.empty(n, dtype=torch.float32, device=dev) for _ in range(nbuf)]
    for k, x in enumerate(xs):
        KI.fill_uniform(x, seed=window_seed(11 + k, lo))
    stream = torch.cuda.current_stream(dev)
    out = torch.empty((), dtype=torch.float64, device=dev)
    it = [0]

    def step():
        comm.reduce_sum(xs[it[0] % nbuf], out_f64=out)
        it[0] += 1

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    cs = torch.cuda.Stream(dev)
    with torch.cuda.stream(cs):
        with torch.cuda.graph(g, stream=cs):
            for _ in range(steps):
                step()
    D.barrier()
    step()
    g.replay()
    torch.cuda.synchronize()
    D.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    step()  # lines the ranks up on the device
    a.record(stream)
    g.replay()
    b.record(stream)
    torch.cuda.synchronize()
    comm.check()
    ms = D.max(a.elapsed_time(b) / steps)
    del g
    # parity: the global 2^24 input of stream 1 (each rank its window) against the oracle's Float64 sum
    x = xs[0]
    KI.fill_uniform(x, seed=window_seed(1, lo))
    tot = comm.reduce_sum(x).item()
    comm.check()
    o = oracle_mod()
    ref = o.sum_f32(o.gen_uniform_f32(1, REDUCE_N))
    same = len(set(D.gather(float(tot)))) == 1
    ok = D.all_ok(same and abs(tot - ref) <= 1e-5 * math.log2(REDUCE_N) * abs(ref))
    gbs = 4 * REDUCE_N / (ms * 1e-3) / 1e9
    res = {"workload": f"Float32 sum n=2^24 in total, {D.world} shard(s), partials exchanged over NVLink",
           "value": round(gbs, 2), "unit": "GB/s", "ms_per_step": round(ms, 5),
           "frac_of_hbm_per_gpu": round(gbs / D.world / hbm, 4),
           "timing": f"one CUDA graph of {steps} back-to-back sharded reduces"
                     + (" (reduce + exchange kernel)" if D.world > 1 else " (one reduce_kernel launch each)"),
           "l2": f"{nbuf} rotating inputs ({nbuf * 4 * n >> 20} MiB per rank > L2): no step reads cached data",
           "algorithmic_bytes": 4 * REDUCE_N, "launches": steps * (2 if D.world > 1 else 1) * D.world,
           "parity": {"result": "ok" if ok else "MISMATCH", "rel_err": abs(tot - ref) / abs(ref),
                      "tolerance": 1e-5 * math.log2(REDUCE_N), "same_bits_on_every_rank": same}}
    del xs
    torch.cuda.empty_cache()
    return res


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
    # property check: differences of the Float64-accumulated prefix are the inputs to Float32 rounding
    d = (y[1:].double() - y[:-1].double() - x[1:].double()).abs().max().item()
    ok = D.all_ok(d <= 2.0 ** -24 * 2 * float(y[-1].item()) and abs(y[0].item() - x[0].item()) == 0)
    gbs = 8 * n * D.world / (mean_ms * 1e-3) / 1e9
    del x, y
    torch.cuda.empty_cache()
    return {"workload": "Float32 inclusive scan (cumsum) n=2^28 per rank, Float64 accumulation", "value": round(gbs, 2),
            "unit": "GB/s", "ms_per_step": round(mean_ms, 4), "frac_of_hbm_per_gpu": round(gbs / D.world / hbm, 4),
            "algorithmic_bytes": 8 * n, "replicas": D.world, "l2": "inputs larger than L2",
            "parity": "ok" if ok else "MISMATCH"}


def bench_compact(KI, D, comm, steps, warmup, hbm):
    """filter/findall of x > 0.5 over 2^28 N(0,1) Float32 in total, sharded: each rank compacts its
    window of the global input with global 1-based indices; counts exchanged over NVLink."""
    import numpy as np
    import torch

    dev = torch.device("cuda", D.dev)
    lo, hi = comm.shard_range(COMPACT_N)
    x = torch.empty(hi - lo, dtype=torch.float32, device=dev)
    KI.fill_normal(x, seed=window_seed(4, lo))  # lo is even: the Box-Muller pairs line up with the global stream
    vals = torch.empty_like(x)
    idx = torch.empty(x.numel(), dtype=torch.int32, device=dev)
    cnt = torch.zeros((), dtype=torch.uint64, device=dev)
    off = torch.zeros((), dtype=torch.uint64, device=dev)
    tot = torch.zeros((), dtype=torch.uint64, device=dev)
    stream = torch.cuda.current_stream(dev)
    step = lambda: comm.compact_gt(x, 0.5, 1 + lo, vals, idx, cnt, off, tot)  # noqa: E731
    mean_ms, med_ms = _timed_steps(D, stream, step, steps, warmup)
    comm.check()
    k = int(cnt.item())
    counts = D.gather(k)
    total = sum(counts)
    o = oracle_mod()
    xs = x.cpu().numpy()
    rv, ri = o.filter_gt_f32(xs, 0.5, index_base=1 + lo)
    ok = (k == rv.size and np.array_equal(vals[:k].cpu().numpy().view(np.uint32), rv.view(np.uint32))
          and np.array_equal(idx[:k].cpu().numpy(), ri) and int(off.item()) == sum(counts[:D.rank])
          and int(tot.item()) == total)
    ok = D.all_ok(ok)
    alg = 4 * COMPACT_N + 8 * total
    gbs = alg / (mean_ms * 1e-3) / 1e9
    res = {"workload": f"filter/findall x>0.5, n=2^28 N(0,1) in total, {D.world} shard(s), counts exchanged over NVLink",
           "value": round(gbs, 2), "unit": "GB/s", "kept": total, "kept_frac": round(total / COMPACT_N, 5),
           "ms_per_step": round(mean_ms, 4), "frac_of_hbm_per_gpu": round(gbs / D.world / hbm, 4),
           "algorithmic_bytes": alg, "l2": "inputs larger than L2",
           "parity": {"result": "ok" if ok else "MISMATCH",
                      "checks": "count, every kept value and 1-based global index of every shard vs the oracle's "
                                "filter/findall; offsets = exclusive prefix of the counts; totals"}}
    sample = xs[:1 << 26].copy()
    del x, vals, idx, xs
    torch.cuda.empty_cache()
    return res, sample


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
    ref = None
    try:  # measured fp8 reference point on this GPU: torch._scaled_mm (cuBLASLt) on the same shape
        a8 = A.view(torch.float8_e4m3fn)
        b8 = B.view(torch.float8_e4m3fn).t().contiguous().t()
        one = torch.ones((), dtype=torch.float32, device=dev)
        f = lambda: torch._scaled_mm(a8, b8, scale_a=one, scale_b=one, out_dtype=torch.float32)  # noqa: E731
        r_ms, _ = _timed_steps(D, stream, f, steps, warmup)
        ref = 2 * M * N * K / (r_ms * 1e-3) / 1e12
    except Exception:  # noqa: BLE001 - the reference point is optional
        ref = None
    # parity on sampled rows against the oracle's Float64 GEMM of the dequantised inputs
    o = oracle_mod()
    import numpy as np

    rows = [0, 1, 4095, 8191]
    Ah, Bh = A.cpu().numpy(), B.cpu().numpy()
    Ch = C.cpu().numpy()
    errs = []
    for r in rows:
        R = o.gemm_e4m3_rows(Ah, Bh, r, r + 1)
        errs.append(float(np.linalg.norm(Ch[r:r + 1].astype(np.float64) - R) / np.linalg.norm(R)))
    ok = D.all_ok(max(errs) <= 1e-3)
    del A, B, C
    torch.cuda.empty_cache()
    fp8_peak = 2 * bf16
    return {"workload": "fp8 e4m3 GEMM M=N=K=8192, Float32 out", "value": round(tflops, 2), "unit": "TFLOP/s",
            "ms_per_step": round(mean_ms, 4), "frac_of_2x_bf16_measured": round(tflops / fp8_peak, 4),
            "frac_of_nominal_4500": round(tflops / 4500.0, 4),
            "cublaslt_fp8_same_shape_tflops": None if ref is None else round(ref, 1),
            "replicas": D.world, "parity": {"result": "ok" if ok else "MISMATCH", "rows": rows,
                                            "max_rel_frobenius": max(errs), "tolerance": 1e-3}}


# ---------------------------------------------------------------------------------------------
# CPU baselines (the oracle on this host's cores, rank 0 at N = 1) and the reference arm
# ---------------------------------------------------------------------------------------------
def _loop(fn, seconds, max_reps=1000):
    reps = 0
    t0 = time.perf_counter()
    while True:
        fn(reps)
        reps += 1
        el = time.perf_counter() - t0
        if el >= seconds or reps >= max_reps:
            return reps, el


def cpu_scan_baseline(seconds):
    """The oracle's multithreaded cumsum (two passes over per-thread blocks) on a 2^28-element sample."""
    import numpy as np

    o = oracle_mod()
    th = os.cpu_count() or 1
    n = 1 << 28
    x = o.gen_int_range_i64(3, -1000, 1000, n, th)
    y = np.empty_like(x)
    reps, el = _loop(lambda k: o.lib().ko_cumsum_i64(x.ctypes.data, y.ctypes.data, n, 0, th), seconds)
    return {"value": round(16 * n * reps / el / 1e9, 3), "unit": "GB/s", "cores": th, "kind": "port",
            "sample": f"{reps} cumsums of 2^28 Int64 (16 B per element), {el:.1f} s"}


def cpu_sum_baseline(seconds):
    o = oracle_mod()
    th = os.cpu_count() or 1
    x = o.gen_uniform_f32(1, REDUCE_N, th)
    reps, el = _loop(lambda k: o.sum_f32(x, th), seconds, 100000)
    return {"value": round(4 * REDUCE_N * reps / el / 1e9, 3), "unit": "GB/s", "cores": th, "kind": "port",
            "sample": f"{reps} Float64-accumulated sums of 2^24 Float32, {el:.1f} s"}


def cpu_filter_baseline(sample, seconds):
    o = oracle_mod()
    th = os.cpu_count() or 1
    kept = [0]

    def f(k):
        kept[0] = o.filter_gt_f32(sample, 0.5, nthreads=th)[0].size

    reps, el = _loop(f, seconds)
    alg = 4 * sample.size + 8 * kept[0]
    return {"value": round(alg * reps / el / 1e9, 3), "unit": "GB/s", "cores": th, "kind": "port",
            "sample": f"{reps} filter/findall passes (count, prefix, write) over 2^26 N(0,1) Float32, {el:.1f} s"}


def cpu_copy_baseline(seconds):
    import numpy as np

    o = oracle_mod()
    th = os.cpu_count() or 1
    src = o.gen_bytes(2, COPY_BYTES + 16, th)
    dst = np.empty_like(src)

    def f(k):
        so, do = PAIRS[(k * 37) % len(PAIRS)]
        o.lib().ko_copy_bytes(dst.ctypes.data + do, src.ctypes.data + so, COPY_BYTES, th)

    reps, el = _loop(f, seconds)
    return {"value": round(2 * COPY_BYTES * reps / el / 1e9, 3), "unit": "GB/s", "cores": th, "kind": "port",
            "sample": f"{reps} copies of 2^28 bytes at cycling (src,dst) offsets, {el:.1f} s"}


def headline_config(world):
    return {"workload": SCAN_WORKLOAD, "n": SCAN_N, "elements_per_step": SCAN_N, "parallelism": f"shard{world}",
            "split": "ki_comm_scan_shard_range (ranks below the last: 2 shares; last rank: 3 shares)",
            "l2": "inputs larger than L2 (8 GiB in + 8 GiB out in total; >= 1 GiB per rank at N = 8)"}


METRIC = "Int64 inclusive scan (cumsum) throughput, algorithmic GB/s (16 B per element)"


def run_reference(args, D):
    """Base.cumsum semantics on the host cores: the oracle's multithreaded C cumsum of the whole 2^30-element
    input per step (rank 0 only; the other ranks exit)."""
    if D.rank != 0:
        return 0
    import numpy as np

    o = oracle_mod()
    th = os.cpu_count() or 1
    x = o.gen_int_range_i64(3, -1000, 1000, SCAN_N, th)
    y = np.empty_like(x)
    lib = o.lib()
    for _ in range(args.warmup):
        lib.ko_cumsum_i64(x.ctypes.data, y.ctypes.data, SCAN_N, 0, th)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        lib.ko_cumsum_i64(x.ctypes.data, y.ctypes.data, SCAN_N, 0, th)
    el = time.perf_counter() - t0
    val = 16 * SCAN_N * args.steps / el / 1e9
    line = {"metric": METRIC, "value": round(val, 3), "unit": "GB/s", "impl": "reference", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(el / args.steps * 1e3, 3),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "int64",
            "data": "synthetic (splitmix64 stream, seed 3, U{-1000..1000})", "config": headline_config(args.gpus),
            "cpu_baseline": {"value": round(val, 3), "unit": "GB/s", "cores": th, "kind": "port",
                             "sample": f"{args.steps} cumsums of the whole 2^30-element input, C oracle on {th} threads"},
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
    from kernelintrinsics import sharded

    KI.context(D.dev)
    comm = sharded.Comm.create([D.dev])[0] if D.world == 1 else sharded.Comm.from_process_group(device=D.dev)
    comm.set_wait_timeout(10.0)  # exchange waits absorb host-side skew between ranks (allocation, parity work)
    hbm, bf16, bf16_sus, src_kind = peaks()
    clocks = Clocks(D.dev)
    clocks.start()
    try:
        head, x, y = bench_scan(KI, D, comm, args.steps, args.warmup, clocks)
        e2e = bench_scan_e2e(KI, D, comm, x, y, 3)
        del x, y
        torch.cuda.empty_cache()
        kernels, sample = {}, None
        if not args.no_extra:
            only = set(filter(None, args.only.split(",")))
            plan = [("copy", lambda: bench_copy(KI, D, args.steps, args.warmup, hbm, src_kind)),
                    ("reduce", lambda: bench_reduce(KI, D, comm, 50, 5, hbm)),
                    ("scan_f32", lambda: bench_scan_f32(KI, D, 10, 3, hbm)),
                    ("compact", lambda: bench_compact(KI, D, comm, 20, 3, hbm)),
                    ("gemm", lambda: bench_gemm(KI, D, 20, 3, bf16))]
            for name, fn in plan:
                if only and name not in only:
                    continue
                t0 = time.time()
                r = fn()
                if name == "compact":
                    r, sample = r
                kernels[name] = r
                clocks.mark(t0, time.time())
    finally:
        clk = clocks.stop()
    cpu = None
    if D.world == 1 and D.rank == 0 and not args.no_cpu_baseline:
        cpu = cpu_scan_baseline(args.cpu_seconds)
        if "reduce" in kernels:
            kernels["reduce"]["cpu_baseline"] = cpu_sum_baseline(3.0)
        if "compact" in kernels and sample is not None:
            kernels["compact"]["cpu_baseline"] = cpu_filter_baseline(sample, 3.0)
        if "copy" in kernels:
            kernels["copy"]["cpu_baseline"] = cpu_copy_baseline(3.0)
    n_local = head["n_local"]
    achieved = head["achieved_gbs"]
    parity = {"scan": head["parity"], "e2e_scan": e2e.pop("parity")}
    for k, v in kernels.items():
        if isinstance(v, dict) and "parity" in v:
            parity[k] = v["parity"]
    bad = [k for k, v in parity.items() if "ok" not in (v if isinstance(v, str) else v.get("result", ""))]
    line = {
        "metric": METRIC,
        "value": round(head["value_gbs"], 2), "unit": "GB/s", "n_gpus": D.world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(head["ms_per_step"], 4), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "int64",
        "data": "synthetic (splitmix64 stream, seed 3, U{-1000..1000}; each rank generates its window of the global input)",
        "config": headline_config(D.world),
        "roofline": roofline("hbm", achieved, hbm, "GB/s", int(NCU_TRAFFIC_PER_ELEM["scan_i64_kernel"] * n_local),
                             src_kind),
        "kernel_ms_avg": round(head["kernel_ms_avg"], 5), "kernel_timing": head["kernel_timing"],
        "e2e": e2e,
        "gpu_launches": head["launches"],
        "clocks": clk,
        "parity": {"result": "ok" if not bad else "MISMATCH: " + ",".join(bad), **parity},
        "kernels": kernels,
    }
    line["roofline"]["kernel"] = "scan_i64_kernel"
    line["roofline"]["elements_per_launch"] = n_local
    if D.world > 1:
        line["roofline"]["rank"] = head["kernel_rank"]
    if cpu is not None:
        line["cpu_baseline"] = cpu
    if D.rank == 0:
        print(json.dumps(line), flush=True)
    comm.close()
    D.close()
    return 0 if not bad else 3


if __name__ == "__main__":
    sys.exit(main())
