"""GPU, 2+ devices: the C-ABI communicator's sharded reduce / scan / compaction against the oracle.

Each rank owns a contiguous shard; only one 8-byte value per rank and operation crosses NVLink.
Two ways to drive the GPUs are tested: one process driving all of them (ki_comm_create) and one
process per GPU (ki_comm_init_rank, with the peer exchange and with the NCCL fallback exchange).
A rank that leaves between steps makes the other ranks' next exchange time out (bounded device
wait, KI_ERR_TIMEOUT), after which they abort.  Skipped when fewer GPUs are visible.
NVLS is off in every child (NCCL_NVLS_ENABLE=0) and no multicast object is used.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

N_SCAN, N_CMP, N_SUM = (1 << 22) + 12345, (1 << 21) + 777, (1 << 22) + 3


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _need(world):
    import torch

    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")


def _inputs(KI, dev):
    """The whole inputs on one device (counter-based generators: every rank makes the same arrays)."""
    import torch

    xi = torch.empty(N_SCAN, dtype=torch.int64, device=dev)
    KI.fill_int_range(xi, seed=3, lo=-1000, hi=1000)
    xf = torch.empty(N_SUM, dtype=torch.float32, device=dev)
    KI.fill_uniform(xf, seed=1)
    xn = torch.empty(N_CMP, dtype=torch.float32, device=dev)
    KI.fill_normal(xn, seed=4)
    return xi, xf, xn


def _check(oracle, world, sums, scans, vals, idxs, counts, offs, totals, xn_host):
    xi = oracle.gen_int_range_i64(3, -1000, 1000, N_SCAN)
    ref_sum = oracle.sum_f32(oracle.gen_uniform_f32(1, N_SUM))
    assert len(set(sums)) == 1  # every rank holds the same bits
    assert abs(sums[0] - ref_sum) <= 1e-5 * np.log2(N_SUM) * ref_sum
    assert np.array_equal(np.concatenate(scans), oracle.cumsum_i64(xi))
    rv, ri = oracle.filter_gt_f32(xn_host, 0.5)
    assert np.array_equal(np.concatenate(vals), rv) and np.array_equal(np.concatenate(idxs), ri)
    assert offs == [int(sum(counts[:r])) for r in range(world)]
    assert all(t == rv.size for t in totals)


@pytest.mark.parametrize("world", [2, 4, 8])
def test_sharded_ops_single_process(world, KI, oracle):
    """One host thread drives `world` GPUs through ki_comm_create; two rounds (both buffer parities)."""
    import torch

    from kernelintrinsics import sharded

    _need(world)
    comms = sharded.Comm.create(list(range(world)))
    try:
        per = []
        for r, c in enumerate(comms):
            dev = torch.device("cuda", r)
            xi, xf, xn = _inputs(KI, dev)
            lo, hi = c.shard_range(N_SCAN)
            slo, shi = c.shard_range(N_SUM)
            clo, chi = c.shard_range(N_CMP)
            per.append((xi[lo:hi].contiguous(), xf[slo:shi].contiguous(), xn[clo:chi].contiguous(), clo))
            torch.cuda.synchronize(dev)
        for _ in range(2):
            # one host thread: each operation is issued on every rank before the next operation (a
            # rank's call may allocate scratch, which can wait for that GPU's pending exchange)
            sums, scans_d, comps = [], [], []
            for c, (xi, xf, xn, clo) in zip(comms, per):
                with torch.cuda.device(c.device):
                    sums.append(c.reduce_sum(xf))
            for c, (xi, xf, xn, clo) in zip(comms, per):
                with torch.cuda.device(c.device):
                    scans_d.append(c.scan(xi))
            for c, (xi, xf, xn, clo) in zip(comms, per):
                with torch.cuda.device(c.device):
                    comps.append(c.compact_gt(xn, 0.5, index_base=1 + clo))
            outs = list(zip(sums, scans_d, comps))
            for c in comms:
                c.check()
            sums = [o[0].item() for o in outs]
            scans = [o[1].cpu().numpy() for o in outs]
            counts = [int(o[2][2].item()) for o in outs]
            vals = [o[2][0][:k].cpu().numpy() for o, k in zip(outs, counts)]
            idxs = [o[2][1][:k].cpu().numpy() for o, k in zip(outs, counts)]
            offs = [int(o[2][3].item()) for o in outs]
            totals = [int(o[2][4].item()) for o in outs]
            xn_host = _inputs(KI, torch.device("cuda", 0))[2].cpu().numpy()
            _check(oracle, world, sums, scans, vals, idxs, counts, offs, totals, xn_host)
    finally:
        for c in comms:
            c.close()


@pytest.mark.parametrize("world", [2, 4])
def test_sharded_ops_with_empty_shards(world, KI, oracle):
    """n smaller than the number of ranks: the ranks past n hold empty shards and still take part in
    every exchange (zero partials, zero totals, zero counts); twice in a row."""
    import torch

    from kernelintrinsics import sharded

    _need(world)
    comms = sharded.Comm.create(list(range(world)))
    try:
        n = world - 1
        xi_h = np.arange(1, n + 1, dtype=np.int64) * 1000
        xf_h = np.full(n, 0.75, dtype=np.float32)
        for _ in range(2):
            parts = []
            for c in comms:
                lo, hi = c.shard_range(n)
                dev = torch.device("cuda", c.device)
                parts.append((torch.from_numpy(xi_h[lo:hi]).to(dev), torch.from_numpy(xf_h[lo:hi]).to(dev), lo))
            sums = [c.reduce_sum(p[1]) for c, p in zip(comms, parts)]
            scans = [c.scan(p[0]) for c, p in zip(comms, parts)]
            comps = [c.compact_gt(p[1], 0.5, index_base=1 + p[2]) for c, p in zip(comms, parts)]
            for c in comms:
                c.check()
            assert all(s.item() == 0.75 * n for s in sums)
            got = np.concatenate([s.cpu().numpy() for s in scans])
            assert np.array_equal(got, np.cumsum(xi_h))
            idx = np.concatenate([cp[1][:int(cp[2].item())].cpu().numpy() for cp in comps])
            assert np.array_equal(idx, np.arange(1, n + 1, dtype=np.int32))
            assert all(int(cp[4].item()) == n for cp in comps)
    finally:
        for c in comms:
            c.close()


def _worker(rank, world, port, exchange, results):
    import datetime
    import sys
    from pathlib import Path

    repo = Path(__file__).resolve().parent.parent
    sys.path.insert(0, str(repo / "kernelintrinsics.jl_b200"))
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import torch
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    comm = None
    try:
        import kernelintrinsics as KI
        from kernelintrinsics import sharded

        comm = sharded.Comm.from_process_group(device=rank, exchange=exchange)
        dev = torch.device("cuda", rank)
        xi, xf, xn = _inputs(KI, dev)
        lo, hi = comm.shard_range(N_SCAN)
        slo, shi = comm.shard_range(N_SUM)
        clo, chi = comm.shard_range(N_CMP)
        res = []
        for _ in range(2):
            tot = comm.reduce_sum(xf[slo:shi].contiguous())
            sc = comm.scan(xi[lo:hi].contiguous())
            v, i, c, off, total = comm.compact_gt(xn[clo:chi].contiguous(), 0.5, index_base=1 + clo)
            comm.check()
            k = int(c.item())
            res.append((float(tot.item()), sc.cpu().numpy().tobytes(), v[:k].cpu().numpy().tobytes(),
                        i[:k].cpu().numpy().tobytes(), k, int(off.item()), int(total.item())))
        # the same scan with the shard in pinned host memory (two-phase host-buffer path)
        xh = xi[lo:hi].cpu().pin_memory()
        yh = comm.scan_host(xh)
        torch.cuda.synchronize()
        comm.check()
        results[("host", rank)] = yh.numpy().tobytes()
        results[rank] = (comm.exchange, res)
        comm.close()
        comm = None
    finally:
        if comm is not None:
            comm.abort()
        dist.destroy_process_group()


@pytest.mark.parametrize("world,exchange", [(2, "peer"), (2, "nccl"), (4, "auto"), (8, "auto")])
def test_sharded_ops_process_per_gpu(world, exchange, KI, oracle):
    import torch
    import torch.multiprocessing as mp

    _need(world)
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    results = mgr.dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, exchange, results)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
        assert p.exitcode == 0
    xn_host = _inputs(KI, torch.device("cuda", 0))[2].cpu().numpy()
    want_mode = "nccl" if exchange == "nccl" else "peer"
    want_scan = oracle.cumsum_i64(oracle.gen_int_range_i64(3, -1000, 1000, N_SCAN))
    got = np.concatenate([np.frombuffer(results[("host", r)], dtype=np.int64) for r in range(world)])
    assert np.array_equal(got, want_scan)
    for rnd in range(2):
        rs = [results[r][1][rnd] for r in range(world)]
        assert all(results[r][0] == want_mode for r in range(world))
        _check(oracle, world, [x[0] for x in rs], [np.frombuffer(x[1], dtype=np.int64) for x in rs],
               [np.frombuffer(x[2], dtype=np.float32) for x in rs], [np.frombuffer(x[3], dtype=np.int32) for x in rs],
               [x[4] for x in rs], [x[5] for x in rs], [x[6] for x in rs], xn_host)


def _leaver(rank, world, port, results):
    """Rank 1 stops taking part between steps (nothing of it in flight) but stays alive, so its
    exchange buffer stays mapped; rank 0's next exchange waits for it, runs out (0.2 s) and reports
    KI_ERR_TIMEOUT.  Rank 1 exits only after rank 0 has aborted its communicator."""
    import datetime
    import sys
    import time
    from pathlib import Path

    repo = Path(__file__).resolve().parent.parent
    sys.path.insert(0, str(repo / "kernelintrinsics.jl_b200"))
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import torch
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    from kernelintrinsics import sharded

    comm = sharded.Comm.from_process_group(device=rank, exchange="peer")
    x = torch.ones(4096, dtype=torch.float32, device=torch.device("cuda", rank))
    comm.reduce_sum(x)  # one good step together
    comm.check()
    dist.barrier()
    if rank == 1:  # leaves the computation, not the process
        deadline = time.time() + 120
        while "after" not in results and time.time() < deadline:
            time.sleep(0.05)
        comm.abort()
        os._exit(0)
    comm.set_wait_timeout(0.2)
    comm.reduce_sum(x)
    try:
        comm.check()
        results[rank] = "no error"
    except Exception as e:  # noqa: BLE001 - the timeout is the expected outcome
        results[rank] = type(e).__name__
    comm.abort()
    results["after"] = x.sum().item()  # the device is still usable afterwards
    os._exit(0)


def test_rank_that_stops_is_detected(KI):
    import torch.multiprocessing as mp

    _need(2)
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    results = mgr.dict()
    port = _free_port()
    procs = [ctx.Process(target=_leaver, args=(r, 2, port, results)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
    assert results.get(0) == "KITimeoutError"
    assert results.get("after") == 4096.0
