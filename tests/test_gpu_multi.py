"""GPU, 2+ devices: range-sharded reduce / scan / compaction over NCCL against the oracle.

Each rank owns a contiguous shard; only one 8-byte value per rank crosses NVLink (an all-gather of
shard totals or counts).  Skipped when fewer than 2 GPUs are visible.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, n_scan, n_cmp, results):
    import datetime
    import sys
    from pathlib import Path

    repo = Path(__file__).resolve().parent.parent
    sys.path.insert(0, str(repo / "kernelintrinsics.jl_b200"))
    import torch
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        import kernelintrinsics as KI
        from kernelintrinsics import sharded

        dev = torch.device("cuda", rank)
        # the whole inputs are generated on every rank (same stream), each rank keeps its shard
        xi = torch.empty(n_scan, dtype=torch.int64, device=dev)
        KI.fill_int_range(xi, seed=3, lo=-1000, hi=1000)
        xf = torch.empty(n_scan, dtype=torch.float32, device=dev)
        KI.fill_uniform(xf, seed=1)
        xn = torch.empty(n_cmp, dtype=torch.float32, device=dev)
        KI.fill_normal(xn, seed=4)
        lo, hi = sharded.shard_range(n_scan, world, rank)
        clo, chi = sharded.shard_range(n_cmp, world, rank)
        tot = sharded.reduce_sharded(xf[lo:hi])
        sc = sharded.scan_sharded(xi[lo:hi].contiguous())
        v, i, k, off, total = sharded.compact_sharded(xn[clo:chi].contiguous(), 0.5, clo)
        KI.context(rank).check()
        torch.cuda.synchronize()
        results[rank] = (float(tot), sc.cpu().numpy().tobytes(), v.cpu().numpy().tobytes(),
                         i.cpu().numpy().tobytes(), k, off, total)
    finally:
        dist.barrier()
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_sharded_ops_nccl(world, oracle):
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    n_scan, n_cmp = (1 << 22) + 12345, (1 << 21) + 777
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    results = mgr.dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, n_scan, n_cmp, results)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
        assert p.exitcode == 0
    xi = oracle.gen_int_range_i64(3, -1000, 1000, n_scan)
    xf = oracle.gen_uniform_f32(1, n_scan)
    ref_sum = oracle.sum_f32(xf)
    sums = [results[r][0] for r in range(world)]
    assert len(set(sums)) == 1  # every rank holds the same bits
    assert abs(sums[0] - ref_sum) <= 1e-9 * ref_sum
    scan = np.concatenate([np.frombuffer(results[r][1], dtype=np.int64) for r in range(world)])
    assert np.array_equal(scan, oracle.cumsum_i64(xi))
    vals = np.concatenate([np.frombuffer(results[r][2], dtype=np.float32) for r in range(world)])
    idx = np.concatenate([np.frombuffer(results[r][3], dtype=np.int32) for r in range(world)])
    # the oracle runs on the device-generated normals (same seed on every rank)
    xn = None
    import torch as _t
    import kernelintrinsics as KI
    d = _t.empty(n_cmp, dtype=_t.float32, device="cuda:0")
    KI.fill_normal(d, seed=4)
    xn = d.cpu().numpy()
    rv, ri = oracle.filter_gt_f32(xn, 0.5)
    assert np.array_equal(vals, rv) and np.array_equal(idx, ri)
    assert all(results[r][6] == rv.size for r in range(world))
