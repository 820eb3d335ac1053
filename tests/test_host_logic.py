"""CPU: the range-sharding logic of kernelintrinsics.sharded, run as 2 gloo ranks.

The per-shard kernels are replaced by CPU implementations (the oracle) injected through
``ShardOps``; the collective plumbing (all-gather of totals / counts, seeds, offsets) is the
product code under test.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from kernelintrinsics.sharded import ShardOps, exclusive_prefix, shard_range, wrap64


def test_shard_range_partition():
    for n in (0, 1, 7, 32, 1000, 2**30 + 3):
        for world in (1, 2, 3, 4, 8):
            spans = [shard_range(n, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            for (a, b), (c, d) in zip(spans, spans[1:]):
                assert b == c and b >= a
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_range(10, 0, 0)


def test_prefix_and_wrap():
    assert exclusive_prefix([3, 0, 5]) == [0, 3, 3]
    assert wrap64(2**63) == -(2**63)
    assert wrap64(-1) == -1


def _oracle_ops():
    import ki_oracle as o

    def compact(x, thr, base):
        v, i = o.filter_gt_f32(x.numpy(), thr, index_base=base)
        return torch.from_numpy(v), torch.from_numpy(i), torch.tensor(len(v), dtype=torch.int64)

    return ShardOps(
        sum_f32_to_f64=lambda x: torch.tensor(o.sum_f32(x.numpy()), dtype=torch.float64),
        sum_i64=lambda x: torch.tensor(o.sum_i64(x.numpy()), dtype=torch.int64),
        scan_i64=lambda x, out, seed: out.copy_(torch.from_numpy(o.cumsum_i64(x.numpy(), seed=seed))),
        compact_gt=compact,
    )


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, results):
    import sys
    from pathlib import Path

    repo = Path(__file__).resolve().parent.parent
    for p in (repo / "kernelintrinsics.jl_b200", repo / "oracle"):
        sys.path.insert(0, str(p))
    from kernelintrinsics import sharded
    import ki_oracle as o

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        ops = _oracle_ops()
        n = 10007
        xi = torch.from_numpy(o.gen_int_range_i64(3, -1000, 1000, n))
        xf = torch.from_numpy(o.gen_uniform_f32(1, n))
        xn = torch.from_numpy(o.gen_normal_f32_host(4, n))
        lo, hi = shard_range(n, world, rank)
        tot = sharded.reduce_sharded(xf[lo:hi], ops=ops)
        sc = sharded.scan_sharded(xi[lo:hi].clone(), ops=ops)
        v, i, k, off, total = sharded.compact_sharded(xn[lo:hi].clone(), 0.5, lo, ops=ops)
        results[rank] = (float(tot), sc.numpy().tobytes(), v.numpy().tobytes(), i.numpy().tobytes(), k, off, total)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_sharded_ops_gloo(world):
    import ki_oracle as o

    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    results = mgr.dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, results)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    n = 10007
    xi = o.gen_int_range_i64(3, -1000, 1000, n)
    xf = o.gen_uniform_f32(1, n)
    xn = o.gen_normal_f32_host(4, n)
    ref_sum = xf.astype(np.float64).sum()
    ref_scan = np.cumsum(xi)
    keep = np.nonzero(xn > np.float32(0.5))[0]
    sums = [results[r][0] for r in range(world)]
    assert len(set(sums)) == 1 and abs(sums[0] - ref_sum) <= 1e-9 * ref_sum  # same bits on every rank
    scan = np.concatenate([np.frombuffer(results[r][1], dtype=np.int64) for r in range(world)])
    assert np.array_equal(scan, ref_scan)
    vals = np.concatenate([np.frombuffer(results[r][2], dtype=np.float32) for r in range(world)])
    idx = np.concatenate([np.frombuffer(results[r][3], dtype=np.int32) for r in range(world)])
    assert np.array_equal(vals, xn[keep]) and np.array_equal(idx, keep + 1)
    offs = [results[r][5] for r in range(world)]
    assert offs == exclusive_prefix([results[r][4] for r in range(world)])
    assert all(results[r][6] == keep.size for r in range(world))


def _dead_rank_worker(rank, world, port, results):
    """Rank 1 leaves before the collective; rank 0's all-gather must end with an error, not hang."""
    import datetime
    import sys
    from pathlib import Path

    repo = Path(__file__).resolve().parent.parent
    sys.path.insert(0, str(repo / "kernelintrinsics.jl_b200"))
    from kernelintrinsics import sharded

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        os._exit(0)  # leaves between steps, nothing in flight
    ops = ShardOps(sum_f32_to_f64=lambda x: torch.tensor(float(x.sum()), dtype=torch.float64),
                   sum_i64=None, scan_i64=None, compact_gt=None)
    try:
        sharded.reduce_sharded(torch.ones(8), ops=ops)
        results[rank] = "no error"
    except Exception as e:  # noqa: BLE001 - any collective error is the expected outcome
        results[rank] = type(e).__name__
    os._exit(0)


def test_dead_rank_is_detected_on_host():
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    results = mgr.dict()
    port = _free_port()
    procs = [ctx.Process(target=_dead_rank_worker, args=(r, 2, port, results)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    assert results.get(0) not in (None, "no error")


# ---------------------------------------------------------------------------------------------
# the C-ABI communicator: host-only parts
# ---------------------------------------------------------------------------------------------
def test_c_shard_range_matches_python():
    import ctypes

    from kernelintrinsics import _abi

    lib = _abi.load()
    lo, cnt = ctypes.c_size_t(), ctypes.c_size_t()
    for n in (0, 1, 7, 1000, 2**30 + 3, 2**28):
        for world in (1, 2, 3, 8, 64):
            for r in range(world):
                assert lib.ki_comm_shard_range(n, world, r, ctypes.byref(lo), ctypes.byref(cnt)) == _abi.KI_OK
                a, b = shard_range(n, world, r)
                assert (lo.value, cnt.value) == (a, b - a)
    from kernelintrinsics.sharded import scan_shard_range

    for n in (0, 1, 255, 256 * 17 + 3, 2**30, 2**30 + 7):
        for world in (1, 2, 3, 4, 8):
            spans = [scan_shard_range(n, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            for (a, b), (c, d) in zip(spans, spans[1:]):
                assert b == c and a <= b and a % 256 == 0
            for r in range(world):
                assert lib.ki_comm_scan_shard_range(n, world, r, ctypes.byref(lo), ctypes.byref(cnt)) == _abi.KI_OK
                assert (lo.value, lo.value + cnt.value) == spans[r]
            if n >= 2**30 and world > 1:  # the last rank holds 3/2 of the others' share
                sizes = [b - a for a, b in spans]
                assert abs(sizes[-1] / sizes[0] - 1.5) < 1e-3
    assert lib.ki_comm_shard_range(10, 0, 0, ctypes.byref(lo), ctypes.byref(cnt)) == _abi.KI_ERR_ARG
    assert lib.ki_comm_shard_range(10, 2, 2, ctypes.byref(lo), ctypes.byref(cnt)) == _abi.KI_ERR_ARG


def test_comm_argument_checks_without_a_gpu():
    """Invalid communicator arguments are rejected before any CUDA or NCCL call."""
    import ctypes

    from kernelintrinsics import _abi

    lib = _abi.load()
    h = ctypes.c_void_p()
    cid = ctypes.create_string_buffer(128)
    assert lib.ki_comm_init_rank(0, 0, 0, cid, 0, ctypes.byref(h)) == _abi.KI_ERR_ARG      # no ranks
    assert lib.ki_comm_init_rank(0, 65, 0, cid, 0, ctypes.byref(h)) == _abi.KI_ERR_ARG     # > KI_COMM_MAX_RANKS
    assert lib.ki_comm_init_rank(0, 2, 2, cid, 0, ctypes.byref(h)) == _abi.KI_ERR_ARG      # rank out of range
    assert lib.ki_comm_init_rank(0, 2, 0, None, 0, ctypes.byref(h)) == _abi.KI_ERR_ARG     # no id
    assert lib.ki_comm_init_rank(0, 2, 0, cid, 7, ctypes.byref(h)) == _abi.KI_ERR_ARG      # unknown exchange
    devs = (ctypes.c_int * 1)(0)
    hs = (ctypes.c_void_p * 1)()
    assert lib.ki_comm_create(0, devs, hs) == _abi.KI_ERR_ARG
    assert lib.ki_comm_destroy(None) == _abi.KI_OK and lib.ki_comm_abort(None) == _abi.KI_OK
    assert lib.ki_reduce_sum_f32_sharded(None, None, 0, None, None, None) == _abi.KI_ERR_ARG
    assert lib.ki_scan_inclusive_i64_sharded(None, None, None, 0, None) == _abi.KI_ERR_ARG
    assert lib.ki_compact_gt_f32_sharded(None, None, 0, 0.5, None, None, 1, None, None, None, None) == _abi.KI_ERR_ARG
    assert b"KI_ERR_NCCL" in lib.ki_status_string(_abi.KI_ERR_NCCL)


def _id_worker(rank, world, port, results):
    import sys
    from pathlib import Path

    repo = Path(__file__).resolve().parent.parent
    sys.path.insert(0, str(repo / "kernelintrinsics.jl_b200"))
    from kernelintrinsics import sharded

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        made = []

        def make_id():
            made.append(rank)
            return bytes(range(128))

        cid = sharded.broadcast_comm_id(make_id)
        results[rank] = (cid, list(made))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_comm_id_broadcast_gloo(world):
    """Rank 0 alone makes the NCCL unique id; every rank receives the same 128 bytes."""
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    results = mgr.dict()
    port = _free_port()
    procs = [ctx.Process(target=_id_worker, args=(r, world, port, results)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    for r in range(world):
        cid, made = results[r]
        assert cid == bytes(range(128))
        assert made == ([0] if r == 0 else [])
