"""GPU, one device: the communicator path and the device-seeded scan, against the oracle.

A one-rank communicator runs the whole sharded protocol (shard kernel, exchange kernel over its own
exchange buffer, epoch counter, seeded phase 2), so this file checks the exchange kernel and the
C-ABI plumbing on a single B200; tests/test_gpu_multi.py runs the same operations on 2, 4 and 8.
"""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n", [1, 15871, 15872 * 3 + 1, (1 << 22) + 12345])
def test_dseed_scan_matches_oracle(KI, dev, oracle, n):
    import ctypes

    import torch

    x = torch.empty(n, dtype=torch.int64, device=dev)
    KI.fill_int_range(x, seed=3, lo=-1000, hi=1000)
    y = torch.empty_like(x)
    seed = torch.tensor([-(1 << 50) + 17], dtype=torch.int64, device=dev)
    KI.context(0).call("ki_scan_inclusive_i64_dseed", ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(y.data_ptr()),
                       n, ctypes.c_void_p(seed.data_ptr()), ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream))
    KI.context(0).check()
    want = oracle.cumsum_i64(oracle.gen_int_range_i64(3, -1000, 1000, n), seed=-(1 << 50) + 17)
    assert np.array_equal(y.cpu().numpy(), want)


def test_single_rank_comm_matches_oracle(KI, dev, oracle):
    """Three rounds of reduce, scan and compaction on a one-rank communicator (the epoch counter
    advances every call; both exchange-buffer parities are used)."""
    import torch

    from kernelintrinsics import sharded

    (comm,) = sharded.Comm.create([0])
    try:
        assert (comm.nranks, comm.rank, comm.device, comm.exchange) == (1, 0, 0, "peer")
        for rnd in range(3):
            n = (1 << 20) + 4099 * rnd + 1
            xf = torch.empty(n, dtype=torch.float32, device=dev)
            KI.fill_uniform(xf, seed=1 + rnd)
            xi = torch.empty(n, dtype=torch.int64, device=dev)
            KI.fill_int_range(xi, seed=3 + rnd, lo=-1000, hi=1000)
            xn = torch.empty(n, dtype=torch.float32, device=dev)
            KI.fill_normal(xn, seed=4 + rnd)
            tot = comm.reduce_sum(xf)
            sc = comm.scan(xi)
            v, i, c, off, total = comm.compact_gt(xn, 0.5, index_base=1)
            comm.check()
            ref = oracle.sum_f32(oracle.gen_uniform_f32(1 + rnd, n))
            assert abs(tot.item() - ref) <= 1e-5 * np.log2(n) * ref
            assert np.array_equal(sc.cpu().numpy(), oracle.cumsum_i64(oracle.gen_int_range_i64(3 + rnd, -1000, 1000, n)))
            rv, ri = oracle.filter_gt_f32(xn.cpu().numpy(), 0.5)
            k = int(c.item())
            assert k == rv.size and int(off.item()) == 0 and int(total.item()) == k
            assert np.array_equal(v[:k].cpu().numpy(), rv) and np.array_equal(i[:k].cpu().numpy(), ri)
    finally:
        comm.close()


def test_single_rank_comm_empty_shard(KI, dev):
    """An empty shard still takes part in the exchange (zero total, zero count)."""
    import torch

    from kernelintrinsics import sharded

    (comm,) = sharded.Comm.create([0])
    try:
        e32 = torch.empty(0, dtype=torch.float32, device=dev)
        e64 = torch.empty(0, dtype=torch.int64, device=dev)
        assert comm.reduce_sum(e32).item() == 0.0
        comm.scan(e64)
        v, i, c, off, total = comm.compact_gt(e32, 0.5, index_base=1)
        comm.check()
        assert int(c.item()) == 0 and int(total.item()) == 0
        # the epoch counter stayed in step: a normal call afterwards is still right
        x = torch.ones(1000, dtype=torch.float32, device=dev)
        assert comm.reduce_sum(x).item() == 1000.0
        comm.check()
    finally:
        comm.close()


def test_comm_create_rejects_repeated_device(KI):
    import ctypes

    from kernelintrinsics import _abi

    lib = _abi.load()
    devs = (ctypes.c_int * 2)(0, 0)
    hs = (ctypes.c_void_p * 2)()
    assert lib.ki_comm_create(2, devs, hs) == _abi.KI_ERR_ARG


@pytest.mark.parametrize("n,inplace", [(1, False), ((1 << 21) + 7, False), (5 * (1 << 21) + 3, False),
                                       (5 * (1 << 21) + 3, True)])
def test_host_buffer_scan_matches_oracle(KI, dev, oracle, n, inplace):
    """cumsum of pinned host buffers through the GPU: chunks of 2^21 elements, each seeded on the
    device with the previous chunk's last value (n spans up to 6 chunks over the 4 staging slots)."""
    import torch

    xh = oracle.gen_int_range_i64(3, -1000, 1000, n)
    x = torch.from_numpy(xh).pin_memory()
    out = x if inplace else torch.empty_like(x).pin_memory()
    KI.warpreduce_scan_host(x, out=out, seed=123456789012, device=0)
    torch.cuda.synchronize()
    KI.context(0).check()
    assert np.array_equal(out.numpy(), oracle.cumsum_i64(xh, seed=123456789012))


def test_single_rank_comm_host_scan(KI, oracle):
    import torch

    from kernelintrinsics import sharded

    (comm,) = sharded.Comm.create([0])
    try:
        n = 3 * (1 << 21) + 11
        xh = oracle.gen_int_range_i64(7, -1000, 1000, n)
        x = torch.from_numpy(xh).pin_memory()
        y = comm.scan_host(x)
        torch.cuda.synchronize()
        comm.check()
        assert np.array_equal(y.numpy(), oracle.cumsum_i64(xh))
    finally:
        comm.close()
