"""GPU: grid reduce (sum) and decoupled-lookback scan (cumsum) against the oracle."""
from __future__ import annotations

import math

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _tol(n):
    return 1e-5 * max(1.0, math.log2(max(n, 2)))


@pytest.mark.parametrize("n", [1, 2, 3, 5, 31, 32, 33, 255, 1000, 4097, (1 << 20) + 7, 1 << 24])
@pytest.mark.parametrize("offset", [0, 1, 3])
def test_reduce_f32_vs_oracle(KI, oracle, dev, n, offset):
    import torch

    base = torch.empty(n + offset, dtype=torch.float32, device=dev)
    KI.fill_uniform(base, seed=1)
    x = base[offset:]
    out = KI.warpfold_reduce(x)
    f32 = torch.empty((), dtype=torch.float32, device=dev)
    KI.warpfold_reduce(x, out_f32=f32)
    ref = oracle.sum_f32(x.cpu().numpy())
    got = out.item()
    assert abs(got - ref) <= _tol(n) * abs(ref), (got, ref)
    assert abs(f32.item() - ref) <= _tol(n) * abs(ref)
    assert KI.warpfold_reduce(x).item() == got  # deterministic bits


def test_reduce_config_size_pinned_to_host_generator(KI, oracle, dev):
    import torch

    n = 1 << 24
    x = torch.empty(n, dtype=torch.float32, device=dev)
    KI.fill_uniform(x, seed=1)
    host = oracle.gen_uniform_f32(1, n)
    assert np.array_equal(x.cpu().numpy(), host)
    ref = oracle.sum_f32(host)
    got = KI.warpfold_reduce(x).item()
    assert abs(got - ref) <= _tol(n) * ref
    assert abs(got - ref) <= 1e-9 * ref  # in practice Float64-accurate


def test_reduce_back_to_back_overlapped_launches(KI, oracle, dev):
    """Reduces launched back to back (in a CUDA graph, where each launch's dispatch and L2
    prefetches overlap the previous launch) give the bits of one reduce at a time, also when the
    kernel before a reduce rewrites that reduce's input (the reduce must wait for it)."""
    import torch

    n = (1 << 22) + 3
    xs = [torch.empty(n, dtype=torch.float32, device=dev) for _ in range(4)]
    for k, x in enumerate(xs):
        KI.fill_uniform(x, seed=40 + k)
    want = [KI.warpfold_reduce(x).item() for x in xs]
    outs = [torch.empty((), dtype=torch.float64, device=dev) for _ in range(12)]
    refill = [torch.empty((), dtype=torch.float64, device=dev) for _ in range(4)]
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    cs = torch.cuda.Stream(dev)
    with torch.cuda.stream(cs):
        KI.warpfold_reduce(xs[0], out_f64=outs[0])  # warm-up on the capture stream
        torch.cuda.synchronize()
        with torch.cuda.graph(g, stream=cs):
            for j in range(12):  # reduce after reduce
                KI.warpfold_reduce(xs[j % 4], out_f64=outs[j])
            for k in range(4):  # a fill of the very input the next reduce reads
                KI.fill_uniform(xs[k], seed=60 + k)
                KI.warpfold_reduce(xs[k], out_f64=refill[k])
    for _ in range(3):
        for k, x in enumerate(xs):  # restore the first inputs before each replay
            KI.fill_uniform(x, seed=40 + k)
        g.replay()
        torch.cuda.synchronize()
        assert [o.item() for o in outs] == [want[j % 4] for j in range(12)]
        for k in range(4):
            ref = oracle.sum_f32(oracle.gen_uniform_f32(60 + k, n))
            assert abs(refill[k].item() - ref) <= _tol(n) * ref
            assert refill[k].item() == KI.warpfold_reduce(xs[k]).item()
    del g


def test_reduce_empty_and_special(KI, dev):
    import torch

    assert KI.warpfold_reduce(torch.empty(0, dtype=torch.float32, device=dev)).item() == 0.0
    x = torch.ones(1 << 20, dtype=torch.float32, device=dev)
    assert KI.warpfold_reduce(x).item() == float(1 << 20)
    x[12345] = float("inf")
    assert math.isinf(KI.warpfold_reduce(x).item())


@pytest.mark.parametrize("n", [1, 2, 7, 4095, 4096, 4097, 8191, 65536 + 3, (1 << 22) + 5])
def test_reduce_i64_vs_oracle(KI, oracle, dev, n):
    import torch

    x = torch.empty(n + 1, dtype=torch.int64, device=dev)
    KI.fill_int_range(x, seed=3, lo=-1000, hi=1000)
    for xs in (x[:n], x[1:]):
        assert KI.reduce_sum_i64(xs).item() == oracle.sum_i64(xs.cpu().numpy())


@pytest.mark.parametrize("n", [1, 2, 3, 31, 32, 4095, 4096, 4097, 8192, 12289, 15871, 15872, 15873, 31745,
                               (1 << 16) + 3, (1 << 22) + 5])
def test_scan_vs_oracle(KI, oracle, dev, n):
    import torch

    x = torch.empty(n, dtype=torch.int64, device=dev)
    KI.fill_int_range(x, seed=3, lo=-1000, hi=1000)
    host = x.cpu().numpy()
    assert np.array_equal(host, oracle.gen_int_range_i64(3, -1000, 1000, n))
    y = KI.warpreduce_scan(x)
    KI.context(0).check()
    assert np.array_equal(y.cpu().numpy(), oracle.cumsum_i64(host))
    ys = KI.warpreduce_scan(x, seed=-123456789)
    assert np.array_equal(ys.cpu().numpy(), oracle.cumsum_i64(host, seed=-123456789))


def test_scan_misaligned_and_in_place(KI, oracle, dev):
    import torch

    n = 3 * 15872 + 17
    base = torch.empty(n + 1, dtype=torch.int64, device=dev)
    KI.fill_int_range(base, seed=9, lo=-5, hi=5)
    x = base[1:]  # 8 mod 16: the plain-load path
    host = x.cpu().numpy()
    assert np.array_equal(KI.warpreduce_scan(x).cpu().numpy(), oracle.cumsum_i64(host))
    KI.warpreduce_scan(x, out=x)  # in place
    assert np.array_equal(x.cpu().numpy(), oracle.cumsum_i64(host))


def test_scan_wraps_like_int64(KI, oracle, dev):
    import torch

    host = np.full(3 * 15872 + 5, 2**61 + 12345, dtype=np.int64)
    host[::7] = -(2**62)
    x = torch.from_numpy(host).to(dev)
    assert np.array_equal(KI.warpreduce_scan(x).cpu().numpy(), oracle.cumsum_i64(host))


def test_scan_repeated_for_races(KI, oracle, dev):
    import torch

    n = (1 << 22) + 11
    x = torch.empty(n, dtype=torch.int64, device=dev)
    KI.fill_int_range(x, seed=31, lo=-1000, hi=1000)
    ref = torch.from_numpy(oracle.cumsum_i64(x.cpu().numpy())).to(dev)
    y = torch.empty_like(x)
    for _ in range(50):
        KI.warpreduce_scan(x, out=y)
        assert torch.equal(y, ref)
    KI.context(0).check()


def test_scan_config_size_properties(KI, dev):
    """n = 2^30: out[0] == in[0] and out[i] - out[i-1] == in[i] for all i (this fixes out exactly)."""
    import torch

    n = 1 << 30
    x = torch.empty(n, dtype=torch.int64, device=dev)
    KI.fill_int_range(x, seed=3, lo=-1000, hi=1000)
    y = KI.warpreduce_scan(x)
    KI.context(0).check()
    assert y[0].item() == x[0].item()
    chunk = 1 << 27
    for s in range(0, n, chunk):
        e = min(n, s + chunk + 1)
        assert torch.equal(y[s + 1:e] - y[s:e - 1], x[s + 1:e])
    assert y[-1].item() == KI.reduce_sum_i64(x).item()
    del x, y
    torch.cuda.empty_cache()
