"""GPU: stream compaction (filter / findall) and the device generators."""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n", [1, 2, 31, 32, 33, 4095, 4096, 4097, 100003, (1 << 20) + 1])
@pytest.mark.parametrize("offset", [0, 1])
def test_compact_vs_oracle(KI, oracle, dev, n, offset):
    import torch

    base = torch.empty(n + offset, dtype=torch.float32, device=dev)
    KI.fill_normal(base, seed=4)
    x = base[offset:]
    host = x.cpu().numpy()
    for index_base in (1, 0, 1000):
        vals, idx, cnt = KI.vote_compact(x, 0.5, index_base=index_base)
        KI.context(0).check()
        rv, ri = oracle.filter_gt_f32(host, 0.5, index_base=index_base)
        assert cnt.item() == rv.size
        assert np.array_equal(vals.cpu().numpy(), rv)
        assert np.array_equal(idx.cpu().numpy(), ri)


def test_compact_edge_values(KI, oracle, dev):
    import torch

    host = np.array([0.5, np.nextafter(np.float32(0.5), np.float32(1)), np.nan, np.inf, -np.inf, 0.49999997, 7.0]
                    * 1000, dtype=np.float32)
    x = torch.from_numpy(host).to(dev)
    vals, idx, cnt = KI.vote_compact(x, 0.5)
    rv, ri = oracle.filter_gt_f32(host, 0.5)
    assert np.array_equal(vals.cpu().numpy(), rv) and np.array_equal(idx.cpu().numpy(), ri)
    e, ei, ec = KI.vote_compact(torch.empty(0, dtype=torch.float32, device=dev), 0.5)
    assert ec.item() == 0 and e.numel() == 0
    none = torch.zeros(10000, dtype=torch.float32, device=dev)
    assert KI.vote_compact(none, 0.5)[2].item() == 0
    allk = torch.ones(10000, dtype=torch.float32, device=dev)
    v, i, c = KI.vote_compact(allk, 0.5)
    assert c.item() == 10000 and torch.equal(i.cpu(), torch.arange(1, 10001, dtype=torch.int32))


def test_compact_single_output_and_top_index(KI, oracle, dev):
    """Values only and indices only (null output pointers through the C ABI), and indices that end
    exactly at typemax(Int32)."""
    import ctypes

    import torch

    n = 3 * 16384 + 999
    x = torch.empty(n, dtype=torch.float32, device=dev)
    KI.fill_normal(x, seed=9)
    host = x.cpu().numpy()
    ctx = KI.context(0)
    stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    for index_base in (1, 2**31 - n):
        rv, ri = oracle.filter_gt_f32(host, 0.5, index_base=index_base)
        vals = torch.full((n,), -7.0, dtype=torch.float32, device=dev)
        idx = torch.full((n,), -7, dtype=torch.int32, device=dev)
        cnt = torch.zeros((), dtype=torch.uint64, device=dev)
        ctx.call("ki_compact_gt_f32", ctypes.c_void_p(x.data_ptr()), n, ctypes.c_float(0.5),
                 ctypes.c_void_p(vals.data_ptr()), None, ctypes.c_int64(index_base), ctypes.c_void_p(cnt.data_ptr()),
                 stream)
        ctx.call("ki_compact_gt_f32", ctypes.c_void_p(x.data_ptr()), n, ctypes.c_float(0.5), None,
                 ctypes.c_void_p(idx.data_ptr()), ctypes.c_int64(index_base), None, stream)
        ctx.check()
        k = rv.size
        assert cnt.item() == k
        assert np.array_equal(vals[:k].cpu().numpy(), rv) and (vals[k:] == -7.0).all().item()
        assert np.array_equal(idx[:k].cpu().numpy(), ri) and (idx[k:] == -7).all().item()
    assert ri[-1] <= 2**31 - 1


def test_compact_rejects_index_overflow(KI, dev):
    import torch

    x = torch.zeros(16, dtype=torch.float32, device=dev)
    with pytest.raises(KI.KIArgumentError):
        KI.vote_compact(x, 0.5, index_base=2**31 - 4)


def test_compact_config_size(KI, dev, oracle):
    """n = 2^28 N(0,1), x > 0.5: bit-exact against the oracle's filter/findall (multithreaded C) on the
    host copy of the same data; k near 0.30854 n."""
    import numpy as np
    import torch

    n = 1 << 28
    x = torch.empty(n, dtype=torch.float32, device=dev)
    KI.fill_normal(x, seed=4)
    vals, idx, cnt = KI.vote_compact(x, 0.5)
    KI.context(0).check()
    k = cnt.item()
    rv, ri = oracle.filter_gt_f32(x.cpu().numpy(), 0.5)
    assert k == rv.size
    assert abs(k / n - 0.308538) < 1e-3
    assert np.array_equal(idx.cpu().numpy(), ri)
    assert np.array_equal(vals.cpu().numpy().view(np.uint32), rv.view(np.uint32))
    del x, vals, idx
    torch.cuda.empty_cache()


def test_generators_match_host(KI, oracle, dev):
    import torch

    n = (1 << 20) + 13
    u = torch.empty(n, dtype=torch.float32, device=dev)
    KI.fill_uniform(u, seed=1)
    assert np.array_equal(u.cpu().numpy(), oracle.gen_uniform_f32(1, n))
    i = torch.empty(n, dtype=torch.int64, device=dev)
    KI.fill_int_range(i, seed=3, lo=-1000, hi=1000)
    assert np.array_equal(i.cpu().numpy(), oracle.gen_int_range_i64(3, -1000, 1000, n))
    b = torch.empty(n, dtype=torch.uint8, device=dev)
    KI.fill_bytes(b, seed=2)
    assert np.array_equal(b.cpu().numpy(), oracle.gen_bytes(2, n))
    bo = torch.empty(n + 3, dtype=torch.uint8, device=dev)[3:]  # unaligned start
    KI.fill_bytes(bo, seed=2)
    assert np.array_equal(bo.cpu().numpy(), oracle.gen_bytes(2, n))
    q = torch.empty(n, dtype=torch.uint8, device=dev)
    KI.fill_e4m3_uniform(q, seed=5, scale=112.0)
    assert np.array_equal(q.cpu().numpy(), oracle.gen_e4m3_uniform(5, 112.0, n))


def test_normal_generator_distribution(KI, dev):
    import torch

    n = 1 << 24
    z = torch.empty(n, dtype=torch.float32, device=dev)
    KI.fill_normal(z, seed=4)
    zd = z.double()
    assert abs(zd.mean().item()) < 2e-3 and abs(zd.std().item() - 1) < 2e-3
    assert abs((z > 0.5).double().mean().item() - 0.308538) < 1e-3
    assert torch.isfinite(z).all()


PRED_FN = {">": np.greater, ">=": np.greater_equal, "<": np.less, "<=": np.less_equal, "==": np.equal,
           "!=": np.not_equal}


@pytest.mark.parametrize("dt", [np.int32, np.uint32, np.int64, np.uint64, np.float32, np.float64],
                         ids=lambda d: np.dtype(d).name)
@pytest.mark.parametrize("pred", list(PRED_FN))
def test_compact_generic_vs_oracle(KI, dev, dt, pred):
    """ki_compact: every predicate and element type; sizes across tile boundaries (8192 / 16384
    elements), an unaligned start, NaN for floats; bit-exact against numpy's IEEE comparisons."""
    import torch

    rng = np.random.default_rng(17)
    for n, off in [(1, 0), (100, 1), (8191, 0), (8193, 1), (16385, 0), (3 * 16384 + 77, 1), ((1 << 20) + 13, 0)]:
        if np.dtype(dt).kind == "f":
            base = rng.integers(-8, 8, n + off).astype(dt) * np.asarray(0.5, dtype=dt)
            base[rng.integers(0, n + off, 5)] = np.nan
            thr = np.asarray(1.5, dtype=dt)
        else:
            base = rng.integers(0 if np.dtype(dt).kind == "u" else -8, 8, n + off).astype(dt)
            thr = np.asarray(3, dtype=dt)
        x = base[off:]
        xd = torch.from_numpy(base).to(dev)[off:]
        vals, idx, cnt = KI.compact(xd, pred, thr.item(), index_base=1)
        keep = np.nonzero(PRED_FN[pred](x, thr))[0]
        assert cnt.item() == keep.size, (n, off)
        assert np.array_equal(idx.cpu().numpy(), (keep + 1).astype(np.int32)), (n, off)
        assert np.array_equal(vals.cpu().numpy().view(np.uint8), x[keep].view(np.uint8)), (n, off)
    KI.context(0).check()


@pytest.mark.parametrize("dt", [np.int32, np.uint32, np.int64, np.uint64, np.float32, np.float64],
                         ids=lambda d: np.dtype(d).name)
@pytest.mark.parametrize("f", ["abs", "abs2"])
def test_compact_mapped_vs_oracle(KI, oracle, dev, dt, f):
    """Fused map-then-compact: filter(v -> f(v) pred t, x) keeps x's own elements; integer maps wrap
    (abs(typemin), abs2 overflow), as Base's do."""
    import torch

    rng = np.random.default_rng(29)
    info = np.iinfo(dt) if np.dtype(dt).kind != "f" else None
    for n, off in [(1, 0), (1000, 1), (16385, 0), ((1 << 20) + 13, 1)]:
        if info is None:
            base = (rng.standard_normal(n + off) * 2).astype(dt)
            base[rng.integers(0, n + off, 4)] = np.nan
            base[rng.integers(0, n + off, 4)] = -0.0
            thr = 1.5
        else:
            base = rng.integers(info.min, info.max, n + off, dtype=dt, endpoint=True)
            base[rng.integers(0, n + off, 4)] = info.min
            base[: min(64, n + off)] = rng.integers(-20 if info.min < 0 else 0, 20, min(64, n + off)).astype(dt)
            thr = 50 if f == "abs2" else 7
        x = base[off:]
        xd = torch.from_numpy(base).to(dev)[off:]
        for pred in (">", "<=", "!="):
            vals, idx, cnt = KI.compact(xd, pred, thr, f=f)
            want_v, want_i = oracle.filter_pred(x, pred, thr, f=f)
            assert cnt.item() == want_i.size, (n, off, pred)
            assert np.array_equal(idx.cpu().numpy(), want_i), (n, off, pred)
            assert np.array_equal(vals.cpu().numpy().view(np.uint8), want_v.view(np.uint8)), (n, off, pred)
            assert KI.count(xd, pred, thr, f=f).item() == want_i.size
    KI.context(0).check()


def test_count_plain(KI, oracle, dev):
    import torch

    x = np.random.default_rng(3).standard_normal((1 << 22) + 5).astype(np.float32)
    xd = torch.from_numpy(x).to(dev)
    for pred, t in ((">", 0.5), ("<", -1.0), ("==", 0.0)):
        assert KI.count(xd, pred, t).item() == oracle.filter_pred(x, pred, t)[1].size
