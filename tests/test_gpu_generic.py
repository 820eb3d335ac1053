"""GPU: device-wide reduce and scan for +, *, max, min, |, &, xor over Int8 ... UInt64, Float32 and
Float64 (ki_reduce, ki_scan, ki_reduce_rows) against the oracle's Julia Base semantics.

Integers are bit-exact.  Float sums: |device - Float64 oracle| <= 1e-5*log2(n) * (running sum of |x|),
the tolerance the workload definition states for Float32 reduce/scan; float products: within
1e-5*log2(n) of the Float64 product, relative.  max/min are exact, NaN included.
"""
from __future__ import annotations

import math

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

NP_TYPES = [np.int8, np.uint8, np.int16, np.uint16, np.int32, np.uint32, np.int64, np.uint64, np.float32, np.float64]
OPS = ["+", "*", "max", "min", "|", "&", "xor"]
BITWISE = ("|", "&", "xor")


def _cases():
    """(dtype, op) pairs the operators take: the bitwise ones take integers only."""
    return [pytest.param(dt, op, id=f"{op}-{np.dtype(dt).name}") for op in OPS for dt in NP_TYPES
            if not (op in BITWISE and np.dtype(dt).kind == "f")]


def _data(dt, n, seed, op="max"):
    rng = np.random.default_rng(seed)
    dt = np.dtype(dt)
    if dt.kind == "f" and op == "*":  # log-normal factors: the product's log is a zero-mean walk
        return np.exp(0.01 * rng.standard_normal(n)).astype(dt)
    if dt.kind == "f":
        x = rng.standard_normal(n).astype(dt)
        if n > 10 and op != "+":  # for max/min: signed zeros, infinities (NaN has its own test)
            x[rng.integers(0, n, 3)] = -0.0
            x[rng.integers(0, n, 3)] = 0.0
            x[rng.integers(0, n, 1)] = np.inf if seed % 2 else -np.inf
        return x
    info = np.iinfo(dt)
    x = rng.integers(info.min, info.max, n, dtype=dt, endpoint=True)
    if op == "*":  # odd factors: the wrapped product never collapses to zero
        x |= dt.type(1)
    return x


def _to_dev(x, dev):
    import torch

    return torch.from_numpy(np.ascontiguousarray(x)).to(dev)


def _check(got, want, x, op):
    if np.dtype(want.dtype).kind == "f" and op == "*":
        n = max(2, x.size)
        err = np.abs(got.astype(np.float64) - want)
        assert (err <= 1e-5 * math.log2(n) * np.abs(want) + 1e-300).all(), float((err / np.abs(want)).max())
    elif np.dtype(want.dtype).kind == "f" and op == "+":
        n = max(2, x.size)
        scale = np.cumsum(np.abs(x.astype(np.float64)))
        err = np.abs(got.astype(np.float64) - want)
        assert (err <= 1e-5 * math.log2(n) * np.maximum(scale, 1e-30)).all(), float((err / np.maximum(scale, 1e-30)).max())
    elif np.dtype(want.dtype).kind == "f":
        assert np.array_equal(np.isnan(got), np.isnan(want))
        m = ~np.isnan(want)
        assert np.array_equal(got[m].view(np.uint8), want[m].astype(got.dtype).view(np.uint8))  # signed zeros too
    else:
        assert np.array_equal(got, want)


SIZES = [1, 2, 31, 33, 1000, 15871, 15872, 15873, 31743, 31744, 31745, 63489, 100_003, 126977, 253952, (1 << 20) + 3]


@pytest.mark.parametrize("dt,op", _cases())
def test_scan_inclusive_and_exclusive(KI, oracle, dev, dt, op):
    for k, n in enumerate(SIZES):
        x = _data(dt, n, 10 * k + 1, op)
        xd = _to_dev(x, dev)
        for excl in (False, True):
            got = KI.scan(xd, op, exclusive=excl).cpu().numpy()
            want = oracle.accumulate(op, x, exclusive=excl)
            _check(got, want, x if not excl else np.concatenate([[0], x[:-1]]).astype(x.dtype), op)
    KI.context(0).check()


@pytest.mark.parametrize("dt", [np.int32, np.int64, np.float32, np.float64], ids=lambda d: np.dtype(d).name)
def test_scan_init_misaligned_and_in_place(KI, oracle, dev, dt):
    import torch

    n = 3 * 31744 + 11
    init = 5 if np.dtype(dt).kind != "f" else 0.25
    for op in OPS:
        if op in BITWISE and np.dtype(dt).kind == "f":
            continue
        x = _data(dt, n + 1, 7, op)
        xs = _to_dev(x, dev)[1:]  # 4- or 8-byte offset: the plain-load path
        got = KI.scan(xs, op, init=init).cpu().numpy()
        want = oracle.accumulate(op, x[1:], init=init)
        _check(got, want, x[1:], op)
    if np.dtype(dt).itemsize == 8:  # result type as wide as the input: in place
        y = xs.clone()
        KI.scan(y, "max", out=y)
        assert np.array_equal(y.cpu().numpy(), oracle.accumulate("max", x[1:]))
    elif np.dtype(dt).kind == "i":  # a widened result cannot alias its input
        wide = torch.empty(n, dtype=torch.int64, device=dev)
        narrow = wide.view(torch.int32)[:n]
        with pytest.raises(KI.KIArgumentError):
            KI.scan(narrow, "+", out=wide)
    KI.context(0).check()


@pytest.mark.parametrize("dt", [np.float32, np.float64], ids=lambda d: np.dtype(d).name)
def test_cumsum_keeps_negative_zeros(KI, oracle, dev, dt):
    """Base.cumsum over negative zeros gives negative zeros (the first output is x[1], sign included):
    bit-exact against the oracle, for plain scans of one to many tiles and for short and long rows."""
    for n in (5, 40000, 300001):
        x = np.full(n, -0.0, dtype=dt)
        x[n // 2] = 1.5
        got = KI.scan(_to_dev(x, dev), "+").cpu().numpy()
        want = oracle.accumulate("+", x).astype(got.dtype)
        assert np.array_equal(got.view(np.uint8), want.view(np.uint8)), n
    for rows, cols in ((6, 1000), (3, 100_003)):
        m = np.full((rows, cols), -0.0, dtype=dt)
        m[1, cols // 3] = 2.0
        got = KI.scan_rows(_to_dev(m.reshape(-1), dev).view(rows, cols), "+").cpu().numpy()
        want = np.stack([oracle.accumulate("+", m[r]) for r in range(rows)]).astype(got.dtype)
        assert np.array_equal(got.view(np.uint8), want.view(np.uint8)), (rows, cols)
    KI.context(0).check()


@pytest.mark.parametrize("dt", [np.int8, np.uint8, np.int16, np.uint16], ids=lambda d: np.dtype(d).name)
def test_scan_narrow_same_type_misaligned(KI, oracle, dev, dt):
    """1- and 2-byte scans that keep their type (lane-wise words inside the kernel) from inputs and
    into outputs that are not 16-byte aligned, inclusive and exclusive, with and without init."""
    import torch

    n = 2 * 126976 + 37  # two full 1-byte tiles and a partial one
    for off in (1, 3):
        for op in ("|", "&", "xor", "max", "min"):
            x = _data(dt, n + off, 11 + off, op)
            xs = _to_dev(x, dev)[off:]
            for excl in (False, True):
                for init in (None, 3):
                    out = torch.empty(n + off, dtype=xs.dtype, device=dev)[off:]
                    got = KI.scan(xs, op, exclusive=excl, init=init, out=out).cpu().numpy()
                    want = oracle.accumulate(op, x[off:], exclusive=excl, init=init)
                    assert np.array_equal(got, want.astype(got.dtype)), (op, excl, init, off)
    KI.context(0).check()


def test_scan_nan_and_extremes(KI, oracle, dev):
    x = np.array([1.0, np.nan, -np.inf, 2.0, -0.0, 0.0] * 7000, dtype=np.float32)
    xd = _to_dev(x, dev)
    for op in ("max", "min"):
        got = KI.scan(xd, op).cpu().numpy()
        _check(got, oracle.accumulate(op, x), x, op)
    # Int64 wrap-around and Int32 widening
    big = np.full(40000, np.iinfo(np.int64).max // 3, dtype=np.int64)
    assert np.array_equal(KI.scan(_to_dev(big, dev), "+").cpu().numpy(), oracle.accumulate("+", big))
    i32 = np.full(40000, np.iinfo(np.int32).max, dtype=np.int32)
    got = KI.scan(_to_dev(i32, dev), "+").cpu().numpy()
    assert got.dtype == np.int64 and np.array_equal(got, oracle.accumulate("+", i32))


@pytest.mark.parametrize("dt,op", _cases())
def test_reduce(KI, oracle, dev, dt, op):
    for k, n in enumerate([1, 7, 33, 4099, 1 << 16, (1 << 22) + 5]):
        x = _data(dt, n, 100 + k, op)
        got = KI.reduce(_to_dev(x, dev), op).cpu().numpy().reshape(1)
        want = np.array([oracle.reduce_op(op, x)])
        if np.dtype(dt).kind == "f" and op == "+":
            assert abs(float(got[0]) - float(want[0])) <= 1e-5 * math.log2(max(2, n)) * float(np.abs(x.astype(np.float64)).sum())
        elif np.dtype(dt).kind == "f" and op == "*":
            assert abs(float(got[0]) - float(want[0])) <= 1e-5 * math.log2(max(2, n)) * abs(float(want[0])) + 1e-300
        else:
            _check(got, want.astype(got.dtype), x, op)
    KI.context(0).check()


def test_reduce_empty_and_nan(KI, dev):
    import torch

    e = torch.empty(0, dtype=torch.float32, device=dev)
    assert KI.reduce(e, "+").item() == 0.0
    assert KI.reduce(e, "*").item() == 1.0
    assert KI.reduce(torch.empty(0, dtype=torch.uint8, device=dev), "*").item() == 1
    with pytest.raises(KI.KIArgumentError):
        KI.reduce(e, "max")
    for op in ("|", "&", "xor"):
        with pytest.raises(KI.KIArgumentError):
            KI.reduce(torch.empty(0, dtype=torch.int16, device=dev), op)
        with pytest.raises(KI.KIArgumentError):  # the bitwise operators take integers
            KI.reduce(torch.ones(8, dtype=torch.float64, device=dev), op)
    x = torch.tensor([1.0, float("nan"), 3.0] * 5000, dtype=torch.float64, device=dev)
    assert math.isnan(KI.reduce(x, "max").item()) and math.isnan(KI.reduce(x, "min").item())
    z = torch.tensor([-0.0, 0.0, -0.0], dtype=torch.float32, device=dev)
    assert math.copysign(1.0, KI.reduce(z, "max").item()) == 1.0
    assert math.copysign(1.0, KI.reduce(z, "min").item()) == -1.0


def test_scan_config_size_f32(KI, dev):
    """Float32 cumsum at n = 2^28 (uniform[0,1) from the device generator): within 1e-5*log2(n) of a
    Float64 scan, checked on the device in Float64."""
    import torch

    n = 1 << 28
    x = torch.empty(n, dtype=torch.float32, device=dev)
    KI.fill_uniform(x, seed=1)
    y = KI.scan(x, "+")
    ref = torch.cumsum(x.double(), 0)
    rel = ((y.double() - ref).abs() / ref.clamp_min(1e-30)).max().item()
    assert rel <= 1e-5 * 28, rel
    del x, y, ref
    torch.cuda.empty_cache()


ROW_SHAPES = [(1, 1), (3, 5), (1000, 33), (257, 2048), (7, 2049), (5, 100_003), (2, (1 << 21) + 5), (600, 4096)]


@pytest.mark.parametrize("dt,op", _cases())
def test_reduce_rows(KI, oracle, dev, dt, op):
    """Segmented reduce (one result per row), with padded rows (ld > cols) and unaligned starts."""
    for k, (rows, cols) in enumerate(ROW_SHAPES):
        for pad in (0, 3):
            ld = cols + pad
            flat = _data(dt, rows * ld + 1, 1000 + k, op)
            m = flat[1:].reshape(rows, ld) if pad else flat[: rows * ld].reshape(rows, ld)
            xd = _to_dev(flat, dev)
            view = (xd[1:] if pad else xd[: rows * ld]).view(rows, ld)[:, :cols]
            got = KI.reduce_rows(view, op).cpu().numpy()
            for r in range(rows) if rows <= 64 else range(0, rows, max(1, rows // 64)):
                want = np.array([oracle.reduce_op(op, m[r, :cols])])
                g = got[r:r + 1]
                if np.dtype(dt).kind == "f" and op == "+":
                    bound = 1e-5 * math.log2(max(2, cols)) * float(np.abs(m[r, :cols].astype(np.float64)).sum())
                    assert abs(float(g[0]) - float(want[0])) <= bound, (rows, cols, r)
                elif np.dtype(dt).kind == "f" and op == "*":
                    bound = 1e-5 * math.log2(max(2, cols)) * abs(float(want[0])) + 1e-300
                    assert abs(float(g[0]) - float(want[0])) <= bound, (rows, cols, r)
                else:
                    _check(g, want.astype(g.dtype), m[r, :cols], op)
    KI.context(0).check()


def test_reduce_rows_empty_rows(KI, dev):
    import torch

    x = torch.empty((4, 0), dtype=torch.float32, device=dev)
    assert KI.reduce_rows(x, "+").tolist() == [0.0] * 4
    assert KI.reduce_rows(x, "*").tolist() == [1.0] * 4
    assert KI.reduce_rows(torch.empty((3, 0), dtype=torch.int8, device=dev), "*").tolist() == [1] * 3
    for op in ("max", "|"):
        with pytest.raises(KI.KIArgumentError):
            KI.reduce_rows(torch.empty((4, 0), dtype=torch.int32, device=dev), op)


SCAN_ROW_SHAPES = [(1, 5), (3, 1), (7, 33), (1000, 100), (300, 2049), (5, 8192), (40, 9000), (3, 100_003), (2, 400_001)]


@pytest.mark.parametrize("dt,op", [c for c in _cases() if c.values[1] == "+" or c.values[0] in (np.int8, np.int32, np.float64)])
def test_scan_rows(KI, oracle, dev, dt, op):
    """Segmented scan (accumulate along each row): short rows (one warp per row) and long rows (tiles
    with a lookback segment per row), padded rows (ld > cols), unaligned starts, exclusive with init."""
    import torch

    for k, (rows, cols) in enumerate(SCAN_ROW_SHAPES):
        for pad, excl in ((0, False), (3, True)):
            ld = cols + pad
            flat = _data(dt, rows * ld + 1, 2000 + k, op)
            m = flat[1:].reshape(rows, ld) if pad else flat[: rows * ld].reshape(rows, ld)
            xd = _to_dev(flat, dev)
            view = (xd[1:] if pad else xd[: rows * ld]).view(rows, ld)[:, :cols]
            init = None if not excl else (3 if np.dtype(dt).kind != "f" else 0.5)
            got = KI.scan_rows(view, op, exclusive=excl, init=init).cpu().numpy()
            for r in range(rows) if rows <= 40 else range(0, rows, max(1, rows // 40)):
                want = oracle.accumulate(op, m[r, :cols], init=init, exclusive=excl)
                x = m[r, :cols] if not excl else np.concatenate([[0], m[r, :cols][:-1]]).astype(m.dtype)
                _check(got[r], want, x, op)
    KI.context(0).check()


def test_scan_rows_strided_output_and_in_place(KI, oracle, dev):
    import torch

    x = _data(np.int64, 64 * 5000, 77, "+").reshape(64, 5000)
    xd = _to_dev(x, dev)
    out = torch.zeros(64, 5008, dtype=torch.int64, device=dev)
    KI.scan_rows(xd, "+", out=out[:, 3:5003])
    got = out.cpu().numpy()
    for r in range(64):
        assert np.array_equal(got[r, 3:5003], oracle.accumulate("+", x[r]))
    assert not got[:, :3].any() and not got[:, 5003:].any()
    y = xd.clone()
    KI.scan_rows(y, "max", out=y)
    for r in range(0, 64, 7):
        assert np.array_equal(y[r].cpu().numpy(), oracle.accumulate("max", x[r]))
    with pytest.raises(KI.KIArgumentError):  # rows overlapping another layout
        KI.scan_rows(xd[:, :4000], "+", out=xd[:, 1000:])
    KI.context(0).check()


@pytest.mark.parametrize("dt", NP_TYPES, ids=lambda d: np.dtype(d).name)
@pytest.mark.parametrize("f", ["abs", "abs2"])
def test_mapreduce(KI, oracle, dev, dt, f):
    """mapreduce(f, op, x) for f in abs, abs2 and op in +, max, min: the map in the element type (integer
    wrap-around included), then Base's reduce."""
    for k, n in enumerate([1, 33, 4099, (1 << 20) + 7]):
        x = _data(dt, n, 300 + k, "+")  # finite floats: a float sum of abs / abs2 stays finite
        xd = _to_dev(x, dev)
        for op in ("+", "max", "min"):
            got = KI.mapreduce(f, op, xd).cpu().numpy().reshape(1)
            want = np.array([oracle.mapreduce_op(f, op, x)])
            if np.dtype(dt).kind == "f" and op == "+":
                scale = float(np.abs(oracle.apply_map(f, x).astype(np.float64)).sum())
                assert abs(float(got[0]) - float(want[0])) <= 1e-5 * math.log2(max(2, n)) * scale, (n, op)
            else:
                _check(got, want.astype(got.dtype), x, op)
    with pytest.raises(KI.KIArgumentError):
        KI.mapreduce(f, "*", _to_dev(_data(dt, 10, 1), dev))
    KI.context(0).check()
