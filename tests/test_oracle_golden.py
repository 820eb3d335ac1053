"""CPU: the oracle reproduces the reference's own known answers and Julia Base semantics."""
from __future__ import annotations

import struct

import numpy as np
import pytest


def test_shfl_golden(oracle, golden):
    for c in golden["shfl"]:
        got = oracle.shfl(c["dir"], c["input"], c["arg"])
        assert got == c["expected"], c["name"]


def test_shfl_struct_golden(oracle, golden):
    # whole values move together, so shuffling indices is enough for the oracle
    for c in golden["shfl_struct"]:
        got = oracle.shfl(c["dir"], [tuple(v) for v in c["input"]], c["arg"])
        assert [list(v) for v in got] == c["expected"], c["name"]


def test_warpreduce_golden(oracle, golden):
    for c in golden["warp"]:
        if "expected" in c:
            got = oracle.warpreduce(c["input"], lambda a, b: a + b)
            assert got == c["expected"], c["name"]
        else:
            got = oracle.warpfold_down(c["input"], lambda a, b: a + b)
            assert got[0] == c["expected_lane1"], c["name"]


def test_warpfold_down_only_lane1_is_total(oracle):
    v = list(range(1, 33))
    got = oracle.warpfold_down(v, lambda a, b: a + b)
    assert got[0] == 528
    assert got[31] != 528  # the top lanes re-add their own value (src/warp.jl:35-37)


def test_vote_golden(oracle, golden):
    for c in golden["vote"]:
        preds = [x > c["threshold"] for x in c["input"]]
        got = oracle.vote(c["mode"], preds)
        assert [bool(g) for g in got] == c["expected"], c["name"]
    assert oracle.vote("ballot", [True] * 32)[0] == 0xFFFFFFFF
    assert oracle.vote("ballot", [l % 2 == 1 for l in range(32)])[0] == 0xAAAAAAAA


def test_generate_partN_golden(oracle, golden):
    for p in golden["patterns"]:
        assert oracle.generate_partN(p["N"])[p["residue"]] == tuple(p["pattern"])
    for N in (1, 2, 4, 8, 16, 32):
        for r, pat in enumerate(oracle.generate_partN(N)):
            assert sum(pat) == N
            pos = r
            for piece in pat:
                assert pos % piece == 0 or piece == 1  # naturally aligned
                if r:
                    assert piece <= max(N // 2, 1)
                pos = (pos + piece) % N


def test_generate_partN_matches_package(oracle):
    import kernelintrinsics as KI

    for N in (1, 2, 4, 8, 16, 64):
        assert KI.generate_partN(N) == oracle.generate_partN(N)


def test_vload_multi_golden(oracle, golden):
    for c in golden["vector"]:
        if c["op"] != "vload" or c["rebase"] or c["nitem"] != 16:
            continue
        pieces = oracle.vload_multi_pieces(0, c["index_1based"], 16)
        elems = [e for start, ln in pieces for e in range(start, start + ln)]
        assert [c["array"][e - 1] for e in elems] == c["expected"], c["name"]


def test_generators_known_answer(oracle):
    # splitmix64 reference value: the first output of a generator seeded with 0
    assert oracle.rand64(0, 0) == 0xE220A8397B1DCDAF
    x = oracle.gen_uniform_f32(1, 1 << 16)
    assert x.min() >= 0 and x.max() < 1
    assert np.all(x * 2**24 == np.floor(x * 2**24))
    y = oracle.gen_int_range_i64(3, -1000, 1000, 1 << 16)
    assert y.min() == -1000 and y.max() == 1000
    b = oracle.gen_bytes(2, 64)
    w = oracle.rand64(2, 0)
    assert bytes(b[:8]) == struct.pack("<Q", w)


def test_e4m3_codec(oracle):
    t = oracle.e4m3_decode_table()
    assert t[0x7E] == 448 and np.isnan(t[0x7F]) and t[0x01] == 2.0**-9 and t[0x08] == 2.0**-6
    for i in range(256):
        if i in (0x7F, 0xFF):
            continue
        assert oracle.e4m3_encode(t[i]) == i
    assert oracle.e4m3_encode(1000.0) == 0x7E and oracle.e4m3_encode(-1000.0) == 0xFE
    assert oracle.e4m3_encode(1.0625) == oracle.e4m3_encode(1.0)      # tie to even
    assert oracle.e4m3_encode(1.1875) == oracle.e4m3_encode(1.25)     # tie to even


def test_e4m3_generator_range(oracle):
    q = oracle.gen_e4m3_uniform(5, 112.0, 1 << 16)
    v = oracle.e4m3_decode_table()[q]
    assert np.abs(v).max() <= 112 and np.isfinite(v).all()


def test_base_semantics_sum(oracle, base_semantics):
    s = oracle.sum_f32(base_semantics["sum_x"])
    assert abs(s - base_semantics["sum_f64"][0]) <= 1e-12 * abs(s)


def test_base_semantics_cumsum(oracle, base_semantics):
    assert np.array_equal(oracle.cumsum_i64(base_semantics["scan_x"]), base_semantics["scan_y"])
    assert np.array_equal(oracle.cumsum_i64(base_semantics["wrap_x"]), base_semantics["wrap_y"])
    for nt in (1, 3, 8):
        assert np.array_equal(oracle.cumsum_i64(base_semantics["scan_x"], nthreads=nt), base_semantics["scan_y"])


def test_base_semantics_filter(oracle, base_semantics):
    v, i = oracle.filter_gt_f32(base_semantics["filt_x"], 0.5)
    assert np.array_equal(v, base_semantics["filt_vals"])
    assert np.array_equal(i, base_semantics["filt_idx1"])
    v0, i0 = oracle.filter_gt_f32(np.zeros(0, np.float32), 0.5)
    assert v0.size == 0 and i0.size == 0


def test_copy_and_gemm_oracle(oracle):
    src = oracle.gen_bytes(9, 1000)
    dst = np.zeros(1000, np.uint8)
    oracle.copy_bytes(dst, src)
    assert np.array_equal(src, dst)
    A = oracle.gen_e4m3_uniform(5, 112.0, 64 * 48).reshape(64, 48)
    B = oracle.gen_e4m3_uniform(6, 112.0, 48 * 40).reshape(48, 40)
    lut = oracle.e4m3_decode_table().astype(np.float64)
    ref = lut[A] @ lut[B]
    got = oracle.gemm_e4m3_rows(A, B, 0, 64)
    assert np.allclose(got, ref, rtol=0, atol=1e-9)
    assert np.allclose(oracle.gemm_e4m3_rows(A, B, 10, 20, scale=0.5), 0.5 * ref[10:20])


def test_accumulate_matches_scalar_base_semantics(oracle):
    """The vectorised Base restatement against a scalar loop of Base.max / Base.min / + on special values."""
    import math

    def jmax(a, b):
        if math.isnan(a):
            return a
        if math.isnan(b):
            return b
        if a == b:
            return b if math.copysign(1.0, a) < 0 else a
        return a if a > b else b

    def jmin(a, b):
        if math.isnan(a):
            return a
        if math.isnan(b):
            return b
        if a == b:
            return a if math.copysign(1.0, a) < 0 else b
        return a if a < b else b

    rng = np.random.default_rng(5)
    pool = np.array([0.0, -0.0, 1.5, -2.0, np.inf, -np.inf, np.nan, 3.25], dtype=np.float64)
    for dt in (np.float32, np.float64):
        x = pool[rng.integers(0, pool.size, 200)].astype(dt)
        for op, f in (("max", jmax), ("min", jmin)):
            got = oracle.accumulate(op, x)
            acc = float(x[0])
            for i in range(x.size):
                acc = float(x[0]) if i == 0 else f(acc, float(x[i]))
                g = float(got[i])
                assert (math.isnan(g) and math.isnan(acc)) or (g == acc and math.copysign(1, g) == math.copysign(1, acc))
    i32 = np.array([2**31 - 1, 2**31 - 1, -5], dtype=np.int32)
    assert oracle.accumulate("+", i32).tolist() == [2**31 - 1, 2**32 - 2, 2**32 - 7]
    i64 = np.array([2**63 - 1, 1], dtype=np.int64)
    assert oracle.accumulate("+", i64).tolist() == [2**63 - 1, -2**63]
    assert oracle.accumulate("+", np.array([1, 2, 3], dtype=np.int64), init=10, exclusive=True).tolist() == [10, 11, 13]
    assert oracle.reduce_op("+", np.zeros(0, dtype=np.int32)) == 0


def test_float_sums_keep_negative_zeros(oracle):
    """Base: cumsum([-0.0, -0.0]) == [-0.0, -0.0] and sum([-0.0, -0.0]) === -0.0 (the first element starts
    the fold, no +0.0 is added), while the sum of an empty collection is +0.0 (zero(T))."""
    for dt in (np.float32, np.float64):
        z = np.full(7, -0.0, dtype=dt)
        assert np.signbit(oracle.accumulate("+", z)).all()
        assert np.signbit(oracle.reduce_op("+", z))
        mixed = oracle.accumulate("+", np.array([-0.0, -0.0, 2.0, -0.0], dtype=dt))
        assert np.signbit(mixed).tolist() == [True, True, False, False]
        empty = oracle.reduce_op("+", np.zeros(0, dtype=dt))
        assert empty == 0 and not np.signbit(empty)


def test_accumulate_products_bitwise_and_small_integers(oracle):
    """cumprod / accumulate(|, &, xor) and the widening of Int8/Int16/UInt8/UInt16 (Base.add_sum and
    Base.mul_prod widen them to 64 bits; the bitwise operators keep the type), against scalar loops
    in Python integers reduced modulo 2^64."""
    rng = np.random.default_rng(11)

    def wrap(v, signed):
        v &= (1 << 64) - 1
        return v - (1 << 64) if signed and v >= 1 << 63 else v

    for dt in (np.int8, np.uint8, np.int16, np.uint16, np.int32, np.uint32, np.int64, np.uint64):
        info = np.iinfo(dt)
        x = rng.integers(info.min, info.max, 300, dtype=dt, endpoint=True)
        signed = info.min < 0
        for op in ("+", "*"):
            got = oracle.accumulate(op, x)
            assert got.dtype == (np.int64 if signed else np.uint64)
            acc = 0 if op == "+" else 1
            for i, v in enumerate(x.tolist()):
                acc = wrap(acc + v if op == "+" else acc * v, signed)
                assert int(got[i]) == acc, (dt, op, i)
        for op, f in (("|", lambda a, b: a | b), ("&", lambda a, b: a & b), ("xor", lambda a, b: a ^ b)):
            got = oracle.accumulate(op, x)
            assert got.dtype == np.dtype(dt)
            acc = int(x[0])
            for i, v in enumerate(x.tolist()):
                acc = v if i == 0 else f(acc, v)
                assert int(got[i]) == acc, (dt, op, i)
            ex = oracle.accumulate(op, x, exclusive=True)
            assert int(ex[0]) == int(oracle.identity(op, dt)) and np.array_equal(ex[1:], got[:-1])
    assert oracle.reduce_op("*", np.zeros(0, dtype=np.int8)) == 1
    assert oracle.identity("&", np.uint16) == 0xFFFF and oracle.identity("&", np.int16) == -1
    f = np.array([1.5, -2.0, 0.25], dtype=np.float32)
    assert oracle.accumulate("*", f).tolist() == [1.5, -3.0, -0.75]
    assert oracle.accumulate("*", f, init=2.0, exclusive=True).tolist() == [2.0, 3.0, -6.0]
    with pytest.raises(ValueError):
        oracle.reduce_op("|", np.zeros(0, dtype=np.int32))
    with pytest.raises(ValueError):
        oracle.accumulate("xor", f)


def test_maps_follow_base_integer_semantics(oracle):
    """abs(typemin) == typemin, abs2 wraps in the element type, abs is the identity on unsigned;
    filter_pred keeps the original elements."""
    i8 = np.array([-128, -3, 5, 127], dtype=np.int8)
    assert oracle.apply_map("abs", i8).tolist() == [-128, 3, 5, 127]
    assert oracle.apply_map("abs2", i8).tolist() == [0, 9, 25, 1]
    i16 = np.array([300, -200], dtype=np.int16)
    assert oracle.apply_map("abs2", i16).tolist() == [(90000 + 32768) % 65536 - 32768, (40000 + 32768) % 65536 - 32768]
    u8 = np.array([200, 3], dtype=np.uint8)
    assert oracle.apply_map("abs", u8).tolist() == [200, 3]
    v, i = oracle.filter_pred(np.array([-3.0, 1.0, 2.5, -0.5], dtype=np.float32), ">", 1.5, f="abs")
    assert v.tolist() == [-3.0, 2.5] and i.tolist() == [1, 3]
    assert oracle.mapreduce_op("abs2", "+", np.array([3, -4], dtype=np.int32)) == 25
