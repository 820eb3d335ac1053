"""CPU oracle for the KernelIntrinsics B200 primitives.

TEST INFRASTRUCTURE ONLY.  Only the test-suite, ``__graft_entry__.smoke()`` and the
CPU-baseline leg of ``bench.py`` import this module, and only as the checker.  The
product package never imports it.

Two layers:

* ``libki_oracle.so`` (``ki_oracle.c``) -- bulk restatements in C with pthreads:
  the splitmix64 generators, the e4m3 codec, Float64 sum, Int64 cumsum,
  filter/findall, byte copy and a Float64 GEMM of dequantised e4m3 operands.
* pure-Python restatements of the warp-level intrinsics on one 32-lane warp,
  following the reference line by line (small cases only):

  - ``shfl``           src/warp.jl:114-158 and ext/CUDA/shuffle_vote.jl:5-21
  - ``warpreduce``     src/warp.jl:226-237  (inclusive scan, Up, 1-based lane > offset)
  - ``warpfold``       src/warp.jl:273-282  (Down fold; lane 1 holds the total)
  - ``vote``           ext/CUDA/shuffle_vote.jl:23-34 (vote.sync semantics; ballot is UInt32)
  - ``generate_partN`` src/vectorization.jl:306-338
  - ``vload_multi``    src/vectorization.jl:365-379 (mod selects the piece pattern)

* numpy restatements of the device-wide reduce and scan for +, max and min (``accumulate``,
  ``reduce_op``) with Julia Base semantics: widening small-integer sums, wrapping Int64 sums,
  NaN-propagating max/min with -0.0 < +0.0.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "_build" / "libki_oracle.so"
WARP = 32

_lib = None


def build() -> Path:
    """Compile the C oracle with its Makefile (gcc, seconds)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        L = ctypes.CDLL(str(LIB_PATH))
        u64, i64, sz, vp, i32 = ctypes.c_uint64, ctypes.c_int64, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_int
        L.ko_mix64.restype = u64
        L.ko_mix64.argtypes = [u64]
        L.ko_rand64.restype = u64
        L.ko_rand64.argtypes = [u64, u64]
        L.ko_default_threads.restype = i32
        L.ko_gen_uniform_f32.argtypes = [u64, vp, sz, i32]
        L.ko_gen_int_range_i64.argtypes = [u64, i64, i64, vp, sz, i32]
        L.ko_gen_bytes.argtypes = [u64, vp, sz, i32]
        L.ko_gen_e4m3_uniform.argtypes = [u64, ctypes.c_float, vp, sz, i32]
        L.ko_e4m3_decode.restype = ctypes.c_float
        L.ko_e4m3_decode.argtypes = [ctypes.c_uint8]
        L.ko_e4m3_encode.restype = ctypes.c_uint8
        L.ko_e4m3_encode.argtypes = [ctypes.c_float]
        L.ko_sum_f32.restype = ctypes.c_double
        L.ko_sum_f32.argtypes = [vp, sz, i32]
        L.ko_sum_i64.restype = i64
        L.ko_sum_i64.argtypes = [vp, sz, i32]
        L.ko_cumsum_i64.argtypes = [vp, vp, sz, i64, i32]
        L.ko_filter_gt_f32.restype = sz
        L.ko_filter_gt_f32.argtypes = [vp, sz, ctypes.c_float, vp, vp, i64, i32]
        L.ko_copy_bytes.argtypes = [vp, vp, sz, i32]
        L.ko_gemm_e4m3_rows.argtypes = [vp, vp, vp, i32, i32, i32, i32, ctypes.c_double, i32]
        L.ko_generate_partN.restype = i32
        L.ko_generate_partN.argtypes = [i32, i32, ctypes.POINTER(ctypes.c_int)]
        _lib = L
    return _lib


def _ptr(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


def threads() -> int:
    return int(lib().ko_default_threads())


# ---------------------------------------------------------------------------
# generators
# ---------------------------------------------------------------------------

def rand64(seed: int, i: int) -> int:
    return int(lib().ko_rand64(seed, i))


def gen_uniform_f32(seed: int, n: int, nthreads: int = 0) -> np.ndarray:
    out = np.empty(n, dtype=np.float32)
    lib().ko_gen_uniform_f32(seed, _ptr(out), n, nthreads)
    return out


def gen_int_range_i64(seed: int, lo: int, hi: int, n: int, nthreads: int = 0) -> np.ndarray:
    out = np.empty(n, dtype=np.int64)
    lib().ko_gen_int_range_i64(seed, lo, hi, _ptr(out), n, nthreads)
    return out


def gen_bytes(seed: int, n: int, nthreads: int = 0) -> np.ndarray:
    out = np.empty(n, dtype=np.uint8)
    lib().ko_gen_bytes(seed, _ptr(out), n, nthreads)
    return out


def gen_e4m3_uniform(seed: int, scale: float, n: int, nthreads: int = 0) -> np.ndarray:
    out = np.empty(n, dtype=np.uint8)
    lib().ko_gen_e4m3_uniform(seed, scale, _ptr(out), n, nthreads)
    return out


def gen_normal_f32_host(seed: int, n: int) -> np.ndarray:
    """Standard normals for CPU-only runs (Box-Muller on the splitmix64 uniforms).

    The GPU parity tests do not need host/device identical normals: they copy the
    device input back and run the oracle on exactly those floats.
    """
    m = (n + 1) // 2
    idx = np.arange(m, dtype=np.uint64)
    r1 = _np_rand64(seed, 2 * idx)
    r2 = _np_rand64(seed, 2 * idx + np.uint64(1))
    u1 = ((r1 >> np.uint64(40)).astype(np.float64) + 1.0) * 2.0**-24
    u2 = (r2 >> np.uint64(40)).astype(np.float64) * 2.0**-24
    rad = np.sqrt(-2.0 * np.log(u1))
    z = np.empty(2 * m, dtype=np.float64)
    z[0::2] = rad * np.cos(2.0 * np.pi * u2)
    z[1::2] = rad * np.sin(2.0 * np.pi * u2)
    return z[:n].astype(np.float32)


def _np_rand64(seed: int, i: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):
        z = np.uint64(seed) + (i + np.uint64(1)) * np.uint64(0x9E3779B97F4A7C15)
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        return z ^ (z >> np.uint64(31))


# ---------------------------------------------------------------------------
# e4m3
# ---------------------------------------------------------------------------

def e4m3_decode_table() -> np.ndarray:
    return np.array([lib().ko_e4m3_decode(i) for i in range(256)], dtype=np.float32)


def e4m3_encode(x: float) -> int:
    return int(lib().ko_e4m3_encode(float(x)))


# ---------------------------------------------------------------------------
# device-wide operations (Julia Base semantics)
# ---------------------------------------------------------------------------

def sum_f32(x: np.ndarray, nthreads: int = 0) -> float:
    x = np.ascontiguousarray(x, dtype=np.float32)
    return float(lib().ko_sum_f32(_ptr(x), x.size, nthreads))


def sum_i64(x: np.ndarray, nthreads: int = 0) -> int:
    x = np.ascontiguousarray(x, dtype=np.int64)
    return int(lib().ko_sum_i64(_ptr(x), x.size, nthreads))


def cumsum_i64(x: np.ndarray, seed: int = 0, nthreads: int = 0) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.int64)
    y = np.empty_like(x)
    lib().ko_cumsum_i64(_ptr(x), _ptr(y), x.size, seed, nthreads)
    return y


# ---------------------------------------------------------------------------------------------
# Device-wide reduce / scan for +, *, max, min, |, &, xor (the device-wide uses of @warpfold and
# @warpreduce, src/warp.jl:273-282 and :226-237, which take any operator): Julia Base semantics of
# sum / prod / maximum / minimum / reduce(op, x) and cumsum / cumprod / accumulate(op, x; init).
#   * + and *  integers narrower than 64 bits widen to Int64 / UInt64 (Base.add_sum, Base.mul_prod),
#          64-bit integers wrap, floats in Float64 (the device's Float32 result is compared within a
#          tolerance);
#   * max  NaN wins, +0.0 > -0.0 (Base.max); min: NaN wins, -0.0 < +0.0 (Base.min);
#   * |, &, xor  integers, in their own type.
# ---------------------------------------------------------------------------------------------
_BITWISE = {"|": np.bitwise_or, "&": np.bitwise_and, "xor": np.bitwise_xor}


def result_dtype(dtype, op: str):
    dtype = np.dtype(dtype)
    if op in ("+", "*"):
        if dtype.kind == "f":
            return np.dtype(np.float64)
        if dtype.itemsize < 8:
            return np.dtype(np.int64 if dtype.kind == "i" else np.uint64)
    return dtype


def identity(op: str, dtype):
    """The operator's identity in the result type (what an exclusive scan starts from)."""
    rd = result_dtype(dtype, op)
    if op in ("+", "|", "xor"):
        return rd.type(0)
    if op == "*":
        return rd.type(1)
    if op == "&":
        return rd.type(-1) if rd.kind == "i" else np.iinfo(rd).max
    if rd.kind == "f":
        return rd.type(-np.inf if op == "max" else np.inf)
    return np.iinfo(rd).min if op == "max" else np.iinfo(rd).max


def _float_keys(x: np.ndarray, op: str) -> np.ndarray:
    """Unsigned keys whose order is Base.isless with -0.0 < +0.0; NaN maps to the winning end."""
    bits_t = np.uint32 if x.dtype == np.float32 else np.uint64
    top = bits_t(1) << bits_t(8 * x.dtype.itemsize - 1)
    b = x.view(bits_t)
    k = np.where(b & top, ~b, b | top).astype(bits_t)
    nan = np.isnan(x)
    return np.where(nan, np.iinfo(bits_t).max if op == "max" else 0, k).astype(bits_t)


def _from_keys(k: np.ndarray, dtype, op: str) -> np.ndarray:
    bits_t = np.uint32 if np.dtype(dtype) == np.float32 else np.uint64
    top = bits_t(1) << bits_t(8 * np.dtype(dtype).itemsize - 1)
    nan_key = np.iinfo(bits_t).max if op == "max" else 0
    b = np.where(k & top, k & ~top, ~k).astype(bits_t)
    v = b.view(dtype).copy()
    v[k == nan_key] = np.nan
    return v


def accumulate(op: str, x: np.ndarray, init=None, exclusive: bool = False) -> np.ndarray:
    """accumulate(op, x; init) with Base semantics; exclusive shifts by one and starts at init."""
    x = np.ascontiguousarray(x)
    rd = result_dtype(x.dtype, op)
    if op in ("+", "*"):
        acc = np.cumsum if op == "+" else np.cumprod
        with np.errstate(over="ignore"):
            v = acc(x.astype(rd), dtype=rd)  # numpy wraps integer overflow like Base
            if init is not None:
                t = rd.type(init)
                v = (v + t if op == "+" else v * t).astype(rd)
    elif op in _BITWISE:
        if x.dtype.kind not in "iu":
            raise ValueError(f"{op} takes integers")
        seq = x if init is None else np.concatenate([np.array([init], dtype=x.dtype), x])
        v = _BITWISE[op].accumulate(seq)
        if init is not None:
            v = v[1:]
    elif x.dtype.kind == "f":
        keys = _float_keys(x, op)
        if init is not None:
            keys = np.concatenate([_float_keys(np.array([init], dtype=x.dtype), op), keys])
        acc = (np.maximum if op == "max" else np.minimum).accumulate(keys)
        if init is not None:
            acc = acc[1:]
        v = _from_keys(acc, x.dtype, op)
    else:
        seq = x if init is None else np.concatenate([np.array([init], dtype=x.dtype), x])
        v = (np.maximum if op == "max" else np.minimum).accumulate(seq)
        if init is not None:
            v = v[1:]
    if not exclusive:
        return v
    if init is None:
        init = identity(op, x.dtype)
    return np.concatenate([np.array([init], dtype=rd), v[:-1]])


def reduce_op(op: str, x: np.ndarray):
    """sum / prod / maximum / minimum / reduce(op, x) with Base semantics (an empty sum is 0, an empty
    product 1; the other operators raise on an empty collection)."""
    x = np.ascontiguousarray(x)
    if x.size == 0:
        if op in ("+", "*"):
            return identity(op, x.dtype)
        raise ValueError("reducing over an empty collection is not allowed")
    return accumulate(op, x)[-1]


def apply_map(f, x: np.ndarray) -> np.ndarray:
    """abs / abs2 in the element type, as Base computes them (integers wrap: abs(typemin) is typemin,
    abs2 is x*x modulo 2^bits; abs is the identity on unsigned types)."""
    x = np.ascontiguousarray(x)
    if f is None:
        return x
    with np.errstate(over="ignore"):
        if f == "abs":
            return x if x.dtype.kind == "u" else np.abs(x).astype(x.dtype)
        if f == "abs2":
            return (x * x).astype(x.dtype)
    raise ValueError(f)


def mapreduce_op(f, op: str, x: np.ndarray):
    """mapreduce(f, op, x): the map in the element type, then reduce_op."""
    return reduce_op(op, apply_map(f, x))


_CMP = {">": np.greater, ">=": np.greater_equal, "<": np.less, "<=": np.less_equal, "==": np.equal,
        "!=": np.not_equal}


def filter_pred(x: np.ndarray, pred: str, thr, f=None, index_base: int = 1):
    """filter(v -> f(v) pred thr, x) and findall (index_base-based Int32 indices): IEEE comparisons in
    the element type, order preserved, the kept elements x's own."""
    x = np.ascontiguousarray(x)
    keep = _CMP[pred](apply_map(f, x), x.dtype.type(thr))
    idx = np.nonzero(keep)[0]
    return x[idx], (idx + index_base).astype(np.int32)


def filter_gt_f32(x: np.ndarray, thr: float, index_base: int = 1, nthreads: int = 0):
    x = np.ascontiguousarray(x, dtype=np.float32)
    k = int(lib().ko_filter_gt_f32(_ptr(x), x.size, thr, None, None, index_base, nthreads))
    vals = np.empty(k, dtype=np.float32)
    idx = np.empty(k, dtype=np.int32)
    lib().ko_filter_gt_f32(_ptr(x), x.size, thr, _ptr(vals) if k else None, _ptr(idx) if k else None,
                           index_base, nthreads)
    return vals, idx


def copy_bytes(dst: np.ndarray, src: np.ndarray, nthreads: int = 0) -> None:
    assert dst.nbytes >= src.nbytes
    lib().ko_copy_bytes(_ptr(dst), _ptr(src), src.nbytes, nthreads)


def copy_2d(dst: np.ndarray, dpitch: int, src: np.ndarray, spitch: int, width: int, height: int,
            dst_offset: int = 0, src_offset: int = 0) -> None:
    """copyto! of a strided byte matrix, one row at a time: the element-by-element semantics of the
    reference's AbstractArray fallback (_vload_batch / _vstore_batch!, src/vectorization.jl:426-448)
    applied to bytes.  dst and src are 1-D uint8 arrays."""
    for r in range(height):
        d0, s0 = dst_offset + r * dpitch, src_offset + r * spitch
        dst[d0:d0 + width] = src[s0:s0 + width]


def copy_strided(dst: np.ndarray, dst_stride: int, src: np.ndarray, src_stride: int, count: int,
                 dst_start: int = 0, src_start: int = 0) -> None:
    """dst[dst_start + i*dst_stride] = src[src_start + i*src_stride] for i < count (element strides of
    either sign), in index order."""
    i = np.arange(count, dtype=np.int64)
    dst[dst_start + i * dst_stride] = src[src_start + i * src_stride]


def gemm_e4m3_rows(A: np.ndarray, B: np.ndarray, r0: int, r1: int, scale: float = 1.0,
                   nthreads: int = 0) -> np.ndarray:
    """Rows [r0, r1) of dec(A) @ dec(B) * scale in Float64 (A: MxK, B: KxN, row-major uint8)."""
    M, K = A.shape
    K2, N = B.shape
    assert K == K2 and 0 <= r0 <= r1 <= M
    A = np.ascontiguousarray(A, dtype=np.uint8)
    B = np.ascontiguousarray(B, dtype=np.uint8)
    C = np.empty((r1 - r0, N), dtype=np.float64)
    lib().ko_gemm_e4m3_rows(_ptr(A), _ptr(B), _ptr(C), r0, r1, N, K, scale, nthreads)
    return C


# ---------------------------------------------------------------------------
# vector access patterns
# ---------------------------------------------------------------------------

def generate_partN(N: int) -> tuple:
    """All N patterns, index r = alignment residue (src/vectorization.jl:306-338)."""
    out = []
    buf = (ctypes.c_int * 64)()
    for r in range(N):
        c = lib().ko_generate_partN(N, r, buf)
        assert c > 0
        out.append(tuple(buf[i] for i in range(c)))
    return tuple(out)


def vload_multi_pieces(base_elem_offset: int, i: int, N: int):
    """Pieces (start element, length) that vload_multi(a, i, Val(N)) issues.

    ``base_elem_offset`` is pointer(a) / sizeof(T); ``i`` is the 1-based start
    index (src/vectorization.jl:374-379): mod = (ptr/sizeof(T) + i-1) % N + 1 picks
    the pattern, which is laid out from element i.
    """
    mod = (base_elem_offset + i - 1) % N
    pat = generate_partN(N)[mod]
    pieces, off = [], 0
    for p in pat:
        pieces.append((i + off, p))
        off += p
    return pieces


# ---------------------------------------------------------------------------
# warp-level intrinsics on one warp of 32 lanes (values are Python ints/floats)
# ---------------------------------------------------------------------------

def shfl(direction: str, vals, src: int, width: int = WARP):
    """@shfl on one warp.  Lanes are 0-based positions in ``vals``.

    Up/Down: lanes whose source falls outside the warp keep their own value
    (shfl.sync clamp rule, src/warp.jl:21-37).  Xor: lane ^ src.  Idx: ``src`` is the
    1-based source lane, as CUDA.jl's shfl_sync takes it and as the reference's own
    tests and fallbacks use it (test/tests/shfl.jl:84-89, src/warp.jl:334,342).
    """
    out = list(vals)
    for lane in range(width):
        if direction == "up":
            s = lane - src
            out[lane] = vals[s] if s >= 0 else vals[lane]
        elif direction == "down":
            s = lane + src
            out[lane] = vals[s] if s < width else vals[lane]
        elif direction == "xor":
            s = lane ^ src
            out[lane] = vals[s] if s < width else vals[lane]
        elif direction == "idx":
            out[lane] = vals[(src - 1) % width]
        else:
            raise ValueError(direction)
    return out


def warpreduce(vals, op, width: int = WARP):
    """@warpreduce: inclusive Up-shuffle scan; 1-based lane combines iff lane > offset."""
    v = list(vals)
    offset = 1
    while offset < width:
        sh = shfl("up", v, offset, width)
        v = [op(sh[l], v[l]) if (l + 1) > offset else v[l] for l in range(width)]
        offset <<= 1
    return v


def warpfold_down(vals, op, width: int = WARP):
    """@warpfold exactly as written: Down shuffles, offsets 1..16; lane 1 holds the total."""
    v = list(vals)
    offset = 1
    while offset < width:
        sh = shfl("down", v, offset, width)
        v = [op(sh[l], v[l]) for l in range(width)]
        offset <<= 1
    return v


def vote(mode: str, preds):
    p = [bool(x) for x in preds]
    if mode == "all":
        return [all(p)] * len(p)
    if mode == "any":
        return [any(p)] * len(p)
    if mode == "uni":
        return [all(p) or not any(p)] * len(p)
    if mode == "ballot":
        b = 0
        for lane, x in enumerate(p):
            b |= int(x) << lane
        return [b] * len(p)
    raise ValueError(mode)
