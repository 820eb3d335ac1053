"""KernelIntrinsics for B200: the host-side mirror of KernelIntrinsics.jl's API over libki_b200.so.

Names and argument meanings follow the reference (epilliat/KernelIntrinsics.jl v0.1.6):

* type lattices ``Workgroup/Device/System``, ``Weak/Volatile/Relaxed/Acquire/Release/AcqRel/SeqCst``
  (src/scopes_orderings.jl:13-120), ``Up/Down/Xor/Idx`` and ``All/AnyLane/Uni/Ballot``
  (src/warp.jl:16-106);
* ``shfl``, ``warpreduce``, ``warpfold``, ``vote`` run the warp intrinsics over every warp of a CUDA
  tensor (lanes are consecutive elements); ``Idx`` lanes and ``laneid`` are 1-based as in Julia;
* ``vload`` / ``vstore`` / ``vload_multi`` / ``vstore_multi`` take 1-based indices;
* ``access`` / ``fence`` validate scope/ordering like ``@access`` / ``@fence`` and raise
  ``KIArgumentError`` (a ``ValueError``) where the reference raises ``ArgumentError``;
* device-wide operations built from them: ``vcopy`` (copyto!), ``warpfold_reduce`` (sum),
  ``warpreduce_scan`` (cumsum), ``vote_compact`` (filter/findall), ``fp8_gemm``.

Every operation runs a hand-written sm_100a kernel from libki_b200.so; tensors are torch CUDA tensors
(torch provides device memory and streams only).  There is no CPU path.
"""
from __future__ import annotations

import ctypes
import threading
from typing import Optional

from . import _abi
from ._abi import KIArgumentError, KIError, KITimeoutError

__all__ = [
    "Workgroup", "Device", "System", "Weak", "Volatile", "Relaxed", "Acquire", "Release", "AcqRel", "SeqCst",
    "Up", "Down", "Xor", "Idx", "All", "AnyLane", "Uni", "Ballot", "KIError", "KIArgumentError",
    "KITimeoutError", "Context", "context", "warpsize", "get_warpsize", "devices", "shfl", "warpreduce",
    "warpfold", "vote", "vload", "vstore", "vload_multi", "vstore_multi", "generate_partN", "access",
    "message_pass", "vcopy", "vcopy_host", "reduce", "reduce_rows", "scan", "compact", "warpfold_reduce", "reduce_sum_i64", "warpreduce_scan", "warpreduce_scan_host", "vote_compact",
    "fp8_gemm", "fill_uniform", "fill_int_range", "fill_bytes", "fill_normal", "fill_e4m3_uniform",
]


# ---------------------------------------------------------------------------------------------
# type lattices (singletons, used like the reference's types)
# ---------------------------------------------------------------------------------------------
class Scope:
    key = "default"


class Workgroup(Scope):
    key = "workgroup"


class Device(Scope):
    key = "device"


class System(Scope):
    key = "system"


class Ordering:
    key = "default"


class Weak(Ordering):
    key = "weak"


class Volatile(Ordering):
    key = "volatile"


class Relaxed(Ordering):
    key = "relaxed"


class Acquire(Ordering):
    key = "acquire"


class Release(Ordering):
    key = "release"


class AcqRel(Ordering):
    key = "acqrel"


class SeqCst(Ordering):
    key = "seqcst"


class Direction:
    key = ""


class Up(Direction):
    key = "up"


class Down(Direction):
    key = "down"


class Xor(Direction):
    key = "xor"


class Idx(Direction):
    key = "idx"


class Mode:
    key = ""


class All(Mode):
    key = "all"


class AnyLane(Mode):
    key = "any"


class Uni(Mode):
    key = "uni"


class Ballot(Mode):
    key = "ballot"


# ---------------------------------------------------------------------------------------------
# context
# ---------------------------------------------------------------------------------------------
def _torch():
    import torch

    return torch


class Context:
    """One libki_b200 context (scratch + device status word) on one device (0-based ``device``)."""

    def __init__(self, device: int = 0):
        self.lib = _abi.load()
        h = ctypes.c_void_p()
        st = self.lib.ki_ctx_create(int(device), ctypes.byref(h))
        if st != _abi.KI_OK:
            raise _abi.status_error(st, f"ki_ctx_create(device={device}): "
                                        f"{self.lib.ki_status_string(st).decode()}")
        self.handle = h
        self.device = int(device)

    def close(self) -> None:
        if getattr(self, "handle", None):
            self.lib.ki_ctx_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _raise(self, st: int, what: str) -> None:
        msg = self.lib.ki_last_error_string(self.handle).decode(errors="replace")
        raise _abi.status_error(st, f"{what}: {msg or self.lib.ki_status_string(st).decode()}")

    def call(self, name: str, *args) -> None:
        st = getattr(self.lib, name)(self.handle, *args)
        if st != _abi.KI_OK:
            self._raise(st, name)

    def check(self, stream=None) -> None:
        """Synchronise ``stream`` and raise if a bounded device-side wait of this context ran out."""
        st = self.lib.ki_ctx_check(self.handle, _stream_ptr(stream, self.device))
        if st != _abi.KI_OK:
            self._raise(st, "ki_ctx_check")

    def set_wait_timeout(self, seconds: float) -> None:
        self.call("ki_ctx_set_wait_timeout_ns", ctypes.c_uint64(int(seconds * 1e9)))


_ctx_lock = threading.Lock()
_ctx_by_key: dict = {}


def context(device: Optional[int] = None) -> Context:
    """The calling thread's context on ``device`` (default: torch's current device)."""
    torch = _torch()
    if device is None:
        device = torch.cuda.current_device()
    key = (threading.get_ident(), int(device))
    with _ctx_lock:
        c = _ctx_by_key.get(key)
        if c is None:
            c = Context(int(device))
            _ctx_by_key[key] = c
    return c


def _stream_ptr(stream, device: int):
    torch = _torch()
    if stream is None:
        stream = torch.cuda.current_stream(device)
    return ctypes.c_void_p(stream.cuda_stream)


def _dev(t) -> int:
    if not t.is_cuda:
        raise KIArgumentError(_abi.KI_ERR_ARG, "tensor must be on a CUDA device (there is no CPU path)")
    return t.device.index


def _ptr(t) -> ctypes.c_void_p:
    return ctypes.c_void_p(t.data_ptr())


def _dtype_code(t) -> int:
    name = str(t.dtype).replace("torch.", "")
    if name not in _abi.DTYPE:
        raise KIArgumentError(_abi.KI_ERR_ARG, f"unsupported dtype {t.dtype}")
    return _abi.DTYPE[name]


# ---------------------------------------------------------------------------------------------
# device queries (src/device.jl, ext/CUDA/device.jl): 1-based device ids as in the reference
# ---------------------------------------------------------------------------------------------
def devices() -> list:
    lib = _abi.load()
    n = ctypes.c_int(0)
    lib.ki_device_count(ctypes.byref(n))
    return list(range(1, n.value + 1))


def get_warpsize(device: int = 1) -> int:
    lib = _abi.load()
    ws = ctypes.c_int(0)
    st = lib.ki_device_info(int(device) - 1, None, ctypes.byref(ws), None, None)
    if st != _abi.KI_OK:
        raise _abi.status_error(st, "ki_device_info")
    return ws.value


warpsize = get_warpsize


# ---------------------------------------------------------------------------------------------
# warp intrinsics over whole warps
# ---------------------------------------------------------------------------------------------
def shfl(direction, x, src: int, out=None):
    """@shfl(direction, val, src) on every warp of ``x`` (x.numel() % 32 == 0).

    ``src``: offset for Up/Down, lane mask for Xor, 1-BASED source lane for Idx.  Works on any
    element type, including structured numpy-style records viewed as bytes (element size 1..64).
    """
    torch = _torch()
    d = _dev(x)
    out = torch.empty_like(x) if out is None else out
    arg = int(src)
    if direction is Idx:
        if not 1 <= arg <= 32:
            raise KIArgumentError(_abi.KI_ERR_ARG, "Idx lane must be in 1..32")
        arg -= 1
    esz = x.element_size()
    n = x.numel()
    if x.dim() >= 2 and x.dtype == torch.uint8:  # rows of raw bytes = one element per row
        esz = x.shape[-1]
        n = x.numel() // esz
    context(d).call("ki_warp_shfl", _abi.DIR[direction.key], _ptr(x), _ptr(out), esz, n, arg,
                    _stream_ptr(None, d))
    return out


def warpreduce(x, op: str = "+", out=None):
    """@warpreduce(val, op): inclusive scan inside each warp (src/warp.jl:226-237)."""
    torch = _torch()
    d = _dev(x)
    out = torch.empty_like(x) if out is None else out
    context(d).call("ki_warp_reduce", _abi.OP[op], _dtype_code(x), _ptr(x), _ptr(out), x.numel(),
                    _stream_ptr(None, d))
    return out


def warpfold(x, op: str = "+", form: str = "xor", out=None):
    """@warpfold(val, op).  form="down" is the reference's exact Down fold (lane 1 holds the total);
    form="xor" gives every lane the total."""
    torch = _torch()
    d = _dev(x)
    out = torch.empty_like(x) if out is None else out
    f = {"xor": 0, "down": 1}[form]
    context(d).call("ki_warp_fold", _abi.OP[op], _dtype_code(x), f, _ptr(x), _ptr(out), x.numel(),
                    _stream_ptr(None, d))
    return out


def vote(mode, pred, out=None):
    """@vote(mode, pred) on every warp; ``pred`` is a bool/uint8 tensor.  Returns uint32 per lane
    (0/1 for All/AnyLane/Uni; the UInt32 ballot mask for Ballot, bit i = 0-based lane i)."""
    torch = _torch()
    d = _dev(pred)
    p = pred.to(torch.uint8) if pred.dtype != torch.uint8 else pred
    out = torch.empty(p.shape, dtype=torch.uint32, device=p.device) if out is None else out
    context(d).call("ki_warp_vote", _abi.MODE[mode.key], _ptr(p), _ptr(out), p.numel(), _stream_ptr(None, d))
    return out


# ---------------------------------------------------------------------------------------------
# vector access (1-based indices, as the reference)
# ---------------------------------------------------------------------------------------------
def vload(a, idx: int, nitem: int, rebase: bool = True, elem_bytes: Optional[int] = None):
    """vload(A, idx, Val(N), Val(Rebase)) -> tensor of N elements (src/vectorization.jl:135-199).

    rebase=True: ``idx`` is a 1-based block index (elements (idx-1)*N+1 .. idx*N);
    rebase=False: ``idx`` is the 1-based first element.  ``elem_bytes`` views a uint8 tensor as
    records of that size (non power-of-two sizes take the scalar path)."""
    torch = _torch()
    d = _dev(a)
    esz = elem_bytes or a.element_size()
    out = torch.empty(nitem * esz, dtype=torch.uint8, device=a.device)
    context(d).call("ki_vload", _ptr(a), esz, int(idx) - 1, int(nitem), int(bool(rebase)), _ptr(out),
                    _stream_ptr(None, d))
    if elem_bytes is None:
        return out.view(a.dtype)
    return out.view(nitem, esz)


def vstore(a, idx: int, values, rebase: bool = True, elem_bytes: Optional[int] = None) -> None:
    """vstore!(A, idx, values, Val(Rebase)) (src/vectorization.jl:218-300)."""
    d = _dev(a)
    esz = elem_bytes or a.element_size()
    nitem = values.numel() * values.element_size() // esz
    context(d).call("ki_vstore", _ptr(a), esz, int(idx) - 1, int(nitem), int(bool(rebase)),
                    _ptr(values.contiguous()), _stream_ptr(None, d))


def vload_multi(a, i: int, nitem: int):
    """vload_multi(a, i, Val(N)): N elements from 1-based element i with the generate_partN pieces."""
    return vload(a, i, nitem, rebase=False)


def vstore_multi(a, i: int, values) -> None:
    """vstore_multi!(a, i, values)."""
    vstore(a, i, values, rebase=False)


def generate_partN(N: int) -> tuple:
    """The reference's piece patterns (src/vectorization.jl:306-338), index = residue (0-based)."""
    if N <= 0 or N & (N - 1):
        raise KIArgumentError(_abi.KI_ERR_ARG, "N must be a positive power of 2")
    out = [(N,)]
    for r in range(1, N):
        pat, remaining, pos = [], N, r
        while remaining > 0:
            m = N // 2
            while m > 0 and not (pos % m == 0 and m <= remaining):
                m //= 2
            m = max(m, 1)
            pat.append(m)
            remaining -= m
            pos = (pos + m) % N
        out.append(tuple(pat))
    return tuple(out)


# ---------------------------------------------------------------------------------------------
# @access / @fence
# ---------------------------------------------------------------------------------------------
def _split_scope_order(args):
    """scope_ordering (src/macros.jl:130-196): 0-2 arguments, one Scope and/or one Ordering, any order."""
    if len(args) > 2:
        raise KIArgumentError(_abi.KI_ERR_ARG, f"Too many arguments: expected 0-2, got {len(args)}.")
    scope = order = None
    for a in args:
        if isinstance(a, type) and issubclass(a, Scope) and a is not Scope and scope is None:
            scope = a
        elif isinstance(a, type) and issubclass(a, Ordering) and a is not Ordering and order is None:
            order = a
        else:
            raise KIArgumentError(_abi.KI_ERR_ARG, "Arguments must be one Scope and one Ordering (in any order).")
    return scope, order


def access(slot, value, *args, fence_args=()):
    """@access store of ``value`` into ``slot[0]``, @fence, then @access load back; returns the value.

    ``args`` are the @access scope/ordering for both accesses, e.g. ``access(t, 5, Device, Relaxed)``;
    the store ordering defaults to Release and the load to Acquire.  ``fence_args`` likewise for
    @fence (default Device, AcqRel)."""
    torch = _torch()
    d = _dev(slot)
    scope, order = _split_scope_order(args)
    fscope, forder = _split_scope_order(fence_args)
    so = lo = _abi.ORDER[order.key] if order else 0
    if order in (Acquire, Release):  # one explicit ordering applies to the access it names
        so = _abi.ORDER["release"] if order is Release else 0
        lo = _abi.ORDER["acquire"] if order is Acquire else 0
    val = torch.tensor([value], dtype=slot.dtype, device=slot.device)
    rb = torch.empty(1, dtype=slot.dtype, device=slot.device)
    context(d).call("ki_access_roundtrip", _dtype_code(slot), _abi.SCOPE[scope.key] if scope else 0, so, lo,
                    _abi.SCOPE[fscope.key] if fscope else 0, _abi.ORDER[forder.key] if forder else 0,
                    _ptr(slot), _ptr(val), _ptr(rb), _stream_ptr(None, d))
    return rb


def message_pass(data, flag, seen, payload: int, produce: bool = True, timeout_s: float = 1.0):
    """Release/acquire message passing across blocks (the reference's @access producer/consumer
    example, src/macros.jl:84-97) with bounded waits.  ``seen[b]`` gets the payload, or -1 if the
    wait of consumer block b ran out (then ``Context.check`` raises KITimeoutError)."""
    d = _dev(data)
    context(d).call("ki_flag_message_pass", _ptr(data), _ptr(flag), _ptr(seen), seen.numel(), int(payload),
                    int(bool(produce)), ctypes.c_uint64(int(timeout_s * 1e9)), _stream_ptr(None, d))


# ---------------------------------------------------------------------------------------------
# device-wide operations
# ---------------------------------------------------------------------------------------------
def vcopy(dst, src, nbytes: Optional[int] = None, dst_offset: int = 0, src_offset: int = 0, stream=None):
    """copyto!: copy ``nbytes`` bytes from ``src`` (+src_offset bytes) to ``dst`` (+dst_offset bytes)
    with 128-bit vector accesses at any alignment."""
    d = _dev(dst)
    if nbytes is None:
        nbytes = min(src.numel() * src.element_size() - src_offset, dst.numel() * dst.element_size() - dst_offset)
    if src_offset + nbytes > src.numel() * src.element_size() or dst_offset + nbytes > dst.numel() * dst.element_size():
        raise KIArgumentError(_abi.KI_ERR_ARG, "vcopy: range outside the tensors")
    context(d).call("ki_vcopy", ctypes.c_void_p(dst.data_ptr() + dst_offset),
                    ctypes.c_void_p(src.data_ptr() + src_offset), int(nbytes), _stream_ptr(stream, d))
    return dst


def vcopy_2d(dst, dpitch: int, src, spitch: int, width: int, height: int, dst_offset: int = 0, src_offset: int = 0,
             stream=None):
    """copyto! of ``height`` rows of ``width`` bytes: row r from byte src_offset + r*spitch of ``src`` to
    byte dst_offset + r*dpitch of ``dst`` (any alignment, any pitch >= width)."""
    d = _dev(dst)
    if width > 0 and height > 0:
        last_d = dst_offset + (height - 1) * dpitch + width
        last_s = src_offset + (height - 1) * spitch + width
        if min(dst_offset, src_offset) < 0 or last_d > dst.numel() * dst.element_size() or \
                last_s > src.numel() * src.element_size():
            raise KIArgumentError(_abi.KI_ERR_ARG, "vcopy_2d: range outside the tensors")
    context(d).call("ki_vcopy_2d", ctypes.c_void_p(dst.data_ptr() + dst_offset), int(dpitch),
                    ctypes.c_void_p(src.data_ptr() + src_offset), int(spitch), int(width), int(height),
                    _stream_ptr(stream, d))
    return dst


def vcopy_strided(dst, dst_stride: int, src, src_stride: int, count: int, dst_start: int = 0, src_start: int = 0,
                  elem_bytes: Optional[int] = None, stream=None):
    """dst[dst_start + i*dst_stride] = src[src_start + i*src_stride] for i < count, in elements of the
    tensors' (equal) element size, or of ``elem_bytes`` bytes (a struct type held in byte tensors);
    strides of either sign, as Julia's strided and reversed views."""
    d = _dev(dst)
    if elem_bytes is None:
        es = dst.element_size()
        if src.element_size() != es:
            raise KIArgumentError(_abi.KI_ERR_ARG, "vcopy_strided: element sizes differ")
    else:
        es = int(elem_bytes)
        if es <= 0:
            raise KIArgumentError(_abi.KI_ERR_ARG, "vcopy_strided: element size must be positive")
    if count > 0:
        for t, st, n0 in ((dst, dst_stride, dst_start), (src, src_stride, src_start)):
            last = n0 + (count - 1) * st
            if min(n0, last) < 0 or (max(n0, last) + 1) * es > t.numel() * t.element_size():
                raise KIArgumentError(_abi.KI_ERR_ARG, "vcopy_strided: range outside the tensors")
    context(d).call("ki_vcopy_strided", ctypes.c_void_p(dst.data_ptr() + dst_start * es), int(dst_stride),
                    ctypes.c_void_p(src.data_ptr() + src_start * es), int(src_stride), es, int(count),
                    _stream_ptr(stream, d))
    return dst


def copyto(dst, src, stream=None):
    """copyto!(dst, src) for device views of the same shape and element size: contiguous ranges go
    through vcopy, 1-D strided views through vcopy_strided, 2-D views with contiguous rows through
    vcopy_2d (one row per leading index)."""
    if tuple(dst.shape) != tuple(src.shape) or dst.element_size() != src.element_size():
        raise KIArgumentError(_abi.KI_ERR_ARG, "copyto: shapes or element sizes differ")
    es = dst.element_size()
    if dst.numel() == 0:
        return dst
    if dst.is_contiguous() and src.is_contiguous():
        return _copy_raw("ki_vcopy", dst, src, dst.numel() * es, stream)
    if dst.dim() == 1:
        return _copy_raw("ki_vcopy_strided", dst, src, dst.numel(), stream, dst.stride(0), src.stride(0), es)
    if dst.dim() == 2 and dst.stride(1) == 1 and src.stride(1) == 1:
        return _copy_raw("ki_vcopy_2d", dst, src, dst.shape[1] * es, stream, dst.stride(0) * es, src.stride(0) * es,
                         dst.shape[0])
    raise KIArgumentError(_abi.KI_ERR_ARG, "copyto: 1-D views, or 2-D views with contiguous rows")


def _copy_raw(fn, dst, src, n, stream, *extra):
    d = _dev(dst)
    pd, ps = ctypes.c_void_p(dst.data_ptr()), ctypes.c_void_p(src.data_ptr())
    s = _stream_ptr(stream, d)
    if fn == "ki_vcopy":
        context(d).call(fn, pd, ps, int(n), s)
    elif fn == "ki_vcopy_strided":
        dstride, sstride, es = extra
        context(d).call(fn, pd, int(dstride), ps, int(sstride), int(es), int(n), s)
    else:
        dpitch, spitch, height = extra
        context(d).call(fn, pd, int(dpitch), ps, int(spitch), int(n), int(height), s)
    return dst


def vcopy_host(dst, src, nbytes: Optional[int] = None, dst_offset: int = 0, src_offset: int = 0, device: int = 0,
               stream=None):
    """copyto! between two host (CPU) tensors through device ``device``: chunks go to the device, are
    copied by the vectorised copy kernel and come back, both directions overlapped.  Pinned host
    tensors make the call asynchronous; it is complete when ``stream`` is."""
    if dst.is_cuda or src.is_cuda:
        raise KIArgumentError(_abi.KI_ERR_ARG, "vcopy_host: host tensors expected")
    if nbytes is None:
        nbytes = min(src.numel() * src.element_size() - src_offset, dst.numel() * dst.element_size() - dst_offset)
    if src_offset + nbytes > src.numel() * src.element_size() or dst_offset + nbytes > dst.numel() * dst.element_size():
        raise KIArgumentError(_abi.KI_ERR_ARG, "vcopy_host: range outside the tensors")
    context(device).call("ki_vcopy_host", ctypes.c_void_p(dst.data_ptr() + dst_offset),
                         ctypes.c_void_p(src.data_ptr() + src_offset), int(nbytes), _stream_ptr(stream, device))
    return dst


def warpfold_reduce(x, out_f64=None, out_f32=None, stream=None):
    """sum(x) for Float32 ``x`` (Float64 accumulation).  Returns the Float64 device scalar."""
    torch = _torch()
    d = _dev(x)
    if x.dtype != torch.float32:
        raise KIArgumentError(_abi.KI_ERR_ARG, "warpfold_reduce: Float32 input")
    if out_f64 is None:
        out_f64 = torch.empty((), dtype=torch.float64, device=x.device)
    context(d).call("ki_reduce_sum_f32", _ptr(x), x.numel(), _ptr(out_f32) if out_f32 is not None else None,
                    _ptr(out_f64), _stream_ptr(stream, d))
    return out_f64


def reduce_sum_i64(x, out=None, stream=None):
    """sum(x) for Int64 ``x`` with wrap-around.  Returns the Int64 device scalar."""
    torch = _torch()
    d = _dev(x)
    out = torch.empty((), dtype=torch.int64, device=x.device) if out is None else out
    context(d).call("ki_reduce_sum_i64", _ptr(x), x.numel(), _ptr(out), _stream_ptr(stream, d))
    return out


def warpreduce_scan(x, out=None, seed: int = 0, stream=None):
    """cumsum(x) for Int64 ``x`` (inclusive, single-pass decoupled lookback), plus ``seed``."""
    torch = _torch()
    d = _dev(x)
    if x.dtype != torch.int64:
        raise KIArgumentError(_abi.KI_ERR_ARG, "warpreduce_scan: Int64 input")
    out = torch.empty_like(x) if out is None else out
    context(d).call("ki_scan_inclusive_i64", _ptr(x), _ptr(out), x.numel(), ctypes.c_int64(int(seed)),
                    _stream_ptr(stream, d))
    return out


def warpreduce_scan_host(x, out=None, seed: int = 0, device: int = 0, stream=None):
    """cumsum of a HOST Int64 tensor through GPU ``device`` (chunks cross PCIe, are scanned there and come
    back, both directions overlapped).  Pinned tensors make it asynchronous; it is complete when
    ``stream`` (of ``device``) is."""
    torch = _torch()
    if x.is_cuda or x.dtype != torch.int64 or not x.is_contiguous():
        raise KIArgumentError(_abi.KI_ERR_ARG, "warpreduce_scan_host: contiguous Int64 host tensor")
    out = torch.empty_like(x) if out is None else out
    if out.is_cuda or out.dtype != torch.int64 or out.numel() != x.numel() or not out.is_contiguous():
        raise KIArgumentError(_abi.KI_ERR_ARG, "warpreduce_scan_host: output must match the input, on the host")
    context(device).call("ki_scan_inclusive_i64_host", _ptr(x), _ptr(out), x.numel(), ctypes.c_int64(int(seed)),
                         _stream_ptr(stream, device))
    return out


def _result_dtype(dtype, op: str):
    """Base's result type: sums and products (add_sum / mul_prod) widen integers narrower than 64
    bits to Int64 / UInt64; every other operator keeps the element type."""
    torch = _torch()
    if op in ("+", "add", "*", "mul"):
        if dtype in (torch.int8, torch.int16, torch.int32):
            return torch.int64
        if dtype in (torch.uint8, torch.uint16, torch.uint32):
            return torch.uint64
    return dtype


_GENERIC_OPS = {"+": 0, "add": 0, "max": 1, "min": 2, "|": 3, "or": 3, "&": 4, "and": 4, "xor": 5, "*": 6, "mul": 6}


def _np_dtype(t):
    import numpy as np

    name = str(t).replace("torch.", "")
    if name not in _abi.DTYPE:
        raise KIArgumentError(_abi.KI_ERR_ARG, f"unsupported dtype {t}")
    return np.dtype(name)


def reduce(x, op: str = "+", out=None, stream=None):
    """sum / prod / maximum / minimum / reduce(|, &, xor) of Int8 ... UInt64, Float32 or Float64 ``x``
    with Julia Base semantics (the device-wide @warpfold): sums and products of narrower integers
    widen to 64 bits, Float32 sums and products accumulate in Float64, maximum/minimum propagate
    NaN; the bitwise operators take integers.  Returns a device scalar."""
    torch = _torch()
    d = _dev(x)
    if op not in _GENERIC_OPS:
        raise KIArgumentError(_abi.KI_ERR_ARG, f"reduce: op must be one of {sorted(_GENERIC_OPS)}")
    x = x.contiguous()
    out = torch.empty((), dtype=_result_dtype(x.dtype, op), device=x.device) if out is None else out
    context(d).call("ki_reduce", _GENERIC_OPS[op], _dtype_code(x), _ptr(x), x.numel(), _ptr(out),
                    _stream_ptr(stream, d))
    return out


_MAPS = {None: 0, "identity": 0, "abs": 1, "abs2": 2}


def mapreduce(f, op: str, x, out=None, stream=None):
    """mapreduce(f, op, x) for f in abs, abs2 (computed in the element type, as Base does) and op in
    +, max, min: sum(abs2, x), maximum(abs, x).  Result types as ``reduce``."""
    torch = _torch()
    d = _dev(x)
    if f not in _MAPS:
        raise KIArgumentError(_abi.KI_ERR_ARG, "mapreduce: f must be 'abs', 'abs2' or None")
    if op not in _GENERIC_OPS:
        raise KIArgumentError(_abi.KI_ERR_ARG, f"mapreduce: op must be one of {sorted(_GENERIC_OPS)}")
    x = x.contiguous()
    out = torch.empty((), dtype=_result_dtype(x.dtype, op), device=x.device) if out is None else out
    context(d).call("ki_mapreduce", _MAPS[f], _GENERIC_OPS[op], _dtype_code(x), _ptr(x), x.numel(), _ptr(out),
                    _stream_ptr(stream, d))
    return out


def reduce_rows(x, op: str = "+", out=None, stream=None):
    """One reduction per row (the operators of ``reduce``) of a 2-D ``x`` whose rows are contiguous
    (``x.stride(1) == 1``; ``x.stride(0)`` is the leading dimension).  Result types as ``reduce``."""
    torch = _torch()
    d = _dev(x)
    if op not in _GENERIC_OPS:
        raise KIArgumentError(_abi.KI_ERR_ARG, f"reduce_rows: op must be one of {sorted(_GENERIC_OPS)}")
    if x.dim() != 2 or (x.shape[1] > 1 and x.stride(1) != 1):
        raise KIArgumentError(_abi.KI_ERR_ARG, "reduce_rows: 2-D input with contiguous rows")
    rows, cols = x.shape
    ld = x.stride(0) if rows > 1 else cols
    out = torch.empty(rows, dtype=_result_dtype(x.dtype, op), device=x.device) if out is None else out
    context(d).call("ki_reduce_rows", _GENERIC_OPS[op], _dtype_code(x), _ptr(x), rows, cols, max(ld, cols), _ptr(out),
                    _stream_ptr(stream, d))
    return out


def scan(x, op: str = "+", exclusive: bool = False, init=None, out=None, stream=None):
    """accumulate(op, x; init) / cumsum / cumprod for the operators and types of ``reduce`` (the
    device-wide @warpreduce).  The result has Base's type (widened for sums and products of narrower
    integers); ``exclusive`` shifts it by one element and starts at ``init`` (the identity when None)."""
    import numpy as np

    torch = _torch()
    d = _dev(x)
    if op not in _GENERIC_OPS:
        raise KIArgumentError(_abi.KI_ERR_ARG, f"scan: op must be one of {sorted(_GENERIC_OPS)}")
    rd = _result_dtype(x.dtype, op)
    out = torch.empty(x.shape, dtype=rd, device=x.device) if out is None else out
    init_buf = None
    if init is not None:
        init_buf = np.array([init], dtype=_np_dtype(rd))
    context(d).call("ki_scan", _GENERIC_OPS[op], _dtype_code(x), int(bool(exclusive)), _ptr(x), _ptr(out), x.numel(),
                    ctypes.c_void_p(init_buf.ctypes.data) if init_buf is not None else None, _stream_ptr(stream, d))
    return out


def scan_rows(x, op: str = "+", exclusive: bool = False, init=None, out=None, stream=None):
    """accumulate(op, x; dims) along each row of a 2-D ``x`` whose rows are contiguous
    (``x.stride(1) == 1``; ``x.stride(0)`` is the leading dimension), every row starting from ``init``.
    Operators and result types as ``scan``; ``out`` (rows contiguous) may have its own row stride."""
    import numpy as np

    torch = _torch()
    d = _dev(x)
    if op not in _GENERIC_OPS:
        raise KIArgumentError(_abi.KI_ERR_ARG, f"scan_rows: op must be one of {sorted(_GENERIC_OPS)}")
    if x.dim() != 2 or (x.shape[1] > 1 and x.stride(1) != 1):
        raise KIArgumentError(_abi.KI_ERR_ARG, "scan_rows: 2-D input with contiguous rows")
    rows, cols = x.shape
    rd = _result_dtype(x.dtype, op)
    out = torch.empty((rows, cols), dtype=rd, device=x.device) if out is None else out
    if out.shape != x.shape or out.dtype != rd or (cols > 1 and out.stride(1) != 1):
        raise KIArgumentError(_abi.KI_ERR_ARG, "scan_rows: output of the input's shape, result type and contiguous rows")
    init_buf = None if init is None else np.array([init], dtype=_np_dtype(rd))
    ld_in = x.stride(0) if rows > 1 else cols
    ld_out = out.stride(0) if rows > 1 else cols
    context(d).call("ki_scan_rows", _GENERIC_OPS[op], _dtype_code(x), int(bool(exclusive)), _ptr(x), max(ld_in, cols),
                    _ptr(out), max(ld_out, cols), rows, cols,
                    ctypes.c_void_p(init_buf.ctypes.data) if init_buf is not None else None, _stream_ptr(stream, d))
    return out


_PREDS = {">": 0, ">=": 1, "<": 2, "<=": 3, "==": 4, "!=": 5}


def compact(x, pred: str, threshold, out_vals=None, out_idx=None, count=None, index_base: int = 1, stream=None,
            trim: bool = True, f=None):
    """filter(v -> f(v) pred threshold, x) and findall for Int32/UInt32/Int64/UInt64/Float32/Float64 ``x``
    (IEEE comparisons; f None, 'abs' or 'abs2', applied in the element type; the kept elements are
    x's own).  Returns (vals, idx, count) like ``vote_compact``."""
    import numpy as np

    torch = _torch()
    d = _dev(x)
    if pred not in _PREDS:
        raise KIArgumentError(_abi.KI_ERR_ARG, f"compact: pred must be one of {sorted(_PREDS)}")
    if f not in _MAPS:
        raise KIArgumentError(_abi.KI_ERR_ARG, "compact: f must be 'abs', 'abs2' or None")
    x = x.contiguous()
    n = x.numel()
    thr = np.array([threshold], dtype=_np_dtype(x.dtype))
    out_vals = torch.empty(n, dtype=x.dtype, device=x.device) if out_vals is None else out_vals
    out_idx = torch.empty(n, dtype=torch.int32, device=x.device) if out_idx is None else out_idx
    count = torch.zeros((), dtype=torch.uint64, device=x.device) if count is None else count
    context(d).call("ki_compact_map", _MAPS[f], _PREDS[pred], _dtype_code(x), _ptr(x), n, ctypes.c_void_p(thr.ctypes.data),
                    _ptr(out_vals), _ptr(out_idx), ctypes.c_int64(int(index_base)), _ptr(count), _stream_ptr(stream, d))
    if trim:
        k = int(count.item())
        return out_vals[:k], out_idx[:k], count
    return out_vals, out_idx, count


def count(x, pred: str, threshold, f=None, out=None, stream=None):
    """count(v -> f(v) pred threshold, x): the compaction pipeline with no outputs.  Returns a UInt64
    device scalar."""
    import numpy as np

    torch = _torch()
    d = _dev(x)
    if pred not in _PREDS or f not in _MAPS:
        raise KIArgumentError(_abi.KI_ERR_ARG, "count: unknown predicate or map")
    x = x.contiguous()
    thr = np.array([threshold], dtype=_np_dtype(x.dtype))
    out = torch.zeros((), dtype=torch.uint64, device=x.device) if out is None else out
    context(d).call("ki_compact_map", _MAPS[f], _PREDS[pred], _dtype_code(x), _ptr(x), x.numel(),
                    ctypes.c_void_p(thr.ctypes.data), None, None, ctypes.c_int64(1), _ptr(out), _stream_ptr(stream, d))
    return out


def vote_compact(x, threshold: float, out_vals=None, out_idx=None, count=None, index_base: int = 1,
                 stream=None, trim: bool = True):
    """filter(v -> v > threshold, x) and findall (1-based Int32 indices by default).

    Returns (vals, idx, count) with ``count`` a device uint64 scalar; with trim=True the outputs are
    sliced to the count (one device-to-host read)."""
    torch = _torch()
    d = _dev(x)
    if x.dtype != torch.float32:
        raise KIArgumentError(_abi.KI_ERR_ARG, "vote_compact: Float32 input")
    n = x.numel()
    out_vals = torch.empty(n, dtype=torch.float32, device=x.device) if out_vals is None else out_vals
    out_idx = torch.empty(n, dtype=torch.int32, device=x.device) if out_idx is None else out_idx
    count = torch.zeros((), dtype=torch.uint64, device=x.device) if count is None else count
    context(d).call("ki_compact_gt_f32", _ptr(x), n, ctypes.c_float(threshold), _ptr(out_vals), _ptr(out_idx),
                    ctypes.c_int64(int(index_base)), _ptr(count), _stream_ptr(stream, d))
    if trim:
        k = int(count.item())
        return out_vals[:k], out_idx[:k], count
    return out_vals, out_idx, count


def fp8_gemm(A, B, C=None, scale_a: float = 1.0, scale_b: float = 1.0, stream=None):
    """C = scale_a*scale_b * A @ B for e4m3 A (MxK) and B (KxN), both row-major; Float32 C."""
    torch = _torch()
    d = _dev(A)
    M, K = A.shape
    K2, N = B.shape
    if K != K2:
        raise KIArgumentError(_abi.KI_ERR_ARG, "fp8_gemm: inner dimensions differ")
    C = torch.empty((M, N), dtype=torch.float32, device=A.device) if C is None else C
    context(d).call("ki_gemm_e4m3_f32", _ptr(A), _ptr(B), _ptr(C), M, N, K, ctypes.c_float(scale_a),
                    ctypes.c_float(scale_b), _stream_ptr(stream, d))
    return C


# ---------------------------------------------------------------------------------------------
# synthetic inputs (splitmix64 streams; bit-identical to the host generator)
# ---------------------------------------------------------------------------------------------
def fill_uniform(out, seed: int, stream=None):
    d = _dev(out)
    context(d).call("ki_fill_uniform_f32", ctypes.c_uint64(seed), _ptr(out), out.numel(), _stream_ptr(stream, d))
    return out


def fill_int_range(out, seed: int, lo: int, hi: int, stream=None):
    d = _dev(out)
    context(d).call("ki_fill_int_range_i64", ctypes.c_uint64(seed), ctypes.c_int64(lo), ctypes.c_int64(hi),
                    _ptr(out), out.numel(), _stream_ptr(stream, d))
    return out


def fill_bytes(out, seed: int, stream=None):
    d = _dev(out)
    context(d).call("ki_fill_bytes", ctypes.c_uint64(seed), _ptr(out), out.numel() * out.element_size(),
                    _stream_ptr(stream, d))
    return out


def fill_normal(out, seed: int, stream=None):
    d = _dev(out)
    context(d).call("ki_fill_normal_f32", ctypes.c_uint64(seed), _ptr(out), out.numel(), _stream_ptr(stream, d))
    return out


def fill_e4m3_uniform(out, seed: int, scale: float, stream=None):
    d = _dev(out)
    context(d).call("ki_fill_e4m3_uniform", ctypes.c_uint64(seed), ctypes.c_float(scale), _ptr(out),
                    out.numel() * out.element_size(), _stream_ptr(stream, d))
    return out
