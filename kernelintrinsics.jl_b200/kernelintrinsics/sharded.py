"""Range-sharded reduce / scan / compaction across several GPUs.

The input of every operation is split into contiguous shards, shard r on rank r.  Only one 8-byte
value per rank and operation crosses between the GPUs:

* reduce     local Float64 partial -> exchange -> every rank adds the partials in rank order
             (deterministic, identical on every rank);
* scan       phase 1 shard total -> exchange -> phase 2 local scan seeded with the sum of the lower
             ranks' totals;
* compaction local single-pass compaction with index_base = 1 + shard start -> exchange of the counts
             -> each rank's output offset is the exclusive prefix of the counts.  The concatenation of
             the ranks' outputs in rank order is filter/findall of the whole input.

Two implementations of the same protocol live here:

* ``Comm`` -- the product path: a libki_b200 communicator (``ki_comm``, C ABI).  The exchange is a
  one-warp kernel that pushes the value into every peer's buffer over NVLink (st.release.sys) and
  waits with bounded ld.acquire.sys loads, so the seed / offset never visits the host.  One process
  per GPU (``Comm.from_process_group``, the NCCL unique id is broadcast over torch.distributed) or one
  process driving several GPUs (``Comm.create``).
* ``reduce_sharded`` / ``scan_sharded`` / ``compact_sharded`` -- the same protocol over any
  torch.distributed backend (an ``all_gather_into_tensor`` of the 8-byte values), with the per-shard
  kernels injected through ``ShardOps``.  The CPU tests run it under gloo with the oracle as the
  per-shard kernels, to check the protocol (shard ranges, seeds, offsets, a rank that leaves).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Optional


def shard_range(n: int, world: int, rank: int) -> tuple:
    """Contiguous shard [lo, hi) of rank ``rank``: the first n % world shards get one extra element."""
    if world <= 0 or not 0 <= rank < world or n < 0:
        raise ValueError("bad shard arguments")
    q, r = divmod(n, world)
    lo = rank * q + min(rank, r)
    hi = lo + q + (1 if rank < r else 0)
    return lo, hi


def scan_shard_range(n: int, world: int, rank: int) -> tuple:
    """[lo, hi) of ``rank`` under ki_comm_scan_shard_range: weights 2, ..., 2, 3 (the last rank of the
    sharded scan reads its shard once, the others twice), boundaries rounded down to 256 elements."""
    if world <= 0 or not 0 <= rank < world or n < 0:
        raise ValueError("bad shard arguments")

    def edge(r):
        return n if r >= world else (n * 2 * r // (2 * world + 1)) & ~255

    return edge(rank), edge(rank + 1)


def exclusive_prefix(values) -> list:
    out, run = [], 0
    for v in values:
        out.append(run)
        run += v
    return out


def wrap64(v: int) -> int:
    v &= (1 << 64) - 1
    return v - (1 << 64) if v >= 1 << 63 else v


@dataclass
class ShardOps:
    """Per-shard operations (device tensors in, device tensors out)."""

    sum_f32_to_f64: Callable            # x -> 0-d float64 tensor
    sum_i64: Callable                   # x -> 0-d int64 tensor
    scan_i64: Callable                  # (x, out, seed:int) -> out
    compact_gt: Callable                # (x, thr, index_base) -> (vals, idx, count 0-d tensor)


def cuda_ops() -> ShardOps:
    """The libki_b200 single-GPU kernels as per-shard operations (for the torch.distributed path)."""
    from . import reduce_sum_i64, vote_compact, warpfold_reduce, warpreduce_scan

    return ShardOps(
        sum_f32_to_f64=lambda x: warpfold_reduce(x),
        sum_i64=lambda x: reduce_sum_i64(x),
        scan_i64=lambda x, out, seed: warpreduce_scan(x, out=out, seed=seed),
        compact_gt=lambda x, thr, base: vote_compact(x, thr, index_base=base, trim=False),
    )


def _gather_scalar(value, group=None):
    """All-gather one 8-byte scalar tensor per rank -> 1-d tensor of world_size values."""
    import torch
    import torch.distributed as dist

    world = dist.get_world_size(group)
    v = value.reshape(1)
    out = torch.empty(world, dtype=v.dtype, device=v.device)
    dist.all_gather_into_tensor(out, v, group=group)
    return out


def reduce_sharded(x_local, group=None, ops: Optional[ShardOps] = None):
    """sum over all ranks' shards (Float32 data, Float64 result), same bits on every rank."""
    import torch

    ops = ops or cuda_ops()
    part = ops.sum_f32_to_f64(x_local).to(torch.float64)
    parts = _gather_scalar(part, group)
    total = torch.zeros((), dtype=torch.float64, device=parts.device)
    for i in range(parts.numel()):   # rank order: deterministic
        total = total + parts[i]
    return total


def scan_sharded(x_local, out_local=None, group=None, ops: Optional[ShardOps] = None):
    """Inclusive Int64 scan of the concatenated shards; rank r gets its slice of cumsum(x)."""
    import torch
    import torch.distributed as dist

    ops = ops or cuda_ops()
    rank = dist.get_rank(group)
    world = dist.get_world_size(group)
    if out_local is None:
        out_local = torch.empty_like(x_local)
    if world == 1:
        return ops.scan_i64(x_local, out_local, 0)
    if rank < world - 1:
        tot = ops.sum_i64(x_local).to(torch.int64)
    else:  # nobody reads the last shard's total; it still joins the all-gather
        tot = torch.zeros((), dtype=torch.int64, device=x_local.device)
    totals = _gather_scalar(tot, group).cpu().tolist()
    seed = wrap64(sum(totals[:rank]))
    return ops.scan_i64(x_local, out_local, seed)


def compact_sharded(x_local, threshold: float, shard_start: int, group=None, ops: Optional[ShardOps] = None):
    """Local filter/findall of the shard with global 1-based indices, plus the global layout.

    Returns (vals, idx, local_count, offset, total): this rank's kept values and indices belong at
    [offset, offset + local_count) of the global output."""
    import torch

    ops = ops or cuda_ops()
    vals, idx, cnt = ops.compact_gt(x_local, threshold, 1 + int(shard_start))
    counts = _gather_scalar(cnt.to(torch.int64), group).cpu().tolist()
    import torch.distributed as dist

    rank = dist.get_rank(group)
    offs = exclusive_prefix(counts)
    k = int(counts[rank])
    return vals[:k], idx[:k], k, offs[rank], sum(counts)


# ---------------------------------------------------------------------------------------------
# the C-ABI communicator (product path)
# ---------------------------------------------------------------------------------------------
_XCHG = {"auto": 0, "peer": 1, "nccl": 2}


def broadcast_comm_id(make_id, group=None) -> bytes:
    """Rank 0 of ``group`` makes the communicator id (``make_id()``, 128 bytes) and every rank
    receives it over torch.distributed (any backend)."""
    import torch.distributed as dist

    rank = dist.get_rank(group)
    src = dist.get_global_rank(group, 0) if group is not None else 0
    obj = [make_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=src, group=group)
    cid = obj[0]
    if not isinstance(cid, (bytes, bytearray)) or len(cid) != 128:
        raise ValueError("communicator id must be 128 bytes")
    return bytes(cid)


class Comm:
    """One rank of a libki_b200 communicator (``ki_comm``): sharded operations on this rank's GPU.

    Every rank must call the same operations in the same order on its own shard; the calls of one
    communicator are stream-ordered (the current torch stream unless ``stream`` is given)."""

    def __init__(self, handle, lib=None):
        import ctypes

        from . import _abi

        self.lib = lib or _abi.load()
        self.handle = handle
        nr, rk, dv, ex = (ctypes.c_int(), ctypes.c_int(), ctypes.c_int(), ctypes.c_int())
        self.lib.ki_comm_info(handle, ctypes.byref(nr), ctypes.byref(rk), ctypes.byref(dv), ctypes.byref(ex))
        self.nranks, self.rank, self.device = nr.value, rk.value, dv.value
        self.exchange = {v: k for k, v in _XCHG.items()}[ex.value]
        c = ctypes.c_void_p()
        self.lib.ki_comm_get_ctx(handle, ctypes.byref(c))
        self.ctx = c

    # -- creation ----------------------------------------------------------------------------
    @staticmethod
    def get_id() -> bytes:
        import ctypes

        from . import _abi

        lib = _abi.load()
        buf = ctypes.create_string_buffer(_abi.COMM_ID_BYTES)
        st = lib.ki_comm_get_id(buf)
        if st != _abi.KI_OK:
            raise _abi.status_error(st, f"ki_comm_get_id: {lib.ki_status_string(st).decode()}")
        return buf.raw

    @classmethod
    def init_rank(cls, device: int, nranks: int, rank: int, comm_id: bytes, exchange: str = "auto") -> "Comm":
        import ctypes

        from . import _abi

        lib = _abi.load()
        buf = ctypes.create_string_buffer(bytes(comm_id), _abi.COMM_ID_BYTES)
        h = ctypes.c_void_p()
        st = lib.ki_comm_init_rank(int(device), int(nranks), int(rank), buf, _XCHG[exchange], ctypes.byref(h))
        if st != _abi.KI_OK:
            raise _abi.status_error(st, f"ki_comm_init_rank: {lib.ki_last_error_string(None).decode(errors='replace')}")
        return cls(h, lib)

    @classmethod
    def from_process_group(cls, device: Optional[int] = None, group=None, exchange: str = "auto") -> "Comm":
        """One process per GPU: rank 0 makes the id, torch.distributed broadcasts it, every rank joins."""
        import torch
        import torch.distributed as dist

        if device is None:
            device = torch.cuda.current_device()
        cid = broadcast_comm_id(cls.get_id, group)
        return cls.init_rank(device, dist.get_world_size(group), dist.get_rank(group), cid, exchange)

    @classmethod
    def create(cls, devices) -> list:
        """One process driving several GPUs (0-based device ids): one Comm per device, rank i on
        devices[i].  Issue each operation on every rank before the next operation and before waiting
        on any of them (a first call may allocate scratch, which can wait for the GPU's pending
        exchange)."""
        import ctypes

        from . import _abi

        lib = _abi.load()
        n = len(devices)
        devs = (ctypes.c_int * n)(*[int(d) for d in devices])
        hs = (ctypes.c_void_p * n)()
        st = lib.ki_comm_create(n, devs, hs)
        if st != _abi.KI_OK:
            raise _abi.status_error(st, f"ki_comm_create: {lib.ki_last_error_string(None).decode(errors='replace')}")
        return [cls(ctypes.c_void_p(hs[i]), lib) for i in range(n)]

    # -- life cycle --------------------------------------------------------------------------
    def close(self) -> None:
        """Collective for process-group communicators (a bounded barrier, then unmap and free)."""
        if self.handle:
            st = self.lib.ki_comm_destroy(self.handle)
            self.handle = None
            if st:
                from . import _abi

                raise _abi.status_error(st, "ki_comm_destroy")

    def abort(self) -> None:
        """Local tear-down without the barrier (peers failed or left)."""
        if self.handle:
            self.lib.ki_comm_abort(self.handle)
            self.handle = None

    def _raise(self, st: int, what: str):
        from . import _abi

        msg = self.lib.ki_last_error_string(self.ctx).decode(errors="replace")
        raise _abi.status_error(st, f"{what}: {msg or self.lib.ki_status_string(st).decode()}")

    def _call(self, name: str, *args) -> None:
        st = getattr(self.lib, name)(self.handle, *args)
        if st:
            self._raise(st, name)

    def check(self, stream=None) -> None:
        """Synchronise ``stream``; raise KITimeoutError if an exchange wait of this rank ran out."""
        st = self.lib.ki_ctx_check(self.ctx, self._stream(stream))
        if st:
            self._raise(st, "ki_ctx_check")

    def set_wait_timeout(self, seconds: float) -> None:
        import ctypes

        st = self.lib.ki_ctx_set_wait_timeout_ns(self.ctx, ctypes.c_uint64(int(seconds * 1e9)))
        if st:
            self._raise(st, "ki_ctx_set_wait_timeout_ns")

    def _stream(self, stream):
        import ctypes

        import torch

        if stream is None:
            stream = torch.cuda.current_stream(self.device)
        return ctypes.c_void_p(stream.cuda_stream)

    def shard_range(self, n: int) -> tuple:
        return shard_range(n, self.nranks, self.rank)

    def scan_shard_range(self, n: int) -> tuple:
        """[lo, hi) of this rank under the split that equalises the sharded scan's bytes per rank."""
        return scan_shard_range(n, self.nranks, self.rank)

    # -- sharded operations ------------------------------------------------------------------
    def reduce_sum(self, x, out_f64=None, out_f32=None, stream=None):
        """sum over all ranks' Float32 shards (Float64 result, the same bits on every rank)."""
        import ctypes

        import torch

        if x.dtype != torch.float32 or not x.is_cuda:
            raise ValueError("reduce_sum: Float32 CUDA shard")
        if out_f64 is None and out_f32 is None:
            out_f64 = torch.empty((), dtype=torch.float64, device=x.device)
        self._call("ki_reduce_sum_f32_sharded", ctypes.c_void_p(x.data_ptr()), x.numel(),
                   ctypes.c_void_p(out_f32.data_ptr()) if out_f32 is not None else None,
                   ctypes.c_void_p(out_f64.data_ptr()) if out_f64 is not None else None, self._stream(stream))
        return out_f64 if out_f64 is not None else out_f32

    def scan(self, x, out=None, stream=None):
        """This rank's slice of cumsum over the concatenated Int64 shards."""
        import ctypes

        import torch

        if x.dtype != torch.int64 or not x.is_cuda:
            raise ValueError("scan: Int64 CUDA shard")
        out = torch.empty_like(x) if out is None else out
        self._call("ki_scan_inclusive_i64_sharded", ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(out.data_ptr()),
                   x.numel(), self._stream(stream))
        return out

    def scan_host(self, x, out=None, stream=None):
        """``scan`` with this rank's shard in HOST memory (contiguous Int64, pinned for asynchrony):
        the shard crosses to the device, is summed, the totals are exchanged, and the scanned chunks
        come back as they finish."""
        import ctypes

        import torch

        if x.is_cuda or x.dtype != torch.int64 or not x.is_contiguous():
            raise ValueError("scan_host: contiguous Int64 host shard")
        out = torch.empty_like(x) if out is None else out
        self._call("ki_scan_inclusive_i64_sharded_host", ctypes.c_void_p(x.data_ptr()),
                   ctypes.c_void_p(out.data_ptr()), x.numel(), self._stream(stream))
        return out

    def compact_gt(self, x, threshold: float, index_base: int, out_vals=None, out_idx=None, count=None, offset=None,
                   total=None, stream=None):
        """filter/findall of x > threshold over the concatenated Float32 shards.  ``index_base`` is the
        1-based global index of this shard's first element.  Returns (vals, idx, count, offset, total):
        untrimmed outputs and device uint64 scalars; this rank's kept elements belong at
        [offset, offset + count) of the global result."""
        import ctypes

        import torch

        if x.dtype != torch.float32 or not x.is_cuda:
            raise ValueError("compact_gt: Float32 CUDA shard")
        n, dev = x.numel(), x.device
        out_vals = torch.empty(n, dtype=torch.float32, device=dev) if out_vals is None else out_vals
        out_idx = torch.empty(n, dtype=torch.int32, device=dev) if out_idx is None else out_idx
        count = torch.zeros((), dtype=torch.uint64, device=dev) if count is None else count
        offset = torch.zeros((), dtype=torch.uint64, device=dev) if offset is None else offset
        total = torch.zeros((), dtype=torch.uint64, device=dev) if total is None else total
        self._call("ki_compact_gt_f32_sharded", ctypes.c_void_p(x.data_ptr()), n, ctypes.c_float(threshold),
                   ctypes.c_void_p(out_vals.data_ptr()), ctypes.c_void_p(out_idx.data_ptr()),
                   ctypes.c_int64(int(index_base)), ctypes.c_void_p(count.data_ptr()),
                   ctypes.c_void_p(offset.data_ptr()), ctypes.c_void_p(total.data_ptr()), self._stream(stream))
        return out_vals, out_idx, count, offset, total
