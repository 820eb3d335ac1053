"""Range-sharded reduce / scan / compaction across one process per GPU.

The input of every operation is split into contiguous shards, shard r on rank r.  Only per-shard
totals and counts cross the interconnect, with one ``all_gather_into_tensor`` of one 8-byte value
per rank (NCCL over NVLink for CUDA tensors; gloo for CPU tensors in host-logic tests):

* reduce     local Float64 partial -> all-gather -> every rank sums the partials in rank order
             (deterministic, identical on every rank);
* scan       phase 1 shard total (reduce) -> all-gather -> phase 2 local scan seeded with the sum of
             lower ranks' totals; the last rank skips phase 1's result use but still joins the
             collective so every rank takes the same collective steps;
* compaction local single-pass compaction with index_base = 1 + shard start -> all-gather of the
             counts -> each rank's output offset is the exclusive prefix of the counts.  The
             concatenation of the ranks' outputs in rank order is filter/findall of the whole input.

``ops`` carries the per-shard kernels.  The default is the libki_b200 kernels; host-logic tests
inject CPU implementations so the collective plumbing runs under gloo without a GPU.
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
