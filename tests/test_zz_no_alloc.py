"""GPU: the allocation-free scan entry point, called through the C ABI.

ki_scan_inclusive_i64_noalloc exists for callers that cannot allocate device memory (code running
while a CUDA graph is captured, hosts whose device memory belongs to another allocator, loops that
forbid allocation after start-up).  It must give exactly what the context-based entry point gives,
on consecutive calls that share its static scratch.  This file is collected last on purpose.
"""
from __future__ import annotations

import ctypes

import pytest

pytestmark = pytest.mark.gpu

MAX_N = 1 << 28


def _noalloc(lib, x, y, n, seed, stream):
    return lib.ki_scan_inclusive_i64_noalloc(ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(y.data_ptr()), n,
                                             ctypes.c_int64(seed), ctypes.c_void_p(stream.cuda_stream))


def test_noalloc_scan_matches_context_scan_twice(KI, dev):
    import torch

    from kernelintrinsics import _abi

    lib = _abi.load()
    stream = torch.cuda.current_stream(dev)
    cases = [((1 << 22) + 5, 3, 0), ((1 << 20) + 4097, 11, -987654321)]
    for n, data_seed, seed in cases:  # two calls in a row on the shared static scratch
        x = torch.empty(n, dtype=torch.int64, device=dev)
        KI.fill_int_range(x, seed=data_seed, lo=-1000, hi=1000)
        want = KI.warpreduce_scan(x, seed=seed)
        got = torch.full_like(x, 7)
        assert _noalloc(lib, x, got, n, seed, stream) == _abi.KI_OK
        torch.cuda.synchronize()
        assert torch.equal(got, want), n  # integer scan: bit-exact is the tolerance


def test_noalloc_scan_rejects_sizes_beyond_its_scratch(KI, dev):
    import torch

    from kernelintrinsics import _abi

    lib = _abi.load()
    stream = torch.cuda.current_stream(dev)
    n = MAX_N + 1  # buffers really hold n elements, so nothing could be touched out of bounds
    x = torch.zeros(n, dtype=torch.int64, device=dev)
    y = torch.zeros(n, dtype=torch.int64, device=dev)
    assert _noalloc(lib, x, y, n, 0, stream) == _abi.KI_ERR_ARG
    torch.cuda.synchronize()
    assert int(y.abs().sum().item()) == 0
    del x, y
    torch.cuda.empty_cache()
