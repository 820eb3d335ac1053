"""GPU: the allocation-free scan entry point, called through the C ABI.

ki_scan_inclusive_i64_noalloc exists for callers that cannot allocate device memory (hosts whose
device memory belongs to another allocator, loops that forbid allocation after start-up, code that
must not stall the device as cudaMalloc may).  It must give exactly Base.cumsum (the oracle) and what the
context-based entry point gives, on consecutive calls that share its static scratch.  This file is
collected last on purpose.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

MAX_N = 1 << 28


def _noalloc(lib, x, y, n, seed, stream):
    return lib.ki_scan_inclusive_i64_noalloc(ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(y.data_ptr()), n,
                                             ctypes.c_int64(seed), ctypes.c_void_p(stream.cuda_stream))


def test_noalloc_scan_matches_oracle_and_context_scan_twice(KI, dev, oracle):
    import torch

    from kernelintrinsics import _abi

    lib = _abi.load()
    stream = torch.cuda.current_stream(dev)
    cases = [((1 << 22) + 5, 3, 0), ((1 << 20) + 4097, 11, -987654321)]
    for n, data_seed, seed in cases:  # two calls in a row on the shared static scratch
        x = torch.empty(n, dtype=torch.int64, device=dev)
        KI.fill_int_range(x, seed=data_seed, lo=-1000, hi=1000)
        want_ctx = KI.warpreduce_scan(x, seed=seed)
        got = torch.full_like(x, 7)
        assert _noalloc(lib, x, got, n, seed, stream) == _abi.KI_OK
        torch.cuda.synchronize()
        want = oracle.cumsum_i64(oracle.gen_int_range_i64(data_seed, -1000, 1000, n), seed=seed)
        got_h = got.cpu().numpy()
        assert np.array_equal(got_h, want), n  # integer scan: bit-exact is the tolerance
        assert torch.equal(got, want_ctx), n


def test_noalloc_scan_inside_a_cuda_graph(KI, dev, oracle):
    """The use it was built for: after one warm-up call (the one-time set-up runs outside capture),
    the call is captured into a CUDA graph under torch's global capture mode, which refuses any
    allocation, and the graph is replayed on new data twice, each replay equal to the oracle and to
    the context scan."""
    import torch

    from kernelintrinsics import _abi

    lib = _abi.load()
    n = (1 << 21) + 77
    seed = -31
    x = torch.empty(n, dtype=torch.int64, device=dev)
    KI.fill_int_range(x, seed=13, lo=-1000, hi=1000)
    y = torch.empty_like(x)
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        assert _noalloc(lib, x, y, n, seed, side) == _abi.KI_OK
    torch.cuda.current_stream(dev).wait_stream(side)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    rcs = []
    with torch.cuda.graph(g):
        rcs.append(_noalloc(lib, x, y, n, seed, torch.cuda.current_stream(dev)))
    assert rcs == [_abi.KI_OK]
    for data_seed in (29, 41):
        KI.fill_int_range(x, seed=data_seed, lo=-1000, hi=1000)
        y.fill_(7)
        g.replay()
        torch.cuda.synchronize()
        want = oracle.cumsum_i64(oracle.gen_int_range_i64(data_seed, -1000, 1000, n), seed=seed)
        assert np.array_equal(y.cpu().numpy(), want), data_seed
        assert torch.equal(y, KI.warpreduce_scan(x, seed=seed)), data_seed
    del g
    torch.cuda.synchronize()


def test_noalloc_scan_at_its_largest_size(KI, dev):
    """n just under the maximum fills nearly every tile slot of the static scratch; the output is
    fixed exactly by out[0] = seed + in[0] and out[i] - out[i-1] = in[i] (checked on the device)."""
    import torch

    from kernelintrinsics import _abi

    lib = _abi.load()
    stream = torch.cuda.current_stream(dev)
    n = MAX_N - 3
    x = torch.empty(n, dtype=torch.int64, device=dev)
    KI.fill_int_range(x, seed=5, lo=-1000, hi=1000)
    y = torch.empty_like(x)
    for seed in (0, 1 << 40):  # twice in a row
        assert _noalloc(lib, x, y, n, seed, stream) == _abi.KI_OK
        torch.cuda.synchronize()
        assert int(y[0].item()) == seed + int(x[0].item())
        assert torch.equal(y[1:] - y[:-1], x[1:])
    del x, y
    torch.cuda.empty_cache()


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
