"""GPU: ki_vcopy (copyto! with 128-bit accesses at any alignment) -- bit-exact, guard bytes intact."""
from __future__ import annotations

import itertools

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

GUARD = 32


def _copy_case(KI, src, dst, so, do, n):
    """dst has GUARD bytes before and after the target range; they must survive."""
    dst.fill_(0xA5)
    KI.vcopy(dst, src, n, dst_offset=GUARD + do, src_offset=so)
    return dst


def test_small_every_alignment_vs_oracle(KI, oracle, dev):
    import torch

    src_h = oracle.gen_bytes(2, 4096 + 64)
    src = torch.from_numpy(src_h).to(dev)
    dst = torch.empty(4096 + 2 * GUARD + 64, dtype=torch.uint8, device=dev)
    lengths = list(range(0, 70)) + [127, 128, 129, 511, 512, 513, 1000, 2047, 2048, 2049, 4096]
    for so, do in itertools.product(range(16), range(16)):
        for n in lengths:
            _copy_case(KI, src, dst, so, do, n)
            got = dst.cpu().numpy()
            want = np.full_like(got, 0xA5)
            oracle.copy_bytes(want[GUARD + do:GUARD + do + n], src_h[so:so + n])
            assert np.array_equal(got, want), (so, do, n)


def test_config_size_all_4096_alignment_cases(KI, dev):
    """Byte copy of 2^28 - t bytes for every (src_offset, dst_offset, t) in 0..15^3."""
    import torch

    N = 1 << 28
    src = torch.empty(N + 16, dtype=torch.uint8, device=dev)
    KI.fill_bytes(src, seed=2)
    dst = torch.empty(N + 2 * GUARD + 16, dtype=torch.uint8, device=dev)
    guard = torch.full((2 * GUARD + 32,), 0xA5, dtype=torch.uint8, device=dev)
    bad = []
    for so, do, t in itertools.product(range(16), range(16), range(16)):
        n = N - t
        d0 = GUARD + do
        dst[:d0].fill_(0xA5)
        dst[d0 + n:].fill_(0xA5)
        KI.vcopy(dst, src, n, dst_offset=d0, src_offset=so)
        ok = torch.equal(dst[d0:d0 + n], src[so:so + n])
        ok = ok and torch.equal(dst[:d0], guard[:d0]) and torch.equal(dst[d0 + n:], guard[:dst.numel() - d0 - n])
        if not ok:
            bad.append((so, do, t))
            if len(bad) > 5:
                break
    assert not bad, bad
    del src, dst
    torch.cuda.empty_cache()


def test_overlap_and_null_rejected(KI, dev):
    import torch

    a = torch.zeros(1024, dtype=torch.uint8, device=dev)
    with pytest.raises(KI.KIArgumentError):
        KI.vcopy(a, a, 512, dst_offset=100, src_offset=0)
    KI.vcopy(a, a, 0)  # empty copy is a no-op


def test_repeatable_on_streams(KI, dev):
    import torch

    src = torch.empty(1 << 22, dtype=torch.uint8, device=dev)
    KI.fill_bytes(src, seed=77)
    s = torch.cuda.Stream()
    dst = torch.zeros_like(src)
    with torch.cuda.stream(s):
        for k in range(10):
            KI.vcopy(dst, src, src.numel() - 16, dst_offset=k, src_offset=15 - k)
            assert torch.equal(dst[k:k + src.numel() - 16], src[15 - k:15 - k + src.numel() - 16])
    s.synchronize()


@pytest.mark.parametrize("pinned", [True, False])
def test_host_buffers_pipelined(KI, oracle, dev, pinned):
    """ki_vcopy_host: host -> device -> kernel -> host in overlapped chunks, any alignment, ragged
    lengths around the chunk size; guard bytes of the host destination survive."""
    import torch

    chunk = 16 << 20  # KI_PIPE_CHUNK
    n_max = 5 * chunk + 4096
    src = torch.from_numpy(oracle.gen_bytes(7, n_max + 32))
    if pinned:
        src = src.pin_memory()
    dst = torch.empty(n_max + 2 * GUARD + 32, dtype=torch.uint8, pin_memory=pinned)
    s_np = src.numpy()
    cases = [(0, 0, 1), (3, 11, 100), (5, 0, chunk - 1), (0, 7, chunk), (15, 1, chunk + 1),
             (9, 9, 4 * chunk), (2, 13, 5 * chunk + 4095), (1, 0, 3 * chunk + 17)]
    for so, do, n in cases:
        dst.fill_(0xA5)
        KI.vcopy_host(dst, src, n, dst_offset=GUARD + do, src_offset=so, device=dev.index or 0)
        torch.cuda.current_stream(dev).synchronize()
        got = dst.numpy()
        assert np.array_equal(got[GUARD + do:GUARD + do + n], s_np[so:so + n]), (so, do, n)
        assert (got[:GUARD + do] == 0xA5).all() and (got[GUARD + do + n:] == 0xA5).all(), (so, do, n)
    KI.context(dev.index or 0).check()


def test_host_buffers_rejects_device_and_overlap(KI, dev):
    import torch

    h = torch.zeros(1024, dtype=torch.uint8)
    with pytest.raises(KI.KIArgumentError):
        KI.vcopy_host(h, h, 100, dst_offset=50, src_offset=0)
    with pytest.raises(KI.KIArgumentError):
        KI.vcopy_host(h, torch.zeros(1024, dtype=torch.uint8, device=dev), 100)
