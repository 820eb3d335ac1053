"""GPU: copyto! between strided views -- ki_vcopy_2d (pitched rows at any byte alignment) and
ki_vcopy_strided (element strides of either sign) against the oracle's element-by-element copies;
bit-exact, bytes outside the destination view untouched."""
from __future__ import annotations

import itertools

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _bytes(oracle, seed, n):
    return oracle.gen_bytes(seed, n)


def test_2d_alignments_pitches_and_widths(KI, oracle, dev):
    import torch

    src_h = _bytes(oracle, 21, 1 << 20)
    src = torch.from_numpy(src_h).to(dev)
    dst = torch.empty(1 << 20, dtype=torch.uint8, device=dev)
    fill = _bytes(oracle, 22, 1 << 20)
    fill_d = torch.from_numpy(fill).to(dev)
    shapes = [(1, 1), (3, 15), (5, 16), (7, 17), (64, 100), (33, 1000), (9, 4099), (300, 2048)]
    for (h, w), (so, do) in itertools.product(shapes, [(0, 0), (1, 0), (0, 5), (7, 3), (15, 15), (4, 12), (8, 9)]):
        for dp_extra, sp_extra in ((0, 0), (1, 13), (16, 32), (29, 3)):
            dp, sp = w + dp_extra, w + sp_extra
            if do + (h - 1) * dp + w > dst.numel() or so + (h - 1) * sp + w > src.numel():
                continue
            dst.copy_(fill_d)
            KI.vcopy_2d(dst, dp, src, sp, w, h, dst_offset=do, src_offset=so)
            want = fill.copy()
            oracle.copy_2d(want, dp, src_h, sp, w, h, dst_offset=do, src_offset=so)
            assert np.array_equal(dst.cpu().numpy(), want), (h, w, so, do, dp, sp)
    KI.context(0).check()


@pytest.mark.parametrize("width", [200, 600, 1500])  # narrow-row kernel (odd pitches up to 1 KiB), warp per row
def test_2d_every_alignment_pair(KI, oracle, dev, width):
    """All 16 x 16 (source, destination) alignments, with a pitch that moves each row's alignment."""
    import torch

    src_h = _bytes(oracle, 23, 1 << 16)
    src = torch.from_numpy(src_h).to(dev)
    dst = torch.zeros(1 << 16, dtype=torch.uint8, device=dev)
    for so, do in itertools.product(range(16), range(16)):
        dst.zero_()
        KI.vcopy_2d(dst, width + 7, src, width + 3, width, 40, dst_offset=do, src_offset=so)
        want = np.zeros(1 << 16, dtype=np.uint8)
        oracle.copy_2d(want, width + 7, src_h, width + 3, width, 40, dst_offset=do, src_offset=so)
        assert np.array_equal(dst.cpu().numpy(), want), (so, do)


@pytest.mark.parametrize("dtype", ["int8", "int16", "float32", "float64", "complex128"])
def test_strided_elements(KI, oracle, dev, dtype):
    import torch

    tdt = getattr(torch, dtype)
    es = torch.empty(0, dtype=tdt).element_size()
    n = 300_000
    src_h = _bytes(oracle, 24, n * es).view(np.dtype(dtype))
    src = torch.from_numpy(src_h.copy()).to(dev)
    for count, ss, ds, s0, d0 in [(1, 1, 1, 0, 0), (1000, 2, 1, 5, 0), (31, -1, 3, 30, 2), (99_999, 3, -2, 0, 200_010),
                                  (4097, 0, 1, 77, 0), (50_000, -5, 5, 299_999, 1)]:
        dst_h = _bytes(oracle, 25, n * es).view(np.dtype(dtype)).copy()
        dst = torch.from_numpy(dst_h.copy()).to(dev)
        KI.vcopy_strided(dst, ds, src, ss, count, dst_start=d0, src_start=s0)
        oracle.copy_strided(dst_h, ds, src_h, ss, count, dst_start=d0, src_start=s0)
        assert np.array_equal(dst.cpu().numpy().view(np.uint8), dst_h.view(np.uint8)), (count, ss, ds)
    KI.context(0).check()


@pytest.mark.parametrize("elem", [3, 6, 12, 24, 40, 48])
def test_strided_structs(KI, oracle, dev, elem):
    """Struct elements of sizes that are not 1, 2, 4, 8 or 16 bytes (the reference's scalar fallback
    for non-power-of-two types), held in byte buffers, strides of either sign."""
    import torch

    vt = np.dtype(f"V{elem}")
    n = 40_000
    src_h = _bytes(oracle, 26, n * elem)
    src = torch.from_numpy(src_h.copy()).to(dev)
    for count, ss, ds, s0, d0 in [(1, 1, 1, 0, 0), (999, 2, 3, 7, 1), (5000, -3, 1, 39_999, 10), (20_000, 1, -2, 0, 39_999),
                                  (333, 0, 5, 12, 0)]:
        dst_h = _bytes(oracle, 27, n * elem)
        dst = torch.from_numpy(dst_h.copy()).to(dev)
        KI.vcopy_strided(dst, ds, src, ss, count, dst_start=d0, src_start=s0, elem_bytes=elem)
        want = dst_h.copy().view(vt)
        oracle.copy_strided(want, ds, src_h.view(vt), ss, count, dst_start=d0, src_start=s0)
        assert np.array_equal(dst.cpu().numpy(), want.view(np.uint8)), (elem, count, ss, ds)
    KI.context(0).check()


def test_copyto_views(KI, dev):
    """copyto! on torch views: a column-major block (2-D, contiguous rows), a strided 1-D view, a
    contiguous range."""
    import torch

    g = torch.Generator(device="cpu").manual_seed(3)
    a = torch.randn(1000, 777, generator=g).to(dev)
    b = torch.zeros(1200, 901, device=dev)
    KI.copyto(b[5:905, 3:700], a[100:1000, 11:708])
    ref = torch.zeros(1200, 901, device=dev)
    ref[5:905, 3:700] = a[100:1000, 11:708]
    assert torch.equal(b, ref)
    c = torch.zeros(3000, dtype=torch.float64, device=dev)
    d = torch.arange(9000, dtype=torch.float64, device=dev)
    KI.copyto(c[1::3], d[::9])
    ref = torch.zeros(3000, dtype=torch.float64, device=dev)
    ref[1::3] = d[::9]
    assert torch.equal(c, ref)
    KI.copyto(c[:100], d[17:117])
    assert torch.equal(c[:100], d[17:117])
    with pytest.raises(KI.KIArgumentError):
        KI.copyto(c[:10], d[:11])
    x = torch.zeros(4, 4, 4, device=dev)
    with pytest.raises(KI.KIArgumentError):
        KI.copyto(x.permute(2, 1, 0), x.clone().permute(2, 1, 0))


def test_errors(KI, dev):
    import torch

    buf = torch.zeros(1 << 16, dtype=torch.uint8, device=dev)
    with pytest.raises(KI.KIArgumentError):  # overlapping ranges
        KI.vcopy_2d(buf, 100, buf, 100, 50, 10, dst_offset=500, src_offset=0)
    with pytest.raises(KI.KIArgumentError):  # pitch below the width
        KI.vcopy_2d(buf, 40, buf, 100, 50, 10, dst_offset=30000, src_offset=0)
    f = torch.zeros(1000, dtype=torch.float32, device=dev)
    with pytest.raises(KI.KIArgumentError):  # destination stride 0
        KI.vcopy_strided(f, 0, f.clone(), 1, 10)
    lib = KI._abi.load()
    st = lib.ki_vcopy_strided(KI.context(0).handle, buf.data_ptr() + 1, 1, f.data_ptr(), 1, 4, 10, None)
    assert st == KI._abi.KI_ERR_ARG  # misaligned element pointer
    KI.context(0).check()


def test_2d_large_column_block(KI, dev):
    """A 8192 x 32768-byte block between pitches 33000 and 40000 (0.27 GB moved): the destination
    view equals the source view and the bytes between rows are untouched."""
    import torch

    h, w = 8192, 32768
    src = torch.empty(h * 33000 + 16, dtype=torch.uint8, device=dev)
    KI.fill_bytes(src, seed=9)
    dst = torch.zeros(h * 40000 + 16, dtype=torch.uint8, device=dev)
    KI.vcopy_2d(dst, 40000, src, 33000, w, h, dst_offset=3, src_offset=11)
    sv = src[11:11 + h * 33000].view(h, 33000)[:, :w]
    dv = dst[3:3 + h * 40000].view(h, 40000)
    assert torch.equal(dv[:, :w], sv)
    assert int(dv[:, w:].count_nonzero()) == 0 and int(dst[:3].count_nonzero()) == 0
    KI.context(0).check()
