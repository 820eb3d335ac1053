"""GPU: fp8 e4m3 tcgen05 GEMM against the Float64 oracle GEMM of the dequantised operands.

Tolerance (stated by the workload definition): relative Frobenius error <= 1e-3.
"""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = 1e-3


def _operands(KI, dev, M, N, K, sa=5, sb=6):
    import torch

    A = torch.empty((M, K), dtype=torch.uint8, device=dev)
    B = torch.empty((K, N), dtype=torch.uint8, device=dev)
    KI.fill_e4m3_uniform(A, seed=sa, scale=112.0)
    KI.fill_e4m3_uniform(B, seed=sb, scale=112.0)
    return A, B


def _relfro(C, R):
    return float(np.linalg.norm(C - R) / np.linalg.norm(R))


@pytest.mark.parametrize("M,N,K", [(128, 256, 128), (256, 256, 256), (128, 512, 1024), (384, 768, 640),
                                   (1024, 1024, 512), (2048, 2048, 2048)])
def test_gemm_vs_oracle(KI, oracle, dev, M, N, K):
    A, B = _operands(KI, dev, M, N, K)
    C = KI.fp8_gemm(A, B)
    KI.context(0).check()
    R = oracle.gemm_e4m3_rows(A.cpu().numpy(), B.cpu().numpy(), 0, M)
    Cn = C.cpu().numpy().astype(np.float64)
    assert np.isfinite(Cn).all()
    err = _relfro(Cn, R)
    assert err <= TOL, err
    # every output tile was written (no stale memory): elementwise check, loose
    assert np.allclose(Cn, R, rtol=1e-3, atol=1e-2 * np.abs(R).max())


def test_gemm_scales_and_reuse(KI, oracle, dev):
    import torch

    M, N, K = 256, 512, 256
    A, B = _operands(KI, dev, M, N, K, 7, 8)
    C = torch.full((M, N), float("nan"), dtype=torch.float32, device=dev)
    KI.fp8_gemm(A, B, C, scale_a=0.5, scale_b=0.25)
    R = oracle.gemm_e4m3_rows(A.cpu().numpy(), B.cpu().numpy(), 0, M, scale=0.125)
    assert _relfro(C.cpu().numpy().astype(np.float64), R) <= TOL
    for _ in range(5):  # repeated launches give the same bits
        C2 = KI.fp8_gemm(A, B, scale_a=0.5, scale_b=0.25)
        assert torch.equal(C, C2)


def test_gemm_rejects_bad_shapes(KI, dev):
    import torch

    A = torch.zeros((128, 100), dtype=torch.uint8, device=dev)
    B = torch.zeros((100, 256), dtype=torch.uint8, device=dev)
    with pytest.raises(KI.KIArgumentError):
        KI.fp8_gemm(A, B)
    A = torch.zeros((100, 128), dtype=torch.uint8, device=dev)
    B = torch.zeros((128, 256), dtype=torch.uint8, device=dev)
    with pytest.raises(KI.KIArgumentError):
        KI.fp8_gemm(A, B)


def test_gemm_config_size_sampled_rows(KI, oracle, dev):
    """M = N = K = 8192: rows from every 128-row tile band checked against the Float64 oracle."""
    import torch

    M = N = K = 8192
    A, B = _operands(KI, dev, M, N, K)
    C = KI.fp8_gemm(A, B)
    KI.context(0).check()
    An, Bn = A.cpu().numpy(), B.cpu().numpy()
    rng = np.random.default_rng(0)
    rows = sorted(set([0, 127, 128, M - 1] + list(rng.integers(0, M, 28))))
    Cn = C.cpu().numpy()
    num = den = 0.0
    for r in rows:
        R = oracle.gemm_e4m3_rows(An, Bn, r, r + 1)[0]
        d = Cn[r].astype(np.float64) - R
        num += float(d @ d)
        den += float(R @ R)
    assert (num / den) ** 0.5 <= TOL
    assert torch.isfinite(C).all()
    del A, B, C
    torch.cuda.empty_cache()
