"""Shared pytest setup: import paths, the `gpu` marker and GPU fixtures."""
from __future__ import annotations

import json
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
PKG = REPO / "kernelintrinsics.jl_b200"
for p in (REPO, PKG, REPO / "oracle"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

GOLDEN = REPO / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU and the built libki_b200.so")


@pytest.fixture(scope="session")
def golden():
    return json.loads((GOLDEN / "reference_vectors.json").read_text())


@pytest.fixture(scope="session")
def base_semantics():
    import numpy as np

    return dict(np.load(GOLDEN / "base_semantics.npz"))


@pytest.fixture(scope="session")
def oracle():
    import ki_oracle

    ki_oracle.lib()
    return ki_oracle


@pytest.fixture(scope="session")
def KI():
    """The package on a GPU box; fails (does not skip) when the library or the GPU is missing."""
    import torch

    if not torch.cuda.is_available():
        pytest.fail("a GPU test ran without a CUDA device")
    import kernelintrinsics as KI

    KI.context(0)
    return KI


@pytest.fixture
def dev():
    import torch

    return torch.device("cuda", 0)
