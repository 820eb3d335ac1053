"""CPU: the C-ABI library loads and exports every entry point include/ki_b200.h declares."""
from __future__ import annotations

import ctypes
import re
import subprocess

from conftest import PKG, REPO


def declared_functions():
    text = (REPO / "include" / "ki_b200.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(?:int|const char\*)\s+(ki_\w+)\s*\(", text)))


def test_header_declares_the_abi():
    names = declared_functions()
    for must in ("ki_vcopy", "ki_reduce_sum_f32", "ki_scan_inclusive_i64", "ki_compact_gt_f32", "ki_gemm_e4m3_f32",
                 "ki_ctx_create", "ki_ctx_check", "ki_warp_shfl", "ki_warp_vote"):
        assert must in names


def test_library_exports_every_declared_symbol():
    from kernelintrinsics import _abi

    lib = _abi.load()
    out = subprocess.run(["nm", "-D", "--defined-only", str(_abi.LIB_PATH)], capture_output=True, text=True,
                         check=True).stdout
    exported = set(re.findall(r"\sT\s+(ki_\w+)", out))
    missing = [n for n in declared_functions() if n not in exported]
    assert not missing, missing
    for n in declared_functions():
        assert hasattr(lib, n)
    # the Python binding declares a signature for every entry point
    assert set(_abi.SIGNATURES) == set(declared_functions())


def test_library_is_sm100a_only():
    from kernelintrinsics import _abi

    out = subprocess.run(["cuobjdump", "--list-elf", str(_abi.LIB_PATH)], capture_output=True, text=True).stdout
    archs = set(re.findall(r"sm_(\d+a?)", out))
    assert archs == {"100a"}, archs


def test_host_only_calls():
    from kernelintrinsics import _abi

    lib = _abi.load()
    assert lib.ki_version() >= 100
    assert b"KI_ERR_TIMEOUT" in lib.ki_status_string(3)
    # a null context is rejected without touching the GPU
    assert lib.ki_vcopy(None, None, None, 16, None) == _abi.KI_ERR_ARG
    assert lib.ki_ctx_check(None, None) == _abi.KI_ERR_ARG


def test_package_has_no_cpu_path():
    import kernelintrinsics as KI
    import pytest
    import torch

    with pytest.raises(KI.KIArgumentError):
        KI.warpreduce_scan(torch.zeros(64, dtype=torch.int64))
