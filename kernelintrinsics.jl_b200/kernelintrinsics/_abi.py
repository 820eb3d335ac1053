"""ctypes binding of libki_b200.so (the C ABI declared in include/ki_b200.h).

The library is built in-tree (``kernelintrinsics.jl_b200/lib/libki_b200.so``).  Loading fails
loudly when it is missing: there is no fallback implementation of any operation.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

PKG_ROOT = Path(__file__).resolve().parent.parent          # kernelintrinsics.jl_b200/
LIB_PATH = PKG_ROOT / "lib" / "libki_b200.so"

# ki_status
KI_OK, KI_ERR_ARG, KI_ERR_CUDA, KI_ERR_TIMEOUT, KI_ERR_UNSUPPORTED, KI_ERR_NOMEM, KI_ERR_NCCL = range(7)
KI_XCHG_AUTO, KI_XCHG_PEER, KI_XCHG_NCCL = range(3)
COMM_ID_BYTES = 128

# enums (include/ki_b200.h)
SCOPE = {"default": 0, "workgroup": 1, "device": 2, "system": 3}
ORDER = {"default": 0, "weak": 1, "volatile": 2, "relaxed": 3, "acquire": 4, "release": 5, "acqrel": 6,
         "seqcst": 7}
DIR = {"up": 0, "down": 1, "xor": 2, "idx": 3}
MODE = {"all": 0, "any": 1, "uni": 2, "ballot": 3}
DTYPE = {"int8": 0, "uint8": 1, "int16": 2, "uint16": 3, "int32": 4, "uint32": 5, "int64": 6, "uint64": 7,
         "float32": 8, "float64": 9}
OP = {"+": 0, "max": 1, "min": 2, "|": 3, "&": 4, "^": 5}

# Every symbol the header declares, with (restype, argtypes).
_vp, _sz, _i32, _i64, _u64, _f32 = (ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int, ctypes.c_int64,
                                    ctypes.c_uint64, ctypes.c_float)
SIGNATURES = {
    "ki_version": (_i32, []),
    "ki_status_string": (ctypes.c_char_p, [_i32]),
    "ki_device_count": (_i32, [ctypes.POINTER(_i32)]),
    "ki_device_info": (_i32, [_i32, ctypes.POINTER(_i32), ctypes.POINTER(_i32), ctypes.POINTER(_i32),
                              ctypes.POINTER(_i32)]),
    "ki_ctx_create": (_i32, [_i32, ctypes.POINTER(_vp)]),
    "ki_ctx_destroy": (_i32, [_vp]),
    "ki_last_error_string": (ctypes.c_char_p, [_vp]),
    "ki_ctx_check": (_i32, [_vp, _vp]),
    "ki_ctx_set_wait_timeout_ns": (_i32, [_vp, _u64]),
    "ki_vcopy": (_i32, [_vp, _vp, _vp, _sz, _vp]),
    "ki_vcopy_host": (_i32, [_vp, _vp, _vp, _sz, _vp]),
    "ki_vcopy_2d": (_i32, [_vp, _vp, _sz, _vp, _sz, _sz, _sz, _vp]),
    "ki_scan_rows": (_i32, [_vp, _i32, _i32, _i32, _vp, _sz, _vp, _sz, _sz, _sz, _vp, _vp]),
    "ki_mapreduce": (_i32, [_vp, _i32, _i32, _i32, _vp, _sz, _vp, _vp]),
    "ki_compact_map": (_i32, [_vp, _i32, _i32, _i32, _vp, _sz, _vp, _vp, _vp, _i64, _vp, _vp]),
    "ki_vcopy_strided": (_i32, [_vp, _vp, _i64, _vp, _i64, _sz, _sz, _vp]),
    "ki_reduce_sum_f32": (_i32, [_vp, _vp, _sz, _vp, _vp, _vp]),
    "ki_reduce_sum_i64": (_i32, [_vp, _vp, _sz, _vp, _vp]),
    "ki_scan_inclusive_i64": (_i32, [_vp, _vp, _vp, _sz, _i64, _vp]),
    "ki_scan_inclusive_i64_dseed": (_i32, [_vp, _vp, _vp, _sz, _vp, _vp]),
    "ki_scan_inclusive_i64_host": (_i32, [_vp, _vp, _vp, _sz, _i64, _vp]),
    "ki_scan_inclusive_i64_sharded_host": (_i32, [_vp, _vp, _vp, _sz, _vp]),
    "ki_comm_shard_range": (_i32, [_sz, _i32, _i32, ctypes.POINTER(_sz), ctypes.POINTER(_sz)]),
    "ki_comm_scan_shard_range": (_i32, [_sz, _i32, _i32, ctypes.POINTER(_sz), ctypes.POINTER(_sz)]),
    "ki_comm_get_id": (_i32, [_vp]),
    "ki_comm_init_rank": (_i32, [_i32, _i32, _i32, _vp, _i32, ctypes.POINTER(_vp)]),
    "ki_comm_create": (_i32, [_i32, ctypes.POINTER(_i32), ctypes.POINTER(_vp)]),
    "ki_comm_destroy": (_i32, [_vp]),
    "ki_comm_abort": (_i32, [_vp]),
    "ki_comm_info": (_i32, [_vp, ctypes.POINTER(_i32), ctypes.POINTER(_i32), ctypes.POINTER(_i32),
                            ctypes.POINTER(_i32)]),
    "ki_comm_get_ctx": (_i32, [_vp, ctypes.POINTER(_vp)]),
    "ki_reduce_sum_f32_sharded": (_i32, [_vp, _vp, _sz, _vp, _vp, _vp]),
    "ki_scan_inclusive_i64_sharded": (_i32, [_vp, _vp, _vp, _sz, _vp]),
    "ki_compact_gt_f32_sharded": (_i32, [_vp, _vp, _sz, _f32, _vp, _vp, _i64, _vp, _vp, _vp, _vp]),
    "ki_reduce": (_i32, [_vp, _i32, _i32, _vp, _sz, _vp, _vp]),
    "ki_compact": (_i32, [_vp, _i32, _i32, _vp, _sz, _vp, _vp, _vp, _i64, _vp, _vp]),
    "ki_reduce_rows": (_i32, [_vp, _i32, _i32, _vp, _sz, _sz, _sz, _vp, _vp]),
    "ki_scan": (_i32, [_vp, _i32, _i32, _i32, _vp, _vp, _sz, _vp, _vp]),
    "ki_scan_inclusive_i64_noalloc": (_i32, [_vp, _vp, _sz, _i64, _vp]),
    "ki_compact_gt_f32": (_i32, [_vp, _vp, _sz, _f32, _vp, _vp, _i64, _vp, _vp]),
    "ki_gemm_e4m3_f32": (_i32, [_vp, _vp, _vp, _vp, _i32, _i32, _i32, _f32, _f32, _vp]),
    "ki_warp_shfl": (_i32, [_vp, _i32, _vp, _vp, _sz, _sz, _i32, _vp]),
    "ki_warp_reduce": (_i32, [_vp, _i32, _i32, _vp, _vp, _sz, _vp]),
    "ki_warp_fold": (_i32, [_vp, _i32, _i32, _i32, _vp, _vp, _sz, _vp]),
    "ki_warp_vote": (_i32, [_vp, _i32, _vp, _vp, _sz, _vp]),
    "ki_vload": (_i32, [_vp, _vp, _sz, _i64, _i32, _i32, _vp, _vp]),
    "ki_vstore": (_i32, [_vp, _vp, _sz, _i64, _i32, _i32, _vp, _vp]),
    "ki_access_roundtrip": (_i32, [_vp, _i32, _i32, _i32, _i32, _i32, _i32, _vp, _vp, _vp, _vp]),
    "ki_flag_message_pass": (_i32, [_vp, _vp, _vp, _vp, _i32, _i64, _i32, _u64, _vp]),
    "ki_fill_uniform_f32": (_i32, [_vp, _u64, _vp, _sz, _vp]),
    "ki_fill_int_range_i64": (_i32, [_vp, _u64, _i64, _i64, _vp, _sz, _vp]),
    "ki_fill_bytes": (_i32, [_vp, _u64, _vp, _sz, _vp]),
    "ki_fill_normal_f32": (_i32, [_vp, _u64, _vp, _sz, _vp]),
    "ki_fill_e4m3_uniform": (_i32, [_vp, _u64, _f32, _vp, _sz, _vp]),
}

_lib = None


class KIError(RuntimeError):
    """A libki_b200 call returned a non-zero ki_status."""

    def __init__(self, status: int, message: str):
        super().__init__(f"[{status}] {message}")
        self.status = status


class KIArgumentError(KIError, ValueError):
    """KI_ERR_ARG: the reference raises ArgumentError for the same misuse."""


class KITimeoutError(KIError, TimeoutError):
    """KI_ERR_TIMEOUT: a bounded device-side wait ran out."""


def load(path: os.PathLike | None = None) -> ctypes.CDLL:
    """Load libki_b200.so and declare every exported signature.  Raises if it is missing."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = Path(path) if path else LIB_PATH
    if not p.exists():
        raise ImportError(f"libki_b200.so not found at {p}; build it with __graft_entry__.build() "
                          f"or `make -C {PKG_ROOT / 'csrc'}`")
    lib = ctypes.CDLL(str(p))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if path is None:
        _lib = lib
    return lib


def status_error(status: int, message: str) -> KIError:
    if status == KI_ERR_ARG:
        return KIArgumentError(status, message)
    if status == KI_ERR_TIMEOUT:
        return KITimeoutError(status, message)
    return KIError(status, message)
