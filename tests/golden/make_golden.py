"""Writes tests/golden/reference_vectors.json: the known answers of KernelIntrinsics.jl's own tests.

Every case restates one @test of the reference (epilliat/KernelIntrinsics.jl v0.1.6) with its
inputs and expected outputs, citing the file:line it comes from.  Julia indices are kept 1-based
in the fixture ("index_1based"); consumers convert.  Warp size is 32 (CUDA).

Also writes tests/golden/base_semantics.npz: small seeded inputs with outputs computed by numpy,
an implementation of the Julia Base semantics (sum, cumsum, findall/filter, copyto!) independent of
the C oracle, used to pin the oracle.

Run:  python tests/golden/make_golden.py
"""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
WS = 32


def shfl_cases():
    r = list(range(1, WS + 1))
    cases = [
        {"name": "Up Int32", "src": "test/tests/shfl.jl:70-75", "dir": "up", "arg": 1, "dtype": "int32",
         "input": r, "expected": [1] + r[:-1]},
        {"name": "Down Int32", "src": "test/tests/shfl.jl:77-82", "dir": "down", "arg": 1, "dtype": "int32",
         "input": r, "expected": r[1:] + [WS]},
        {"name": "Idx Int32", "src": "test/tests/shfl.jl:84-89", "dir": "idx", "arg": 1, "dtype": "int32",
         "input": r, "expected": [1] * WS},
        {"name": "Up Float32", "src": "test/tests/shfl.jl:91-96", "dir": "up", "arg": 1, "dtype": "float32",
         "input": r, "expected": [1] + r[:-1]},
        {"name": "Up Float64", "src": "test/tests/shfl.jl:98-103", "dir": "up", "arg": 1, "dtype": "float64",
         "input": r, "expected": [1] + r[:-1]},
        {"name": "Up Float16", "src": "test/tests/shfl.jl:105-110", "dir": "up", "arg": 1, "dtype": "float16",
         "input": r, "expected": [1] + r[:-1]},
    ]
    return cases


def shfl_struct_cases():
    # NTuple{2,Int32}: (i, i+100) -> lane 1 keeps (1,101), lane i gets (i-1, i+99)  (shfl.jl:112-125)
    tup_in = [[i, i + 100] for i in range(1, WS + 1)]
    tup_out = [[1, 101]] + [[i - 1, i + 99] for i in range(2, WS + 1)]
    # ComplexType(x::Int32, y::SubType(a::Float16, b::UInt8), z::Float64)  (shfl.jl:2-11,127-136)
    # Julia layout: x @0 (4 B), y @4 (Float16 @4, UInt8 @6, size 4), z @8 (8 B) -> 16 bytes.
    cpx_in = [[i, i, i, float(i)] for i in range(1, WS + 1)]
    cpx_out = [[1, 1, 1, 1.0]] + [[i - 1, i - 1, i - 1, float(i - 1)] for i in range(2, WS + 1)]
    return [
        {"name": "Up NTuple{2,Int32}", "src": "test/tests/shfl.jl:112-125", "dir": "up", "arg": 1,
         "layout": [["int32", 0], ["int32", 4]], "size": 8, "input": tup_in, "expected": tup_out},
        {"name": "Up ComplexType", "src": "test/tests/shfl.jl:127-136", "dir": "up", "arg": 1,
         "layout": [["int32", 0], ["float16", 4], ["uint8", 6], ["float64", 8]], "size": 16,
         "input": cpx_in, "expected": cpx_out},
    ]


def warp_cases():
    r = list(range(1, WS + 1))
    return [
        {"name": "@warpreduce Int32 prefix sum", "src": "test/tests/shfl.jl:150-155", "dtype": "int32",
         "input": r, "expected": list(np.cumsum(r).tolist()), "exact": True},
        {"name": "@warpreduce Float32 prefix sum", "src": "test/tests/shfl.jl:157-163", "dtype": "float32",
         "input": r, "expected": list(np.cumsum(r).tolist()), "exact": False},
        {"name": "@warpfold Int32 sum (lane 1)", "src": "test/tests/shfl.jl:177-182", "dtype": "int32",
         "input": r, "expected_lane1": 528},
    ]


def vote_cases():
    any_in = [0] * WS
    any_in[-1] = 200
    return [
        {"name": "All", "src": "test/tests/shfl.jl:209-214", "mode": "all", "input": [10] * WS, "threshold": 5,
         "expected": [True] * WS},
        {"name": "AnyLane", "src": "test/tests/shfl.jl:216-223", "mode": "any", "input": any_in,
         "threshold": 100, "expected": [True] * WS},
        {"name": "Uni", "src": "test/tests/shfl.jl:225-230", "mode": "uni", "input": [10] * WS, "threshold": 5,
         "expected": [True] * WS},
    ]


def vector_cases():
    a16 = list(range(1, 17))
    c = []
    # vload (test/tests/cuda/vectorization_test.jl)
    c.append({"name": "vload rebase Int32", "src": "test/tests/cuda/vectorization_test.jl:19-35", "op": "vload",
              "dtype": "int32", "array": a16, "view_offset": 0, "index_1based": 2, "nitem": 4, "rebase": True,
              "expected": [5, 6, 7, 8], "expected_sum": 26})
    c.append({"name": "vload norebase Int32", "src": "test/tests/cuda/vectorization_test.jl:37-48", "op": "vload",
              "dtype": "int32", "array": a16, "view_offset": 0, "index_1based": 3, "nitem": 4, "rebase": False,
              "expected": [3, 4, 5, 6], "expected_sum": 18})
    for shift in range(1, 17):
        c.append({"name": f"vload_multi N=16 shift {shift}", "src": "test/tests/cuda/vectorization_test.jl:84-91",
                  "op": "vload", "dtype": "int32", "array": list(range(1, 101)), "view_offset": 0,
                  "index_1based": shift, "nitem": 16, "rebase": False,
                  "expected": list(range(shift, shift + 16))})
    # vstore
    c.append({"name": "vstore rebase Int32", "src": "test/tests/cuda/vectorization_test.jl:96-111", "op": "vstore",
              "dtype": "int32", "length": 16, "view_offset": 0, "index_1based": 2, "rebase": True,
              "values": [10, 20, 30, 40], "expected_at_1based": {"5": 10, "6": 20, "7": 30, "8": 40}})
    c.append({"name": "vstore norebase Int32", "src": "test/tests/cuda/vectorization_test.jl:113-123",
              "op": "vstore", "dtype": "int32", "length": 16, "view_offset": 0, "index_1based": 3, "rebase": False,
              "values": [100, 200, 300, 400], "expected_at_1based": {"3": 100, "4": 200, "5": 300, "6": 400}})
    c.append({"name": "vstore_multi Int32", "src": "test/tests/cuda/vectorization_test.jl:142-157",
              "op": "vstore", "dtype": "int32", "length": 100, "view_offset": 0, "index_1based": 2, "rebase": False,
              "values": [10, 20, 30, 40], "expected_at_1based": {"2": 10, "3": 20, "4": 30, "5": 40}})
    c.append({"name": "roundtrip rebase Int32", "src": "test/tests/cuda/vectorization_test.jl:160-171",
              "op": "roundtrip", "dtype": "int32", "array": a16, "view_offset": 0, "index_1based": 2, "nitem": 4,
              "rebase": True, "expected_at_1based": {"5": 5, "6": 6, "7": 7, "8": 8}})
    # contiguous views (view offset = elements skipped before the view)
    for off, exp_sum in ((1, 14), (2, 18)):
        for rebase, lines in ((False, "176-196"), (True, "198-218")):
            c.append({"name": f"vload view offset {off} rebase={rebase}",
                      "src": f"test/tests/cuda/vectorization_test.jl:{lines}", "op": "vload", "dtype": "int32",
                      "array": a16, "view_offset": off, "index_1based": 1, "nitem": 4, "rebase": rebase,
                      "expected": list(range(off + 1, off + 5)), "expected_sum": exp_sum})
        for rebase, lines in ((False, "220-239"), (True, "241-260")):
            c.append({"name": f"vstore view offset {off} rebase={rebase}",
                      "src": f"test/tests/cuda/vectorization_test.jl:{lines}", "op": "vstore", "dtype": "int32",
                      "length": 16, "view_offset": off, "index_1based": 1, "rebase": rebase,
                      "values": [10, 20, 30, 40],
                      "expected_at_1based": {str(off + 1 + k): v for k, v in enumerate([10, 20, 30, 40])}})
        c.append({"name": f"roundtrip view offset {off}", "src": "test/tests/cuda/vectorization_test.jl:262-285",
                  "op": "roundtrip", "dtype": "int32", "array": a16, "view_offset": off, "index_1based": 1,
                  "nitem": 4, "rebase": False,
                  "expected_at_1based": {str(off + 1 + k): off + 1 + k for k in range(4)}})
    # UInt8
    u16 = list(range(1, 17))
    c.append({"name": "vload UInt8 rebase", "src": "test/tests/cuda/vectorization_test.jl:404-410", "op": "vload",
              "dtype": "uint8", "array": u16, "view_offset": 0, "index_1based": 1, "nitem": 4, "rebase": True,
              "expected": [1, 2, 3, 4]})
    c.append({"name": "vload UInt8 norebase", "src": "test/tests/cuda/vectorization_test.jl:412-425",
              "op": "vload", "dtype": "uint8", "array": u16, "view_offset": 0, "index_1based": 3, "nitem": 4,
              "rebase": False, "expected": [3, 4, 5, 6]})
    c.append({"name": "vstore UInt8 rebase", "src": "test/tests/cuda/vectorization_test.jl:427-432",
              "op": "vstore", "dtype": "uint8", "length": 16, "view_offset": 0, "index_1based": 1, "rebase": True,
              "values": [10, 20, 30, 40], "expected_at_1based": {"1": 10, "2": 20, "3": 30, "4": 40}})
    c.append({"name": "vload UInt8 rebase view offset 1", "src": "test/tests/cuda/vectorization_test.jl:434-441",
              "op": "vload", "dtype": "uint8", "array": u16, "view_offset": 1, "index_1based": 1, "nitem": 4,
              "rebase": True, "expected": [2, 3, 4, 5]})
    c.append({"name": "vload UInt8 rebase view offset 3", "src": "test/tests/cuda/vectorization_test.jl:443-450",
              "op": "vload", "dtype": "uint8", "array": u16, "view_offset": 3, "index_1based": 1, "nitem": 4,
              "rebase": True, "expected": [4, 5, 6, 7]})
    c.append({"name": "vload UInt8 norebase view offset 1",
              "src": "test/tests/cuda/vectorization_test.jl:452-466", "op": "vload", "dtype": "uint8",
              "array": u16, "view_offset": 1, "index_1based": 1, "nitem": 4, "rebase": False,
              "expected": [2, 3, 4, 5]})
    c.append({"name": "vstore UInt8 view offset 1", "src": "test/tests/cuda/vectorization_test.jl:468-474",
              "op": "vstore", "dtype": "uint8", "length": 16, "view_offset": 1, "index_1based": 1, "rebase": True,
              "values": [10, 20, 30, 40], "expected_at_1based": {"2": 10, "3": 20, "4": 30, "5": 40}})
    c.append({"name": "vload UInt8 32 threads rebase", "src": "test/tests/cuda/vectorization_test.jl:476-491",
              "op": "vload_threads", "dtype": "uint8", "array": list(range(1, 129)), "threads": 32, "nitem": 4,
              "expected": list(range(1, 129))})
    return c


def custom_struct_cases():
    """test/tests/vectorization_custom_test.jl: records with their Julia byte layouts."""
    return [
        {"name": "Vec3_1 (12 B, scalar path)", "src": "test/tests/vectorization_custom_test.jl:38-83",
         "layout": [["float32", 0], ["float32", 4], ["float32", 8]], "size": 12,
         "array": [[i, i + 10, i + 20] for i in range(1, 17)],
         "load_view_offset": 2,
         "stored": [[1, 2, 3], [4, 5, 6], [7, 8, 9], [10, 11, 12]]},
        {"name": "S6 (6 B, scalar path)", "src": "test/tests/vectorization_custom_test.jl:85-132",
         "layout": [["float16", 0], ["float16", 2], ["float16", 4]], "size": 6,
         "array": [[i, i + 10, i + 20] for i in range(1, 17)],
         "load_view_offset": 1,
         "stored": [[1, 2, 3], [4, 5, 6], [7, 8, 9], [10, 11, 12]]},
        {"name": "Vec3_2 (16 B, vector path)", "src": "test/tests/vectorization_custom_test.jl:134-181",
         "layout": [["uint8", 0], ["float16", 2], ["uint8", 4], ["float32", 8], ["float32", 12]], "size": 16,
         "array": [[i, i + 10, i + 20, i + 30, i + 40] for i in range(1, 17)],
         "load_view_offset": 1,
         "stored": [[1, 2, 3, 4, 5], [6, 7, 8, 9, 10], [11, 12, 13, 14, 15], [16, 17, 18, 19, 20]]},
        {"name": "TupleStruct (4 B)", "src": "test/tests/vectorization_custom_test.jl:183-227",
         "layout": [["float16", 0], ["uint8", 2]], "size": 4,
         "array": [[i, i + 10] for i in range(1, 17)],
         "load_view_offset": 1,
         "stored": [[1, 2], [3, 4], [5, 6], [7, 8]]},
    ]


def access_cases():
    return [
        {"name": "@access multi-dim store data[2,2] = 0x20", "src": "test/tests/cuda/access_fences.jl:47-54",
         "shape": [50, 50], "index_1based": [2, 2], "value": 32, "dtype": "uint8",
         "linear_index_1based": 2 + (2 - 1) * 50},
    ]


def patterns():
    # generate_partN examples stated in the reference's docs / tests
    return [
        {"N": 4, "residue": 1, "pattern": [1, 2, 1], "src": "test/tests/cuda/vectorization_test.jl:50-65"},
        {"N": 4, "residue": 2, "pattern": [2, 2], "src": "src/vectorization.jl:306-338"},
        {"N": 16, "residue": 1, "pattern": [1, 2, 4, 8, 1], "src": "src/vectorization.jl:306-338"},
        {"N": 16, "residue": 8, "pattern": [8, 8], "src": "src/vectorization.jl:306-338"},
    ]


def base_semantics():
    rng = np.random.default_rng(20261201)
    x32 = rng.random(4099, dtype=np.float32)
    i64 = rng.integers(-1000, 1001, size=5003, dtype=np.int64)
    big = np.array([2**62, 2**62, 2**62, -5, 7], dtype=np.int64)  # wraps like Julia Int64
    with np.errstate(over="ignore"):
        big_cs = np.cumsum(big.astype(np.uint64)).astype(np.int64)
    nrm = rng.standard_normal(6007).astype(np.float32)
    keep = np.nonzero(nrm > np.float32(0.5))[0]
    return {
        "sum_x": x32, "sum_f64": np.array([x32.astype(np.float64).sum()]),
        "scan_x": i64, "scan_y": np.cumsum(i64),
        "wrap_x": big, "wrap_y": big_cs,
        "filt_x": nrm, "filt_vals": nrm[keep], "filt_idx1": (keep + 1).astype(np.int32),
    }


def main():
    doc = {
        "reference": "epilliat/KernelIntrinsics.jl v0.1.6",
        "warpsize": WS,
        "shfl": shfl_cases(),
        "shfl_struct": shfl_struct_cases(),
        "warp": warp_cases(),
        "vote": vote_cases(),
        "vector": vector_cases(),
        "custom_struct": custom_struct_cases(),
        "access": access_cases(),
        "patterns": patterns(),
    }
    (HERE / "reference_vectors.json").write_text(json.dumps(doc, indent=1) + "\n")
    np.savez_compressed(HERE / "base_semantics.npz", **base_semantics())
    print("wrote", HERE / "reference_vectors.json", HERE / "base_semantics.npz")


if __name__ == "__main__":
    main()
