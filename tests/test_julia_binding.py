"""CPU: the Julia binding (kernelintrinsics.jl_b200/julia/KernelIntrinsicsB200.jl) against the C ABI.

Julia is not installed here, so the module cannot be run; this test parses every
``ccall((:ki_..., libki), Ret, (Types...), args...)`` in it and checks, against include/ki_b200.h,
that the symbol is declared, the return type and the number of arguments match, and that each
argument type is of the same class as the C parameter (pointer, int, size_t, int64_t, uint64_t,
float).  It also checks that no CuPtr argument is given a host C_NULL (CUDA.jl refuses that
conversion) and that every hot-path entry of the reference has a mirror.
"""
from __future__ import annotations

import re

from conftest import PKG, REPO

JL = PKG / "julia" / "KernelIntrinsicsB200.jl"


def _split_top(s: str) -> list:
    out, depth, cur = [], 0, ""
    for ch in s:
        if ch in "({[":
            depth += 1
        elif ch in ")}]":
            depth -= 1
        if ch == "," and depth == 0:
            out.append(cur.strip())
            cur = ""
        else:
            cur += ch
    if cur.strip():
        out.append(cur.strip())
    return out


def _balanced(s: str, i: int) -> int:
    """Index just past the bracket group that opens at s[i]."""
    depth = 0
    for j in range(i, len(s)):
        if s[j] in "({[":
            depth += 1
        elif s[j] in ")}]":
            depth -= 1
            if depth == 0:
                return j + 1
    raise ValueError("unbalanced")


def header_decls() -> dict:
    text = (REPO / "include" / "ki_b200.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    decls = {}
    for m in re.finditer(r"\b(int|const char\*)\s+(ki_\w+)\s*\(([^)]*)\)\s*;", text):
        ret, name, params = m.group(1), m.group(2), m.group(3).strip()
        kinds = []
        if params and params != "void":
            for p in _split_top(params):
                if "*" in p:
                    kinds.append("ptr")
                else:
                    base = p.replace("const ", "").split()[0]
                    kinds.append({"int": "int", "size_t": "size_t", "int64_t": "int64_t", "uint64_t": "uint64_t",
                                  "float": "float"}[base])
        decls[name] = ("int" if ret == "int" else "ptr", kinds)
    return decls


def _jl_kind(t: str) -> str:
    t = t.strip()
    if t.startswith(("Ptr{", "CuPtr{", "Ref{")) or t == "Cstring":
        return "ptr"
    return {"Cint": "int", "Csize_t": "size_t", "Int64": "int64_t", "UInt64": "uint64_t", "Float32": "float"}[t]


def julia_ccalls() -> list:
    src = JL.read_text()
    src = re.sub(r"#.*", "", src)  # comments
    calls = []
    for m in re.finditer(r"ccall\(\(:(ki_\w+),\s*libki\)\s*,", src):
        name = m.group(1)
        open_paren = src.rfind("(", 0, m.start() + len("ccall("))
        end = _balanced(src, open_paren)
        body = src[open_paren + 1:end - 1]
        parts = _split_top(body)
        ret, types = parts[1], parts[2]
        assert types.startswith("(") and types.endswith(")"), (name, types)
        tlist = _split_top(types[1:-1])
        calls.append((name, ret, tlist, parts[3:]))
    return calls


def test_every_ccall_matches_the_header():
    decls = header_decls()
    calls = julia_ccalls()
    assert len(calls) >= 40
    for name, ret, types, args in calls:
        assert name in decls, f"{name} is not declared in include/ki_b200.h"
        cret, ckinds = decls[name]
        assert _jl_kind(ret) == cret or (ret == "Cint" and cret == "int"), (name, ret)
        jk = [_jl_kind(t) for t in types]
        assert jk == ckinds, f"{name}: Julia {jk} vs C {ckinds}"
        assert len(args) == len(types), f"{name}: {len(args)} arguments for {len(types)} types"
        for t, a in zip(types, args):
            if t.startswith("CuPtr"):
                assert a.strip() != "C_NULL", f"{name}: C_NULL given for {t} (use CuPtr{{T}}(0))"


def test_hot_path_entries_have_mirrors():
    src = JL.read_text()
    bound = {c[0] for c in julia_ccalls()}
    for sym in ("ki_reduce_sum_f32", "ki_scan_inclusive_i64", "ki_compact_gt_f32", "ki_vcopy", "ki_vcopy_host",
                "ki_gemm_e4m3_f32", "ki_warp_shfl", "ki_warp_reduce", "ki_warp_fold", "ki_warp_vote", "ki_vload",
                "ki_vstore", "ki_access_roundtrip", "ki_reduce", "ki_scan", "ki_compact_map", "ki_comm_init_rank",
                "ki_comm_create", "ki_reduce_sum_f32_sharded", "ki_scan_inclusive_i64_sharded",
                "ki_compact_gt_f32_sharded", "ki_scan_inclusive_i64_noalloc"):
        assert sym in bound, sym
    # reference names (src/KernelIntrinsics.jl:5-10, src/warp.jl, src/vectorization.jl, src/device.jl)
    for fn in ("get_warpsize", "devices", "deviceid", "shfl!", "warpreduce!", "warpfold!", "vote!", "vload",
               "vstore!", "warpfold_reduce", "warpreduce_scan!", "vote_compact", "vcopy!", "fp8_gemm!"):
        assert re.search(rf"\bfunction {re.escape(fn)}\(|^{re.escape(fn)}\(", src, flags=re.M), fn
    for ty in ("Workgroup", "Device", "System", "Acquire", "Release", "AcqRel", "SeqCst", "Up", "Down", "Xor",
               "Idx", "All", "AnyLane", "Uni", "Ballot"):
        assert re.search(rf"struct {ty} <:", src), ty


def test_library_path_points_at_the_in_tree_build():
    src = JL.read_text()
    assert 'joinpath(@__DIR__, "..", "lib", "libki_b200.so")' in src
    assert (JL.parent / ".." / "lib").resolve() == (PKG / "lib").resolve()
