"""GPU: the warp-level intrinsics against the reference's own known answers and the oracle."""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

NP = {"int8": np.int8, "uint8": np.uint8, "int16": np.int16, "uint16": np.uint16, "int32": np.int32,
      "uint32": np.uint32, "int64": np.int64, "uint64": np.uint64, "float16": np.float16,
      "float32": np.float32, "float64": np.float64}
TORCH = None


def _t(dtype):
    import torch

    return getattr(torch, dtype)


def _records(rows, layout, size):
    """Pack a list of field tuples into bytes with the given (dtype, offset) layout."""
    buf = np.zeros((len(rows), size), dtype=np.uint8)
    for r, fields in enumerate(rows):
        for (dt, off), v in zip(layout, fields):
            b = np.array([v], dtype=NP[dt]).view(np.uint8)
            buf[r, off:off + b.size] = b
    return buf


def test_shfl_golden(KI, golden, dev):
    import torch

    for c in golden["shfl"]:
        x = torch.tensor(c["input"], dtype=_t(c["dtype"]), device=dev)
        d = {"up": KI.Up, "down": KI.Down, "xor": KI.Xor, "idx": KI.Idx}[c["dir"]]
        got = KI.shfl(d, x, c["arg"]).cpu().tolist()
        assert got == c["expected"], c["name"]


def test_shfl_struct_golden(KI, golden, dev):
    import torch

    for c in golden["shfl_struct"]:
        src = _records(c["input"], c["layout"], c["size"])
        want = _records(c["expected"], c["layout"], c["size"])
        out = KI.shfl(KI.Up, torch.from_numpy(src).to(dev), c["arg"]).cpu().numpy()
        assert np.array_equal(out, want), c["name"]


@pytest.mark.parametrize("esz", [1, 2, 3, 4, 6, 8, 12, 16, 24, 40, 64])
@pytest.mark.parametrize("direction", ["up", "down", "xor", "idx"])
def test_shfl_any_size_vs_oracle(KI, oracle, dev, esz, direction):
    import torch

    rng = np.random.default_rng(esz * 7 + len(direction))
    rows = rng.integers(0, 256, size=(64, esz), dtype=np.uint8)  # two warps
    d = {"up": KI.Up, "down": KI.Down, "xor": KI.Xor, "idx": KI.Idx}[direction]
    for arg in ([1, 2, 5, 16, 31] if direction != "idx" else [1, 7, 32]):
        got = KI.shfl(d, torch.from_numpy(rows).to(dev), arg).cpu().numpy()
        for w in range(2):
            lanes = [bytes(rows[w * 32 + l]) for l in range(32)]
            want = oracle.shfl(direction, lanes, arg)
            assert [bytes(got[w * 32 + l]) for l in range(32)] == want, (esz, direction, arg)


def test_warpreduce_golden(KI, golden, dev):
    import torch

    for c in golden["warp"]:
        x = torch.tensor(c["input"], dtype=_t(c["dtype"]), device=dev)
        if "expected" in c:
            got = KI.warpreduce(x, "+").cpu().numpy()
            want = np.array(c["expected"], dtype=got.dtype)
            if c["exact"]:
                assert np.array_equal(got, want), c["name"]
            else:
                assert np.allclose(got, want, rtol=1e-6), c["name"]
        else:
            assert KI.warpfold(x, "+", form="down").cpu()[0].item() == c["expected_lane1"]
            assert (KI.warpfold(x, "+", form="xor").cpu() == c["expected_lane1"]).all()


OPS = {"+": lambda a, b: a + b, "max": max, "min": min, "|": lambda a, b: a | b, "&": lambda a, b: a & b,
       "^": lambda a, b: a ^ b}


@pytest.mark.parametrize("dtype", ["int8", "uint8", "int16", "uint16", "int32", "uint32", "int64", "uint64",
                                   "float32", "float64"])
def test_warp_scan_fold_vs_oracle(KI, oracle, dev, dtype):
    import torch

    rng = np.random.default_rng(len(dtype))
    npdt = NP[dtype]
    if np.issubdtype(npdt, np.integer):
        info = np.iinfo(npdt)
        x = rng.integers(max(info.min, -50), min(info.max, 50), size=96).astype(npdt)
        ops = ["+", "max", "min", "|", "&", "^"]
    else:
        x = rng.integers(-50, 50, size=96).astype(npdt)  # small integers: every order gives exact sums
        ops = ["+", "max", "min"]
    xt = torch.from_numpy(x).to(dev)
    for op in ops:
        f = OPS[op]

        def cast(v):
            return npdt(v) if np.issubdtype(npdt, np.floating) else np.array(v).astype(npdt)[()]

        def fop(a, b):
            with np.errstate(over="ignore"):
                return cast(f(a, b))

        scan = KI.warpreduce(xt, op).cpu().numpy()
        down = KI.warpfold(xt, op, form="down").cpu().numpy()
        xor = KI.warpfold(xt, op, form="xor").cpu().numpy()
        for w in range(3):
            lanes = list(x[w * 32:(w + 1) * 32])
            assert np.array_equal(scan[w * 32:(w + 1) * 32], np.array(oracle.warpreduce(lanes, fop), npdt)), op
            assert np.array_equal(down[w * 32:(w + 1) * 32], np.array(oracle.warpfold_down(lanes, fop), npdt)), op
            tot = oracle.warpreduce(lanes, fop)[-1]
            assert np.all(xor[w * 32:(w + 1) * 32] == tot), op


def test_vote_golden_and_ballot(KI, oracle, golden, dev):
    import torch

    modes = {"all": KI.All, "any": KI.AnyLane, "uni": KI.Uni, "ballot": KI.Ballot}
    for c in golden["vote"]:
        p = torch.tensor([v > c["threshold"] for v in c["input"]], device=dev)
        got = KI.vote(modes[c["mode"]], p).cpu().numpy()
        assert [bool(g) for g in got] == c["expected"], c["name"]
    rng = np.random.default_rng(3)
    for trial in range(20):
        pr = rng.random(64) < rng.random()
        if trial == 0:
            pr[:] = True
        if trial == 1:
            pr[:] = False
        p = torch.from_numpy(pr).to(dev)
        for m in modes:
            got = KI.vote(modes[m], p).cpu().numpy().astype(np.uint64)
            for w in range(2):
                want = oracle.vote(m, list(pr[w * 32:(w + 1) * 32]))
                assert list(got[w * 32:(w + 1) * 32]) == [int(v) for v in want], m


def _view(a, off, dev):
    import torch

    return torch.tensor(a, device=dev)[off:]


def test_vector_golden(KI, golden, dev):
    import torch

    for c in golden["vector"]:
        dt = _t(c["dtype"])
        if c["op"] == "vload":
            base = torch.tensor(c["array"], dtype=dt, device=dev)
            a = base[c["view_offset"]:]
            got = KI.vload(a, c["index_1based"], c["nitem"], rebase=c["rebase"]).cpu().tolist()
            assert got == c["expected"], c["name"]
            if "expected_sum" in c:
                assert sum(got) == c["expected_sum"], c["name"]
        elif c["op"] == "vstore":
            base = torch.zeros(c["length"], dtype=dt, device=dev)
            a = base[c["view_offset"]:]
            KI.vstore(a, c["index_1based"], torch.tensor(c["values"], dtype=dt, device=dev), rebase=c["rebase"])
            host = base.cpu().tolist()
            for k, v in c["expected_at_1based"].items():
                assert host[int(k) - 1] == v, c["name"]
            assert sum(1 for v in host if v) == len(c["expected_at_1based"]), c["name"]
        elif c["op"] == "roundtrip":
            src = torch.tensor(c["array"], dtype=dt, device=dev)[c["view_offset"]:]
            dbase = torch.zeros(len(c["array"]), dtype=dt, device=dev)
            d = dbase[c["view_offset"]:]
            vals = KI.vload(src, c["index_1based"], c["nitem"], rebase=c["rebase"])
            KI.vstore(d, c["index_1based"], vals, rebase=c["rebase"])
            host = dbase.cpu().tolist()
            for k, v in c["expected_at_1based"].items():
                assert host[int(k) - 1] == v, c["name"]
        elif c["op"] == "vload_threads":
            a = torch.tensor(c["array"], dtype=dt, device=dev)
            got = []
            for i in range(1, c["threads"] + 1):
                got += KI.vload(a, i, c["nitem"]).cpu().tolist()
            assert got == c["expected"], c["name"]


def test_vload_multi_every_alignment(KI, oracle, dev):
    """Every (element size, N, base misalignment, start) against the oracle's piece layout."""
    import torch

    rng = np.random.default_rng(11)
    raw = torch.from_numpy(rng.integers(0, 256, size=4096, dtype=np.uint8)).to(dev)
    for esz in (1, 2, 4, 8, 16):
        for N in (1, 2, 4, 8, 16):
            for off_elems in range(0, 17):
                a = raw[off_elems * esz:]  # element-aligned, N-misaligned in every way
                for i in (1, 2, 3, 5, 9):
                    got = KI.vload(a, i, N, rebase=False, elem_bytes=esz).cpu().numpy().reshape(-1)
                    want = raw.cpu().numpy()[(off_elems + i - 1) * esz:(off_elems + i - 1 + N) * esz]
                    assert np.array_equal(got, want), (esz, N, off_elems, i)


def test_vstore_multi_every_alignment(KI, dev):
    import torch

    for esz in (1, 4, 8):
        for N in (2, 4, 16):
            for off in range(0, 17):
                base = torch.zeros(2048, dtype=torch.uint8, device=dev)
                a = base[off * esz:]
                vals = torch.arange(1, N * esz + 1, dtype=torch.uint8, device=dev)
                KI.vstore(a, 3, vals, rebase=False, elem_bytes=esz)
                host = base.cpu().numpy()
                s = (off + 2) * esz
                assert np.array_equal(host[s:s + N * esz], np.arange(1, N * esz + 1, dtype=np.uint8))
                assert host[:s].sum() == 0 and host[s + N * esz:].sum() == 0


def test_custom_struct_golden(KI, golden, dev):
    import torch

    for c in golden["custom_struct"]:
        size = c["size"]
        arr = torch.from_numpy(_records(c["array"], c["layout"], size)).to(dev).reshape(-1)
        got = KI.vload(arr, 1, 4, rebase=False, elem_bytes=size).cpu().numpy()
        assert np.array_equal(got, _records(c["array"][:4], c["layout"], size)), c["name"]
        view = arr[c["load_view_offset"] * size:]
        got = KI.vload(view, 1, 4, rebase=False, elem_bytes=size).cpu().numpy()
        off = c["load_view_offset"]
        assert np.array_equal(got, _records(c["array"][off:off + 4], c["layout"], size)), c["name"]
        dst = torch.zeros(8 * size, dtype=torch.uint8, device=dev)
        vals = torch.from_numpy(_records(c["stored"], c["layout"], size)).to(dev).reshape(-1)
        KI.vstore(dst, 1, vals, rebase=False, elem_bytes=size)
        host = dst.cpu().numpy().reshape(8, size)
        assert np.array_equal(host[:4], _records(c["stored"], c["layout"], size)), c["name"]
        assert host[4:].sum() == 0


SCOPES = [None, "Workgroup", "Device", "System"]


def test_access_matrix(KI, dev):
    """Every valid (type, scope, ordering) store/fence/load round trip; invalid ones raise."""
    import torch

    dtypes = [torch.int8, torch.uint8, torch.int16, torch.uint16, torch.int32, torch.uint32, torch.int64,
              torch.uint64, torch.float32, torch.float64]
    orders = [None, KI.Weak, KI.Volatile, KI.Relaxed, KI.Acquire, KI.Release]
    fences = [(), (KI.Workgroup,), (KI.Device, KI.AcqRel), (KI.System, KI.SeqCst), (KI.AcqRel, KI.Device),
              (KI.Acquire,), (KI.Release,)]
    n_ok = 0
    for dt in dtypes:
        slot = torch.zeros(4, dtype=dt, device=dev)
        for sc in SCOPES:
            for o in orders:
                args = tuple(a for a in (getattr(KI, sc) if sc else None, o) if a is not None)
                invalid = sc is not None and o in (KI.Weak, KI.Volatile)
                for fa in fences[:3] if dt != torch.int64 else fences:
                    if invalid:
                        with pytest.raises(KI.KIArgumentError):
                            KI.access(slot, 7, *args, fence_args=fa)
                        continue
                    rb = KI.access(slot, 7, *args, fence_args=fa)
                    assert rb.cpu().item() == 7
                    n_ok += 1
    assert n_ok > 300
    slot = torch.zeros(1, dtype=torch.int64, device=dev)
    for bad in ((KI.AcqRel,), (KI.SeqCst,), (KI.Device, KI.Device), (KI.Device, KI.Relaxed, KI.Weak)):
        with pytest.raises(KI.KIArgumentError):
            KI.access(slot, 1, *bad)
    for bad in ((KI.Relaxed,), (KI.Weak,), (KI.Volatile,)):
        with pytest.raises(KI.KIArgumentError):
            KI.access(slot, 1, fence_args=bad)


def test_access_multidim_golden(KI, golden, dev):
    import torch

    c = golden["access"][0]
    data = torch.zeros(c["shape"][0] * c["shape"][1], dtype=torch.uint8, device=dev)
    li = c["linear_index_1based"] - 1
    KI.access(data[li:li + 1], c["value"])
    host = data.cpu().numpy().reshape(c["shape"][::-1]).T  # column-major like Julia
    i, j = c["index_1based"]
    assert host[i - 1, j - 1] == 0x20 and int(host.sum()) == 0x20


def test_message_passing_release_acquire(KI, dev):
    import torch

    data = torch.zeros(1, dtype=torch.int64, device=dev)
    for trial in range(20):
        flag = torch.zeros(1, dtype=torch.uint32, device=dev)
        seen = torch.zeros(64, dtype=torch.int64, device=dev)
        KI.message_pass(data, flag, seen, payload=1000 + trial, produce=True, timeout_s=2.0)
        KI.context(0).check()
        assert (seen[1:].cpu() == 1000 + trial).all()


def test_bounded_wait_times_out_without_hanging(KI, dev):
    """A flag that nothing sets: every consumer gives up after the limit and the host sees an error."""
    import torch

    data = torch.zeros(1, dtype=torch.int64, device=dev)
    flag = torch.zeros(1, dtype=torch.uint32, device=dev)
    seen = torch.zeros(8, dtype=torch.int64, device=dev)
    KI.message_pass(data, flag, seen, payload=5, produce=False, timeout_s=0.05)
    with pytest.raises(KI.KITimeoutError):
        KI.context(0).check()
    assert (seen[1:].cpu() == -1).all()
    KI.context(0).check()  # the latch was cleared and the context is still usable
    KI.message_pass(data, flag, seen, payload=6, produce=True, timeout_s=1.0)
    KI.context(0).check()
    assert (seen[1:].cpu() == 6).all()
