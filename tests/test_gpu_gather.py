"""Gather-RMW through the C ABI against a host restatement of the reference's
unit-by-unit semantics (duplicates within a unit apply once, across units
once per unit), on tables with many duplicate indices, and the two-pass form
a sharded call uses (count everything, apply an owned row range)."""

import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _descriptor(n_units, unit_len, row_len, op="FADD", imm=1.0):
    from ktir_cpu_b200 import runtime as R
    from ktir_cpu_b200.lower import EwBuilder, mkview, program
    b = EwBuilder()
    b.view("g")
    b.view("s")
    x = b.alloc()
    b.emit("LD", x, aux=0)
    c = b.imm(imm, np.float16)
    y = b.alloc()
    b.emit(op, y, x, c, dt=R.F16)
    b.emit("ST", 0, y, dt=R.F16, aux=1)
    d = R.KtirGatherRmwDesc()
    d.table_slot, d.idx_slot, d.idx_dtype = 0, 1, R.I32
    d.n_units, d.unit_len, d.row_len = n_units, unit_len, row_len
    d.table_off, d.row_stride = 0, row_len
    d.idx_off, d.idx_unit_stride = 0, unit_len
    d.f = program(b, (1,), 1, 0, lambda k: mkview(0, np.float16, 0, (0,)))
    return d


def _host(table, idx, n_units, unit_len, op, imm, calls):
    want = table.copy()
    c = np.float32(imm)
    for _ in range(calls):
        for u in range(n_units):
            for r in np.unique(idx[u * unit_len:(u + 1) * unit_len]):
                x = want[r].astype(np.float32)
                y = x * c if op == "FMUL" else (x - c if op == "FSUB" else x + c)
                want[r] = y.astype(np.float16)
    return want


def _call(lib, R, d, t, i, counts, status, stream):
    bufs = R.KtirBuffers()
    bufs.base[0], bufs.numel[0] = t.data_ptr(), t.numel()
    bufs.base[1], bufs.numel[1] = i.data_ptr(), i.numel()
    R.check(lib.ktir_gather_rmw(C.byref(d), C.byref(bufs), C.c_void_p(counts.data_ptr()),
                                counts.numel(), C.c_void_p(status.data_ptr()), stream),
            "ktir_gather_rmw")


@pytest.mark.parametrize("row_len,op", [(128, "FADD"), (64, "FMUL"), (200, "FSUB")])
def test_gather_rmw_matches_host(row_len, op):
    import torch
    from ktir_cpu_b200 import runtime as R
    lib = R.load_library()
    n_rows, n_units, unit_len = 3000, 24, 700
    imm = 1.5 if op == "FMUL" else 1.0
    rng = np.random.default_rng(row_len)
    table = rng.standard_normal((n_rows, row_len)).astype(np.float16)
    idx = rng.integers(0, n_rows // 3, n_units * unit_len).astype(np.int32)
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    t = torch.from_numpy(table.copy()).cuda()
    i = torch.from_numpy(idx).cuda()
    counts = torch.zeros(n_rows, dtype=torch.int32, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    d = _descriptor(n_units, unit_len, row_len, op, imm)
    for _ in range(2):   # the scratch must come back clean for the second call
        _call(lib, R, d, t, i, counts, status, stream)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    assert int(counts.abs().sum().item()) == 0
    want = _host(table, idx, n_units, unit_len, op, imm, 2)
    assert np.array_equal(t.cpu().numpy().view(np.uint16), want.view(np.uint16))


def test_two_pass_owned_row_ranges_merge():
    """Two emulated shards: both count every unit, each applies its own range
    of rows to its own copy; the ranges together are the full result and both
    count arrays end zero."""
    import torch
    from ktir_cpu_b200 import runtime as R
    lib = R.load_library()
    n_rows, n_units, unit_len, row_len = 2048, 16, 512, 128
    rng = np.random.default_rng(5)
    table = rng.standard_normal((n_rows, row_len)).astype(np.float16)
    idx = rng.integers(0, n_rows, n_units * unit_len).astype(np.int32)
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    i = torch.from_numpy(idx).cuda()
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    merged = np.empty_like(table)
    for lo, hi in [(0, 1000), (1000, n_rows)]:
        t = torch.from_numpy(table.copy()).cuda()
        counts = torch.zeros(n_rows, dtype=torch.int32, device="cuda")
        d = _descriptor(n_units, unit_len, row_len)
        d.phases = 1
        _call(lib, R, d, t, i, counts, status, stream)
        d.phases, d.row_lo, d.row_hi = 2, lo, hi
        _call(lib, R, d, t, i, counts, status, stream)
        torch.cuda.synchronize()
        assert int(counts.abs().sum().item()) == 0
        out = t.cpu().numpy()
        assert np.array_equal(out[:lo].view(np.uint16), table[:lo].view(np.uint16))
        assert np.array_equal(out[hi:].view(np.uint16), table[hi:].view(np.uint16))
        merged[lo:hi] = out[lo:hi]
    want = _host(table, idx, n_units, unit_len, "FADD", 1.0, 1)
    assert np.array_equal(merged.view(np.uint16), want.view(np.uint16))
