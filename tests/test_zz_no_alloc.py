"""The allocation-free gather -> +1 -> scatter entry point agrees with the regular one.

ktir_gather_rmw_static serves callers that cannot allocate device memory:
its scratch is a fixed array inside the library.  These tests drive both
entry points through the C ABI on identical copies of a table whose index
list has many duplicates, and require bit-identical tables (integer and byte
work: no tolerance).  The first test also checks the result against the
NumPy oracle of the reference interpreter on the same KTIR program, and runs
two calls in a row (the second must start from cleared counts).  This file
is collected last and builds everything it needs itself, so it also passes
when run alone in a fresh process.
"""

import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

MAX_ROWS = 1 << 20   # KTIR_STATIC_RMW_MAX_ROWS in include/ktir_b200.h


def _lib():
    from ktir_cpu_b200 import runtime as R
    lib = R.load_library()
    lib.ktir_gather_rmw_static.argtypes = [C.POINTER(R.KtirGatherRmwDesc),
                                           C.POINTER(R.KtirBuffers), C.c_int64, C.c_void_p,
                                           C.c_void_p]
    lib.ktir_gather_rmw_static.restype = C.c_int
    return lib


def _descriptor(n_units, unit_len, row_len, phases=0, row_lo=0, row_hi=0):
    from ktir_cpu_b200 import runtime as R
    from ktir_cpu_b200.lower import EwBuilder, mkview, program
    b = EwBuilder()
    b.view("g")
    b.view("s")
    x = b.alloc()
    b.emit("LD", x, aux=0)
    one = b.imm(1.0, np.float16)
    y = b.alloc()
    b.emit("FADD", y, x, one, dt=R.F16)
    b.emit("ST", 0, y, dt=R.F16, aux=1)
    d = R.KtirGatherRmwDesc()
    d.table_slot, d.idx_slot, d.idx_dtype = 0, 1, R.I32
    d.n_units, d.unit_len, d.row_len = n_units, unit_len, row_len
    d.table_off, d.row_stride = 0, row_len
    d.idx_off, d.idx_unit_stride = 0, unit_len
    d.row_lo, d.row_hi, d.phases = row_lo, row_hi, phases
    d.f = program(b, (1,), 1, 0, lambda k: mkview(0, np.float16, 0, (0,)))
    return d


class _Pair:
    """Two device copies of one table, one per entry point, and a shared index list."""

    def __init__(self, table, idx):
        import torch
        from ktir_cpu_b200 import runtime as R
        self.R = R
        self.lib = _lib()
        dev = torch.device("cuda")
        self.table = table
        self.t_ref = torch.from_numpy(table.copy()).to(dev)
        self.t_new = torch.from_numpy(table.copy()).to(dev)
        self.idx_d = torch.from_numpy(idx).to(dev)
        self.n_rows = table.shape[0]
        self.counts = torch.zeros(self.n_rows, dtype=torch.int32, device=dev)
        self.status = torch.zeros(2, dtype=torch.int32, device=dev)
        self.stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)

    def _bufs(self, t):
        b = self.R.KtirBuffers()
        b.base[0], b.numel[0] = t.data_ptr(), t.numel()
        b.base[1], b.numel[1] = self.idx_d.data_ptr(), self.idx_d.numel()
        return b

    def call(self, d, n_rows=None):
        n = self.n_rows if n_rows is None else n_rows
        self.R.check(self.lib.ktir_gather_rmw(C.byref(d), C.byref(self._bufs(self.t_ref)),
                                              C.c_void_p(self.counts.data_ptr()), n,
                                              C.c_void_p(self.status.data_ptr()), self.stream),
                     "ktir_gather_rmw")
        self.R.check(self.lib.ktir_gather_rmw_static(C.byref(d), C.byref(self._bufs(self.t_new)), n,
                                                     C.c_void_p(self.status.data_ptr() + 4),
                                                     self.stream),
                     "ktir_gather_rmw_static")

    def check(self, what):
        import torch
        torch.cuda.synchronize()
        assert self.status.tolist() == [0, 0], what
        assert torch.equal(self.t_ref, self.t_new), f"{what}: tables differ"


def test_static_scratch_entry_point_matches_allocating_one_and_oracle():
    from ktir_cpu_b200 import workloads as W
    from oracle.interp import OracleInterpreter
    n_rows, row_len, n_units, unit_len = 4096, 128, 16, 512
    rng = np.random.default_rng(99)
    table = rng.standard_normal((n_rows, row_len)).astype(np.float16)
    idx = rng.integers(0, n_rows // 4, n_units * unit_len).astype(np.int32)  # many duplicates
    pair = _Pair(table, idx)
    d = _descriptor(n_units, unit_len, row_len)
    # the same computation as a KTIR program on the oracle: one unit per core
    p = dict(rows=n_rows, cols=row_len, n_idx=n_units * unit_len, grid=n_units, chunk=unit_len)
    ora = OracleInterpreter()
    ora.load(W.source("gather_add", **p))
    want = table.copy()
    for call in range(2):
        pair.call(d)
        pair.check(f"call {call}")
        want = ora.execute_function("gather_add", table_ptr=want, idx_ptr=idx.copy())["table_ptr"]
        got = pair.t_new.cpu().numpy()
        assert np.array_equal(got, want), f"call {call}: differs from the oracle"
    assert not np.array_equal(want, table), "nothing was updated"


def test_static_scratch_count_then_apply_split():
    """A count-only call then an apply-only call over a row range (the flow of
    a split execution) keeps the counts between the two calls."""
    n_rows, row_len, n_units, unit_len = 2048, 64, 8, 256
    rng = np.random.default_rng(7)
    table = rng.standard_normal((n_rows, row_len)).astype(np.float16)
    idx = rng.integers(0, n_rows, n_units * unit_len).astype(np.int32)
    idx[::3] = idx[0]   # one row named by every unit
    pair = _Pair(table, idx)
    for lo, hi in ((0, 700), (700, n_rows)):
        pair.call(_descriptor(n_units, unit_len, row_len, phases=1))
        pair.call(_descriptor(n_units, unit_len, row_len, phases=2, row_lo=lo, row_hi=hi))
        pair.check(f"rows [{lo}, {hi})")
    # both halves applied: the whole table equals one unsplit call's result
    whole = _Pair(table, idx)
    whole.call(_descriptor(n_units, unit_len, row_len))
    whole.check("unsplit")
    assert np.array_equal(pair.t_new.cpu().numpy(), whole.t_new.cpu().numpy())


def test_static_scratch_limits():
    """n_rows == the maximum is accepted (the whole array in use, indices near
    the top row); n_rows == 0 leaves the table unchanged; one more row than the
    maximum is rejected with a message naming the limit."""
    import torch
    row_len, n_units, unit_len = 8, 4, 256
    rng = np.random.default_rng(3)
    table = rng.standard_normal((MAX_ROWS, row_len)).astype(np.float16)
    idx = (MAX_ROWS - 1 - rng.integers(0, 64, n_units * unit_len)).astype(np.int32)
    pair = _Pair(table, idx)
    d = _descriptor(n_units, unit_len, row_len)
    pair.call(d)
    pair.check("n_rows at the maximum")
    assert not torch.equal(pair.t_new.cpu(), torch.from_numpy(table))
    before = pair.t_new.clone()
    pair.call(d, n_rows=0)
    pair.check("n_rows = 0")
    assert torch.equal(pair.t_new, before)
    lib = pair.lib
    rc = lib.ktir_gather_rmw_static(C.byref(d), C.byref(pair.R.KtirBuffers()), MAX_ROWS + 1,
                                    C.c_void_p(pair.status.data_ptr()), None)
    assert rc == -3
    assert b"KTIR_STATIC_RMW_MAX_ROWS" in lib.ktir_last_error()
