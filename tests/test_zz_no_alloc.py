"""The allocation-free gather -> +1 -> scatter entry point agrees with the regular one.

ktir_gather_rmw_static serves callers that cannot allocate device memory:
its scratch is a fixed array inside the library.  This test drives both entry
points through the C ABI on identical copies of a table whose index list has
many duplicates, twice in a row (the second call must start from cleared
counts), and requires bit-identical tables after each call.  It lives in its
own file, collected last, and builds everything it needs itself so it also
passes when run alone in a fresh process.
"""

import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _descriptor(n_units, unit_len, row_len, n_rows):
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
    d.f = program(b, (1,), 1, 0, lambda k: mkview(0, np.float16, 0, (0,)))
    return d


def test_static_scratch_entry_point_matches_allocating_one():
    import torch
    from ktir_cpu_b200 import runtime as R
    lib = R.load_library()
    lib.ktir_gather_rmw_static.argtypes = [C.POINTER(R.KtirGatherRmwDesc),
                                           C.POINTER(R.KtirBuffers), C.c_int64, C.c_void_p,
                                           C.c_void_p]
    lib.ktir_gather_rmw_static.restype = C.c_int
    n_rows, row_len, n_units, unit_len = 4096, 128, 16, 512
    rng = np.random.default_rng(99)
    table = rng.standard_normal((n_rows, row_len)).astype(np.float16)
    idx = rng.integers(0, n_rows // 4, n_units * unit_len).astype(np.int32)  # many duplicates
    dev = torch.device("cuda")
    t_ref = torch.from_numpy(table.copy()).to(dev)
    t_new = torch.from_numpy(table.copy()).to(dev)
    idx_d = torch.from_numpy(idx).to(dev)
    counts = torch.zeros(n_rows, dtype=torch.int32, device=dev)
    status = torch.zeros(2, dtype=torch.int32, device=dev)
    d = _descriptor(n_units, unit_len, row_len, n_rows)

    def bufs(t):
        b = R.KtirBuffers()
        b.base[0], b.numel[0] = t.data_ptr(), t.numel()
        b.base[1], b.numel[1] = idx_d.data_ptr(), idx_d.numel()
        return b
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    for call in range(2):
        R.check(lib.ktir_gather_rmw(C.byref(d), C.byref(bufs(t_ref)), C.c_void_p(counts.data_ptr()),
                                    n_rows, C.c_void_p(status.data_ptr()), stream), "ktir_gather_rmw")
        R.check(lib.ktir_gather_rmw_static(C.byref(d), C.byref(bufs(t_new)), n_rows,
                                           C.c_void_p(status.data_ptr() + 4), stream),
                "ktir_gather_rmw_static")
        torch.cuda.synchronize()
        assert status.tolist() == [0, 0]
        # integer/byte work: the two entry points must agree bit for bit
        assert torch.equal(t_ref, t_new), f"call {call}: tables differ"
        assert not torch.equal(t_ref.cpu(), torch.from_numpy(table)), "nothing was updated"


def test_static_scratch_rejects_oversized_tables():
    import torch
    from ktir_cpu_b200 import runtime as R
    lib = R.load_library()
    lib.ktir_gather_rmw_static.argtypes = [C.POINTER(R.KtirGatherRmwDesc),
                                           C.POINTER(R.KtirBuffers), C.c_int64, C.c_void_p,
                                           C.c_void_p]
    d = _descriptor(1, 8, 128, 8)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc = lib.ktir_gather_rmw_static(C.byref(d), C.byref(R.KtirBuffers()), (1 << 20) + 1,
                                    C.c_void_p(status.data_ptr()), None)
    assert rc == -3
