"""Failure detection on the device, without faulting a GPU.

A device wait that runs out must come back as a status bit the host turns
into an exception; a negative indirect index must surface as IndexError.
"""

import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_bounded_wait_reports_timeout_and_returns():
    import torch
    from ktir_cpu_b200 import runtime as R
    lib = R.load_library()
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    R.check(lib.ktir_wait_selftest(C.c_void_p(status.data_ptr()), 1000, None), "selftest")
    torch.cuda.synchronize()
    assert int(status.item()) & R.STATUS_TIMEOUT
    # the context is still usable afterwards
    x = torch.ones(4, device="cuda") * 2
    assert float(x.sum()) == 8.0


def test_timeout_status_raises_on_host():
    import torch
    from ktir_cpu_b200 import KTIRInterpreter, runtime as R
    from ktir_cpu_b200 import workloads as W
    p = dict(n=1024, grid=2)
    interp = KTIRInterpreter()
    interp.load(W.source("vector_add", **p))
    interp.execute_function("add_kernel", **W.inputs("vector_add", **p))
    exe = interp.last_executable
    exe.plan.status_check = True
    R.load_library().ktir_wait_selftest(C.c_void_p(exe.status.data_ptr()), 10, None)
    torch.cuda.synchronize()
    with pytest.raises(RuntimeError, match="timed out"):
        exe.check_status()
