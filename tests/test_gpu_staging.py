"""Host staging (ktir_host_upload / ktir_host_download) round trips: sizes
that split into many chunks, ragged tails, empty buffers, host-to-host copies
alongside, and repeated calls on the same pinned buffers."""

import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

SIZES = [0, 1, 4095, (1 << 20) + 3, 17 * (1 << 20) + 129]


def test_upload_download_round_trip():
    import torch
    from ktir_cpu_b200 import runtime as R
    lib = R.load_library()
    rng = np.random.default_rng(1)
    src = [rng.integers(0, 256, n, dtype=np.uint8) for n in SIZES]
    dev = [torch.empty(max(n, 1), dtype=torch.uint8, device="cuda") for n in SIZES]
    pin = [torch.empty(max(n, 1), dtype=torch.uint8, pin_memory=True) for n in SIZES]
    stream = torch.cuda.current_stream()
    sp = C.c_void_p(stream.cuda_stream)
    for rep in range(3):
        xs = (R.KtirHostXfer * len(SIZES))()
        for k, n in enumerate(SIZES):
            xs[k].host, xs[k].pinned = src[k].ctypes.data, pin[k].data_ptr()
            xs[k].device, xs[k].bytes = dev[k].data_ptr(), n
        R.check(lib.ktir_host_upload(xs, len(SIZES), torch.cuda.current_device(), sp), "upload")
        for t in dev:           # the device copy is changed before it comes back
            t.add_(1)
        out = [np.zeros(n, np.uint8) for n in SIZES]
        other_src = rng.integers(0, 256, 5 * (1 << 20) + 7, dtype=np.uint8)
        other_dst = np.zeros_like(other_src)
        ys = (R.KtirHostXfer * len(SIZES))()
        for k, n in enumerate(SIZES):
            ys[k].host, ys[k].pinned = out[k].ctypes.data, pin[k].data_ptr()
            ys[k].device, ys[k].bytes = dev[k].data_ptr(), n
        cs = (R.KtirHostCopy * 1)()
        cs[0].dst, cs[0].src, cs[0].bytes = other_dst.ctypes.data, other_src.ctypes.data, other_src.size
        R.check(lib.ktir_host_download(ys, len(SIZES), cs, 1, torch.cuda.current_device(), sp),
                "download")
        for k in range(len(SIZES)):
            assert np.array_equal(out[k], (src[k] + 1).astype(np.uint8)), (rep, SIZES[k])
        assert np.array_equal(other_dst, other_src)
        src = [rng.integers(0, 256, n, dtype=np.uint8) for n in SIZES]


def test_execute_function_returns_fresh_arrays():
    """The caller's arrays are not written and each call returns new arrays."""
    from ktir_cpu_b200 import KTIRInterpreter
    import ktir_cpu_b200.workloads as W
    src = W.source("softmax")
    kw = W.inputs("softmax", seed=3)
    keep = {k: v.copy() for k, v in kw.items()}
    interp = KTIRInterpreter()
    interp.load(src)
    a = interp.execute_function(W.FUNC["softmax"], **kw)
    b = interp.execute_function(W.FUNC["softmax"], **kw)
    for k in kw:
        assert np.array_equal(kw[k], keep[k])
        assert a[k] is not kw[k] and b[k] is not a[k]
        assert np.array_equal(a[k], b[k])
    assert np.array_equal(a["in_ptr"].view(np.uint16), kw["in_ptr"].view(np.uint16))


def test_results_held_or_viewed_are_never_reused():
    """Results come back in pooled page-locked buffers: a buffer is reused only
    once nothing refers to it, so a kept result, or a view that outlives its
    result, keeps its contents across later calls."""
    import gc
    from ktir_cpu_b200 import KTIRInterpreter
    import ktir_cpu_b200.workloads as W
    src = W.source("vector_add")
    interp = KTIRInterpreter()
    interp.load(src)
    fn = W.FUNC["vector_add"]
    kws = [W.inputs("vector_add", seed=s) for s in range(4)]
    first = interp.execute_function(fn, **kws[0])
    keep = {k: v.copy() for k, v in first.items()}
    name = [k for k in first if not np.array_equal(first[k], kws[0][k])][0]   # the output
    view = first[name][3:]
    view_copy = view.copy()
    other = interp.execute_function(fn, **kws[1])
    del other
    gc.collect()
    for s in range(2, 4):
        interp.execute_function(fn, **kws[s])
    for k in first:
        assert np.array_equal(first[k].view(np.uint16), keep[k].view(np.uint16))
    del first
    gc.collect()
    for s in range(4):
        interp.execute_function(fn, **kws[s])
    assert np.array_equal(view.view(np.uint16), view_copy.view(np.uint16))
