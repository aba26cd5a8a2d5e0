"""tcgen05 GEMM through the C ABI against a PyTorch float32 matmul."""

import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

# max relative error on f16 outputs of an f32-accumulated product; values below
# magnitude 1 judged absolutely (rtol = atol = 1e-2)
TOL = 1e-2


def _gemm(a, b, c):
    import torch
    from ktir_cpu_b200 import runtime as R
    lib = R.load_library()
    status = torch.zeros(1, dtype=torch.int32, device=a.device)
    d = R.KtirGemmDesc()
    d.a, d.b, d.c = a.data_ptr(), b.data_ptr(), c.data_ptr()
    d.lda, d.ldb, d.ldc = a.shape[1], b.shape[1], c.shape[1]
    d.m, d.n, d.k = a.shape[0], b.shape[1], a.shape[1]
    d.add_zero = 1
    d.status = status.data_ptr()
    stream = torch.cuda.current_stream().cuda_stream
    R.check(lib.ktir_gemm_f16(C.byref(d), C.c_void_p(stream)), "ktir_gemm_f16")
    torch.cuda.synchronize()
    assert int(status.item()) == 0


@pytest.mark.parametrize("m,n,k", [(128, 256, 64), (256, 512, 128), (512, 256, 1024),
                                   (384, 768, 320)])
def test_gemm_matches_fp32(m, n, k):
    import torch
    g = torch.Generator(device="cpu").manual_seed(m * 7 + n + k)
    a = (torch.rand(m, k, generator=g) * 2 - 1).half().cuda()
    b = (torch.rand(k, n, generator=g) * 2 - 1).half().cuda()
    c = torch.full((m, n), float("nan"), dtype=torch.float16, device="cuda")
    _gemm(a, b, c)
    ref = a.float() @ b.float()
    err = ((c.float() - ref).abs() / ref.abs().clamp_min(1.0)).max().item()
    assert err <= TOL, err


def test_gemm_rejects_unaligned_shapes():
    import torch
    from ktir_cpu_b200 import runtime as R
    lib = R.load_library()
    d = R.KtirGemmDesc()
    a = torch.zeros(100, 64, dtype=torch.float16, device="cuda")
    d.a = d.b = d.c = a.data_ptr()
    d.status = a.data_ptr()
    d.m, d.n, d.k, d.lda, d.ldb, d.ldc = 100, 256, 64, 64, 256, 256
    assert lib.ktir_gemm_f16(C.byref(d), None) != 0


def test_gemm_split_tail_with_workspace():
    """200 tiles on 148 SMs leave a last wave of 52 tiles: with a workspace
    those are split in K across two SMs each.  Two calls in a row (the
    workspace must come back clean) against float32 and against the unsplit
    schedule."""
    import torch
    from ktir_cpu_b200 import runtime as R
    lib = R.load_library()
    m, n, k = 3200, 2048, 512
    nbytes = int(lib.ktir_gemm_workspace_bytes(m, n, k))
    n_sm = torch.cuda.get_device_properties(0).multi_processor_count
    if (m // 128) * (n // 256) % n_sm == 0 or nbytes <= 0:
        pytest.skip("this device would not split the tail")
    g = torch.Generator(device="cpu").manual_seed(11)
    a = (torch.rand(m, k, generator=g) * 2 - 1).half().cuda()
    b = (torch.rand(k, n, generator=g) * 2 - 1).half().cuda()
    ws = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    ref = a.float() @ b.float()
    outs = []
    for use_ws in (True, True, False):
        c = torch.full((m, n), float("nan"), dtype=torch.float16, device="cuda")
        d = R.KtirGemmDesc()
        d.a, d.b, d.c = a.data_ptr(), b.data_ptr(), c.data_ptr()
        d.lda, d.ldb, d.ldc, d.m, d.n, d.k = k, n, n, m, n, k
        d.add_zero = 1
        d.status = status.data_ptr()
        if use_ws:
            d.workspace, d.workspace_bytes = ws.data_ptr(), nbytes
        R.check(lib.ktir_gemm_f16(C.byref(d), C.c_void_p(torch.cuda.current_stream().cuda_stream)),
                "ktir_gemm_f16")
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        err = ((c.float() - ref).abs() / ref.abs().clamp_min(1.0)).max().item()
        assert err <= TOL, err
        outs.append(c)
    # the per-row counters are back to zero after each call
    n_split = (m // 128) * (n // 256) % n_sm
    assert int(ws[:n_split * 128 * 4].view(torch.int32).abs().sum().item()) == 0
    assert torch.equal(outs[0], outs[1])
