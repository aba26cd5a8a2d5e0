"""tcgen05 GEMM through the C ABI against a PyTorch float32 matmul."""

import ctypes as C

import pytest

pytestmark = pytest.mark.gpu

from golden_util import assert_contraction

# max relative error of every f16 output against the float64 product, plus the
# f32 rounding noise of outputs that cancel (golden_util.assert_contraction)
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


# the last two take more than one wave of the persistent grid on a 148-SM B200
# (512 tiles, 68 in the last wave; 160 tiles, 12)
@pytest.mark.parametrize("m,n,k", [(128, 256, 64), (256, 512, 128), (512, 256, 1024),
                                   (384, 768, 320), (4096, 4096, 256), (1280, 4096, 192)])
def test_gemm_matches_fp32(m, n, k):
    import torch
    g = torch.Generator(device="cpu").manual_seed(m * 7 + n + k)
    a = (torch.rand(m, k, generator=g) * 2 - 1).half().cuda()
    b = (torch.rand(k, n, generator=g) * 2 - 1).half().cuda()
    c = torch.full((m, n), float("nan"), dtype=torch.float16, device="cuda")
    _gemm(a, b, c)
    exact = (a.double() @ b.double()).half().cpu().numpy()
    mag = (a.float().abs() @ b.float().abs()).cpu().numpy()
    assert_contraction(f"gemm {m}x{n}x{k}", c.cpu().numpy(), exact, mag, TOL)


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

