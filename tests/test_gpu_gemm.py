"""tcgen05 GEMMs through the C ABI against float64 products on the GPU."""

import ctypes as C

import pytest

from golden_util import assert_contraction

pytestmark = pytest.mark.gpu

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
    d.lda, d.ldb, d.ldc = a.stride(0), b.stride(0), c.stride(0)
    d.m, d.n, d.k = a.shape[0], b.shape[1], a.shape[1]
    d.add_zero = 1
    d.status = status.data_ptr()
    stream = torch.cuda.current_stream().cuda_stream
    R.check(lib.ktir_gemm_f16(C.byref(d), C.c_void_p(stream)), "ktir_gemm_f16")
    torch.cuda.synchronize()
    assert int(status.item()) == 0


# (4096, 4096, 256) and (1280, 4096, 192) take more than one wave of the
# persistent grid of 128 x 256 tiles on a 148-SM B200 (512 tiles, 68 in the
# last wave; 160 tiles, 12); the smaller ones, too few 256-wide tiles to fill
# half the SMs, run 128 x 128 tiles, as do N = 384 and 1408 (not multiples of
# 256); (2048, 1024, 4096) is one GPU's slice of the 4096^3 GEMM split over
# eight (128 tiles of 128 x 128, one wave), (4096, 1408, 128) two waves of them
@pytest.mark.parametrize("m,n,k", [(128, 256, 64), (256, 512, 128), (512, 256, 1024),
                                   (384, 768, 320), (4096, 4096, 256), (1280, 4096, 192),
                                   (256, 384, 512), (2048, 1024, 4096), (4096, 1408, 128)])
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



def _blocked(a, b, c, block_k, acc_f16):
    import torch
    from ktir_cpu_b200 import runtime as R
    lib = R.load_library()
    status = torch.zeros(1, dtype=torch.int32, device=a.device)
    d = R.KtirGemmBlockedDesc()
    d.a, d.b, d.c = a.data_ptr(), b.data_ptr(), c.data_ptr()
    d.lda, d.ldb, d.ldc = a.stride(0), b.stride(0), c.stride(0)
    d.m, d.n, d.k = a.shape[0], b.shape[1], a.shape[1]
    d.block_k, d.acc_f16 = block_k, acc_f16
    d.status = status.data_ptr()
    R.check(lib.ktir_gemm_f16_blocked(C.byref(d), C.c_void_p(torch.cuda.current_stream().cuda_stream)),
            "ktir_gemm_f16_blocked")
    torch.cuda.synchronize()
    assert int(status.item()) == 0


# shapes the aligned kernel does not take (M, N, K not multiples of 128, 256,
# 64; M below one tile; the row strides of A and B multiples of 8 elements, as
# TMA row strides are multiples of 16 bytes: N = 130 has B rows 136 apart),
# widened (block_k 0) and f16 block products rounded per block into an f16 or
# f32 running sum (the reference's matmul_fwd example)
@pytest.mark.parametrize("m,n,k,block_k,acc_f16", [
    (64, 8192, 2048, 128, 1), (100, 200, 72, 0, 0), (257, 130, 296, 0, 0),
    (32, 512, 256, 32, 1), (200, 136, 512, 128, 0), (1, 8, 16, 16, 1)])
def test_blocked_gemm_matches_reference_rounding(m, n, k, block_k, acc_f16):
    import torch
    g = torch.Generator(device="cpu").manual_seed(m + 3 * n + 7 * k)
    a = (torch.rand(m, k, generator=g) * 2 - 1).half().cuda()
    b = (torch.rand(k, n, generator=g) * 2 - 1).half().cuda()
    if n % 8:
        b = torch.zeros(k, (n + 7) // 8 * 8, dtype=torch.float16, device="cuda")[:, :n].copy_(b)
    c = torch.full((m, n), float("nan"), dtype=torch.float16, device="cuda")
    _blocked(a, b, c, block_k, acc_f16)
    if block_k == 0:
        want = (a.double() @ b.double()).half()
        mag = a.float().abs() @ b.float().abs()
        assert_contraction(f"blocked {m}x{n}x{k} widened", c.cpu().numpy(), want.cpu().numpy(),
                           mag.cpu().numpy(), TOL)
        return
    # each block product rounded to f16, then added to the running sum
    acc = torch.zeros(m, n, dtype=torch.float64, device="cuda")
    mag = torch.zeros(m, n, dtype=torch.float64, device="cuda")
    for k0 in range(0, k, block_k):
        prod = (a[:, k0:k0 + block_k].double() @ b[k0:k0 + block_k].double()).half().double()
        acc = acc + prod
        if acc_f16:
            acc = acc.half().double()
        else:
            acc = acc.float().double()
        mag += prod.abs()
    assert_contraction(f"blocked {m}x{n}x{k} block {block_k} acc {'f16' if acc_f16 else 'f32'}",
                       c.cpu().numpy(), acc.half().cpu().numpy(), mag.cpu().numpy(), TOL,
                       u=2.0 ** -11)
