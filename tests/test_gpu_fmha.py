"""tcgen05 flash attention through the C ABI against float64 attention on the GPU."""

import ctypes as C
import math

import pytest

from golden_util import assert_contraction, attention_exact

pytestmark = pytest.mark.gpu

# max relative error of every f16 output, |o - exact| / max(|exact|, 2^-14), plus
# the f32 rounding noise of outputs that cancel (golden_util.assert_contraction)
TOL = 1e-2


def _fmha(q, k, v, o, bh, seq, scale, causal):
    import torch
    from ktir_cpu_b200 import runtime as R
    lib = R.load_library()
    status = torch.zeros(1, dtype=torch.int32, device=q.device)
    d = R.KtirFmhaDesc()
    d.q, d.k, d.v, d.o = q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr()
    d.bh, d.seq, d.d = bh, seq, 128
    d.scale = scale
    d.causal = 1 if causal else 0
    d.row_stride = 128
    d.status = status.data_ptr()
    R.check(lib.ktir_fmha_f16(C.byref(d), C.c_void_p(torch.cuda.current_stream().cuda_stream)),
            "ktir_fmha_f16")
    torch.cuda.synchronize()
    assert int(status.item()) == 0


def _check(name, o, q, k, v, bh, seq, scale, causal):
    want, mag = attention_exact(q, k, v, bh, seq, scale, causal)
    return assert_contraction(name, o.cpu().numpy(), want, mag, TOL)


@pytest.mark.parametrize("bh,seq,causal", [(1, 128, True), (2, 256, True), (3, 384, False),
                                           (4, 1024, True)])
def test_fmha_matches_fp32(bh, seq, causal):
    import torch
    g = torch.Generator(device="cpu").manual_seed(bh * 1000 + seq)
    q, k, v = (torch.randn(bh * seq, 128, generator=g).half().cuda() for _ in range(3))
    o = torch.full((bh * seq, 128), float("nan"), dtype=torch.float16, device="cuda")
    scale = float(1.0 / math.sqrt(128))
    _fmha(q, k, v, o, bh, seq, scale, causal)
    _check(f"bh{bh} s{seq} causal={causal}", o, q, k, v, bh, seq, scale, causal)


@pytest.mark.parametrize("causal", [True, False])
def test_fmha_running_max_moves(causal):
    """Keys whose logits grow along the sequence force the running max (and O, l)
    to be rescaled many times."""
    import torch
    bh, seq = 2, 1024
    g = torch.Generator(device="cpu").manual_seed(99)
    q, k, v = (torch.randn(bh * seq, 128, generator=g) for _ in range(3))
    ramp = 1.0 + 6.0 * torch.arange(seq).repeat(bh).float() / seq
    k = k * ramp[:, None]
    q, k, v = q.half().cuda(), k.half().cuda(), v.half().cuda()
    o = torch.full((bh * seq, 128), float("nan"), dtype=torch.float16, device="cuda")
    scale = float(1.0 / math.sqrt(128))
    _fmha(q, k, v, o, bh, seq, scale, causal)
    _check(f"ramp causal={causal}", o, q, k, v, bh, seq, scale, causal)


def test_fmha_no_corrupted_rows_across_shapes_and_seeds():
    """Repeated launches over several shapes and seeds: every output row is
    finite and within tolerance (a TMEM hazard between the softmax warps and
    the tensor pipe shows up as whole warps of NaN rows on some launches
    only)."""
    import torch
    for seed in range(3):
        for bh, seq, causal in [(3, 384, False), (1, 512, False), (2, 256, True), (2, 512, True),
                                (4, 1024, True), (2, 1024, False)]:
            g = torch.Generator(device="cpu").manual_seed(seed * 100 + bh * 10 + seq)
            q, k, v = (torch.randn(bh * seq, 128, generator=g).half().cuda() for _ in range(3))
            o = torch.full((bh * seq, 128), float("nan"), dtype=torch.float16, device="cuda")
            scale = float(1.0 / math.sqrt(128))
            _fmha(q, k, v, o, bh, seq, scale, causal)
            assert not torch.isnan(o).any().item(), (seed, bh, seq, causal)
            _check(f"seed {seed} bh{bh} s{seq} causal={causal}", o, q, k, v, bh, seq, scale,
                   causal)


@pytest.mark.parametrize("world", [2, 4, 8])
def test_fmha_partial_steps_of_the_ring(world):
    """The steps one GPU of the K/V ring runs (ktir_fmha_f16_part), emulated for
    every rank on one GPU: each rank's query tiles take the key tiles share by
    share in its ring order, the softmax state carried between steps; the
    query tiles of all ranks together must equal whole attention."""
    import torch
    from ktir_cpu_b200 import runtime as R
    from ktir_cpu_b200.ring import share_mask, staging_layout, step_shares
    lib = R.load_library()
    bh, seq, d = 3, 2048, 128
    n_tiles = seq // 128
    pairs = [(t, n_tiles - 1 - t) for t in range(n_tiles // 2)]
    per = len(pairs) // world
    tiles_of = [sorted(x for pr in pairs[r * per:(r + 1) * per] for x in pr) for r in range(world)]
    owner, local, kv_tiles = staging_layout(tiles_of, n_tiles)
    g = torch.Generator(device="cpu").manual_seed(world)
    q, k, v = (torch.randn(bh * seq, d, generator=g).half().cuda() for _ in range(3))
    scale = float(1.0 / math.sqrt(128))
    # the staging buffers: share s holds the K / V rows of rank s's tiles, every head
    share = bh * kv_tiles * 128
    k_sh = torch.zeros(world * share, d, dtype=torch.float16, device="cuda")
    v_sh = torch.zeros_like(k_sh)
    for s, tl in enumerate(tiles_of):
        for i, t in enumerate(tl):
            for h in range(bh):
                dst = slice(((s * bh + h) * kv_tiles + i) * 128, ((s * bh + h) * kv_tiles + i + 1) * 128)
                src = slice(h * seq + t * 128, h * seq + (t + 1) * 128)
                k_sh[dst] = k[src]
                v_sh[dst] = v[src]
    o = torch.full((bh * seq, d), float("nan"), dtype=torch.float16, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    for rank in range(world):
        mine = tiles_of[rank]
        o_acc = torch.full((bh * len(mine) * 128 * d,), float("nan"), device="cuda")
        ml = torch.full((bh * len(mine) * 128 * 2,), float("nan"), device="cuda")
        for t, s in enumerate(step_shares(rank, world)):
            dsc = R.KtirFmhaPartDesc()
            dsc.q, dsc.k, dsc.v, dsc.o = q.data_ptr(), k_sh.data_ptr(), v_sh.data_ptr(), o.data_ptr()
            dsc.bh, dsc.seq, dsc.d, dsc.kv_rows = bh, seq, d, world * share
            dsc.scale, dsc.causal = scale, 1
            dsc.n_qtiles, dsc.kv_tiles = len(mine), kv_tiles
            dsc.key_mask = share_mask(tiles_of[s])
            dsc.flags = (1 if t == 0 else 0) | (2 if t == world - 1 else 0)
            dsc.o_acc, dsc.ml, dsc.status = o_acc.data_ptr(), ml.data_ptr(), status.data_ptr()
            for i, qt in enumerate(mine):
                dsc.qtiles[i] = qt
            for kt in range(n_tiles):
                dsc.kv_owner[kt], dsc.kv_local[kt] = owner[kt], local[kt]
            R.check(lib.ktir_fmha_f16_part(C.byref(dsc), stream), "ktir_fmha_f16_part")
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    assert not torch.isnan(o).any().item()
    _check(f"ring emulated over {world} GPUs", o, q, k, v, bh, seq, scale, True)


def test_fmha_head_groups_of_the_ring():
    """The exchange of a program with head groups, emulated on one GPU as the
    plan issues it for the default ("gather") exchange: two groups of two
    heads, each served by two GPUs with zigzag query tiles.  Each emulated
    GPU packs its share from K and V offset to its group's first head
    (ktir_pack_kv) into its group's staging buffer, and one partial-attention
    call per GPU over every key tile of the staging layout writes its query
    tiles of O at the same head offset; all GPUs together must give whole
    attention."""
    import torch
    from ktir_cpu_b200 import runtime as R
    from ktir_cpu_b200.ring import share_mask, staging_layout
    lib = R.load_library()
    bh, seq, d, groups = 4, 1024, 128, 2
    hg, n_tiles, row_bytes = bh // groups, seq // 128, d * 2
    tiles_of = [[0, 1, 6, 7], [2, 3, 4, 5]]          # the two GPUs of every group
    owner, local, kv_tiles = staging_layout(tiles_of, n_tiles)
    g = torch.Generator(device="cpu").manual_seed(17)
    q, k, v = (torch.randn(bh * seq, d, generator=g).half().cuda() for _ in range(3))
    scale = float(1.0 / math.sqrt(128))
    o = torch.full((bh * seq, d), float("nan"), dtype=torch.float16, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    share_rows = hg * kv_tiles * 128
    for grp in range(groups):
        hoff = grp * hg * seq * row_bytes
        kv_all = torch.full((len(tiles_of) * 2 * share_rows * d,), float("nan"),
                            dtype=torch.float16, device="cuda")
        for pos, tl in enumerate(tiles_of):
            dst = kv_all.data_ptr() + pos * 2 * share_rows * row_bytes
            R.check(lib.ktir_pack_kv(C.c_void_p(dst), C.c_void_p(k.data_ptr() + hoff),
                                     C.c_void_p(v.data_ptr() + hoff), hg, seq, d,
                                     share_mask(tl), stream), "ktir_pack_kv")
        for pos, mine in enumerate(tiles_of):
            dsc = R.KtirFmhaPartDesc()
            dsc.q, dsc.o = q.data_ptr() + hoff, o.data_ptr() + hoff
            dsc.k = kv_all.data_ptr()
            dsc.v = kv_all.data_ptr() + share_rows * row_bytes
            dsc.bh, dsc.seq, dsc.d = hg, seq, d
            dsc.kv_tiles, dsc.kv_rows = kv_tiles, (2 * len(tiles_of) - 1) * share_rows
            dsc.scale, dsc.causal = scale, 1
            dsc.n_qtiles = len(mine)
            dsc.key_mask = share_mask(range(n_tiles))
            dsc.flags = 3
            dsc.status = status.data_ptr()
            for i, qt in enumerate(mine):
                dsc.qtiles[i] = qt
            for kt in range(n_tiles):
                dsc.kv_owner[kt], dsc.kv_local[kt] = 2 * owner[kt], local[kt]
            R.check(lib.ktir_fmha_f16_part(C.byref(dsc), stream), "ktir_fmha_f16_part")
        torch.cuda.synchronize()
    assert int(status.item()) == 0
    assert not torch.isnan(o).any().item()
    _check("head groups emulated over 2 x 2 GPUs", o, q, k, v, bh, seq, scale, True)
