"""Tensor-core programs: GEMM and attention matchers over the traced graph.

GEMM: every store must be ``truncf(acc_K)`` with ``acc_k = acc_{k-1} +
extf(A_k) @ extf(B_k)`` (the K loop of ``linalg.matmul`` with an f32
iter_arg accumulator, ktir_cpu/dialects/linalg_ops.py:273-297), starting from
a zero constant, where the A_k / B_k loads sweep K contiguously, and the
stores must tile the output matrix exactly.  The whole call then becomes one
tcgen05 GEMM launch over C = A @ B (f32 accumulation, f16 store).  Numerics:
the reference accumulates per 128-wide K tile in OpenBLAS order; the tensor
cores accumulate the full K in their own order — equal within the stated
tolerance, not bit-exact.

Attention: see :mod:`ktir_cpu_b200.rewrite`.
"""

from __future__ import annotations

import ctypes as C
from typing import List

import numpy as np

from . import runtime as R
from .trace import Node, RectTarget, Store

GEMM_TILE_M, GEMM_TILE_N, GEMM_TILE_K = 128, 256, 64


def _is_cast(n, src, dst) -> bool:
    return isinstance(n, Node) and n.kind == "ew" and n.attrs.get("op") == "cast" and \
        n.dtype == dst and n.ins[0].dtype == src


def _rect2d(n) -> bool:
    return isinstance(n, Node) and n.kind == "load" and n.attrs["mode"] == "rect" and \
        len(n.shape) == 2 and n.attrs["strides"][1] == 1


def gemm_chain(store: Store):
    """(i0, j0, bm, bn, [(A load, B load), ...]) for one output tile, or None."""
    t = store.target
    if not isinstance(t, RectTarget) or len(t.shape) != 2 or t.strides[1] != 1 or \
            t.dtype != np.float16:
        return None
    root = store.value
    if not _is_cast(root, np.float32, np.float16):
        return None
    acc = root.ins[0]
    pairs = []
    while isinstance(acc, Node) and acc.kind == "ew" and acc.attrs.get("matmul_accumulate"):
        prev, mm = acc.ins
        if not (isinstance(mm, Node) and mm.kind == "matmul"):
            return None
        a, b = mm.ins
        if not (_is_cast(a, np.float16, np.float32) and _is_cast(b, np.float16, np.float32)):
            return None
        la, lb = a.ins[0], b.ins[0]
        if not (_rect2d(la) and _rect2d(lb)):
            return None
        pairs.append((la, lb))
        acc = prev
    if not (isinstance(acc, Node) and acc.kind == "const" and float(acc.attrs["value"]) == 0.0):
        return None
    if not pairs:
        return None
    pairs.reverse()
    ldc = t.strides[0]
    i0, j0 = divmod(t.off, ldc)
    bm, bn = t.shape
    return i0, j0, bm, bn, pairs


def match_gemm(low, stores: List[Store]):
    if not stores:
        return None
    tiles = []
    abuf = bbuf = cbuf = None
    lda = ldb = ldc = None
    K = None
    for s in stores:
        ch = gemm_chain(s)
        if ch is None:
            return None
        i0, j0, bm, bn, pairs = ch
        la0, lb0 = pairs[0]
        if abuf is None:
            abuf, bbuf, cbuf = la0.attrs["buf"], lb0.attrs["buf"], s.target.buf
            lda, ldb, ldc = la0.attrs["strides"][0], lb0.attrs["strides"][0], s.target.strides[0]
        if s.target.buf is not cbuf or s.target.strides[0] != ldc:
            return None
        k_next = 0
        for la, lb in pairs:
            if la.attrs["buf"] is not abuf or lb.attrs["buf"] is not bbuf:
                return None
            if la.attrs["strides"][0] != lda or lb.attrs["strides"][0] != ldb:
                return None
            ai, ak = divmod(la.attrs["off"], lda)
            bk_, bj = divmod(lb.attrs["off"], ldb)
            if ai != i0 or bj != j0 or ak != k_next or bk_ != k_next:
                return None
            if la.shape[0] != bm or lb.shape[1] != bn or la.shape[1] != lb.shape[0]:
                return None
            k_next += la.shape[1]
        if K is None:
            K = k_next
        elif K != k_next:
            return None
        tiles.append((i0, j0, bm, bn))
    if abuf is cbuf or bbuf is cbuf:
        return None
    Mfull = cbuf.numel // ldc
    Nfull = ldc
    if lda != K or abuf.numel != Mfull * K or bbuf.numel != K * Nfull or ldb != Nfull:
        return None
    # the stores must tile one rectangle of C exactly (all of C, or the block
    # a shard of the core grid owns)
    i_lo = min(t[0] for t in tiles)
    j_lo = min(t[1] for t in tiles)
    i_hi = max(t[0] + t[2] for t in tiles)
    j_hi = max(t[1] + t[3] for t in tiles)
    M, N = i_hi - i_lo, j_hi - j_lo
    if i_hi > Mfull or j_hi > Nfull:
        return None
    cover = np.zeros((M, N), dtype=np.int8) if M * N <= (1 << 26) else None
    area = 0
    for i0, j0, bm, bn in tiles:
        area += bm * bn
        if cover is not None:
            cover[i0 - i_lo:i0 - i_lo + bm, j0 - j_lo:j0 - j_lo + bn] += 1
    if area != M * N or (cover is not None and not np.all(cover == 1)):
        return None
    if M % GEMM_TILE_M or N % GEMM_TILE_N or K % GEMM_TILE_K:
        return None
    lib = R.load_library()
    sa, sb, sc = low.slots[abuf.index], low.slots[bbuf.index], low.slots[cbuf.index]
    a_off, b_off, c_off = i_lo * lda * 2, j_lo * 2, (i_lo * ldc + j_lo) * 2

    def run(bufs, stream, status):
        d = R.KtirGemmDesc()
        d.a, d.b, d.c = bufs.base[sa] + a_off, bufs.base[sb] + b_off, bufs.base[sc] + c_off
        d.lda, d.ldb, d.ldc = lda, ldb, ldc
        d.m, d.n, d.k = M, N, K
        d.add_zero = 1
        d.status = status
        R.check(lib.ktir_gemm_f16(C.byref(d), stream), "ktir_gemm_f16")

    from .lower import Launch, Plan
    plan = Plan("gemm", [Launch(run, "gemm")], [], status_check=True)
    plan.info.update(m=M, n=N, k=K, tiles=len(tiles), flops=2 * M * N * K)
    return plan


def match_attention(low, stores: List[Store]):
    from .rewrite import match_attention_plan
    return match_attention_plan(low, stores)
