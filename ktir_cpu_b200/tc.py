"""Tensor-core programs: GEMM and attention matchers over the traced graph.

GEMM: every store must be the K loop of ``linalg.matmul`` over one output
tile, starting from a zero constant, with the A_k / B_k loads sweeping K
contiguously, and the stores must tile one rectangle of C exactly.  Two
forms (ktir_cpu/dialects/linalg_ops.py:273-297, ops/arith_ops.py:403-419):

* widened: ``truncf(acc_K)``, ``acc_k = acc_{k-1} + extf(A_k) @ extf(B_k)``
  (f32 tiles, f32 accumulator): one f32 sum over all of K, rounded once;
* f16 products: ``acc_k = acc_{k-1} + A_k @ B_k`` with f16 tiles, where
  NumPy rounds each block product to f16 and the accumulator is f16 (each
  sum rounded) or f32 (the reference's matmul_fwd example, and matmuls of
  f16 tiles into f32 outs).

The whole call becomes one tcgen05 GEMM launch: the aligned persistent
kernel for widened tilings of 128 x 128 x 64 multiples (256-wide output tiles
where they fill the GPU, 128-wide ones for a slice too small to), else the blocked
kernel (any shape, per-block rounding).  Numerics: the reference sums each
tile in OpenBLAS / NumPy order, the tensor cores in their own order — equal
within the stated tolerance, not bit-exact.

Attention: see :mod:`ktir_cpu_b200.rewrite`.
"""

from __future__ import annotations

import ctypes as C
from typing import List

import numpy as np

from . import runtime as R
from .trace import Node, RectTarget, Store

GEMM_TILE_M, GEMM_TILE_N, GEMM_TILE_K = 128, 128, 64


def _is_cast(n, src, dst) -> bool:
    return isinstance(n, Node) and n.kind == "ew" and n.attrs.get("op") == "cast" and \
        n.dtype == dst and n.ins[0].dtype == src


def _rect2d(n) -> bool:
    return isinstance(n, Node) and n.kind == "load" and n.attrs["mode"] == "rect" and \
        len(n.shape) == 2 and n.attrs["strides"][1] == 1


def _is_zero(n) -> bool:
    return isinstance(n, Node) and n.kind == "const" and float(n.attrs["value"]) == 0.0


def _block_term(n):
    """(kind, A load, B load) when n is one K block's product: "wide" for
    extf(A) @ extf(B), "f16" for A @ B of f16 tiles (rounded to f16)."""
    if not (isinstance(n, Node) and n.kind == "matmul"):
        return None
    a, b = n.ins
    if _is_cast(a, np.float16, np.float32) and _is_cast(b, np.float16, np.float32) and \
            _rect2d(a.ins[0]) and _rect2d(b.ins[0]):
        return "wide", a.ins[0], b.ins[0]
    if n.dtype == np.float16 and _rect2d(a) and _rect2d(b) and \
            a.dtype == np.float16 and b.dtype == np.float16:
        return "f16", a, b
    return None


def gemm_chain(store: Store):
    """(i0, j0, bm, bn, [(A load, B load), ...], kind, accumulator dtype) for
    one output tile, or None."""
    t = store.target
    if not isinstance(t, RectTarget) or len(t.shape) != 2 or t.strides[1] != 1 or \
            t.dtype != np.float16:
        return None
    root = store.value
    if _is_cast(root, np.float32, np.float16):
        acc, acc_dt = root.ins[0], np.dtype(np.float32)
    elif isinstance(root, Node) and root.dtype == np.float16:
        acc, acc_dt = root, np.dtype(np.float16)
    else:
        return None
    pairs, kinds = [], set()
    while not _is_zero(acc):
        if not (isinstance(acc, Node) and acc.kind == "ew" and acc.attrs.get("op") == "add" and
                acc.dtype == acc_dt and len(acc.ins) == 2):
            return None
        prev, term = acc.ins
        if acc.attrs.get("matmul_accumulate"):
            bt = _block_term(term)                       # outs + A @ B
        else:
            # acc + (empty + A @ B): the block product added to the running sum
            if _block_term(prev) is not None or (isinstance(prev, Node) and
                                                 prev.attrs.get("matmul_accumulate")):
                prev, term = term, prev
            inner = term
            if isinstance(term, Node) and term.kind == "ew" and term.attrs.get("matmul_accumulate") \
                    and _is_zero(term.ins[0]):
                inner = term.ins[1]
            bt = _block_term(inner)
            if bt is not None and bt[0] != "f16":
                return None
        if bt is None:
            return None
        kinds.add(bt[0])
        pairs.append((bt[1], bt[2]))
        acc = prev
    if not pairs or len(kinds) != 1:
        return None
    kind = kinds.pop()
    if kind == "wide" and acc_dt != np.float32:
        return None
    pairs.reverse()
    ldc = t.strides[0]
    i0, j0 = divmod(t.off, ldc)
    bm, bn = t.shape
    return i0, j0, bm, bn, pairs, kind, acc_dt


def match_gemm(low, stores: List[Store]):
    if not stores:
        return None
    tiles = []
    abuf = bbuf = cbuf = None
    lda = ldb = ldc = None
    K = None
    mode = None
    for s in stores:
        ch = gemm_chain(s)
        if ch is None:
            return None
        i0, j0, bm, bn, pairs, kind, acc_dt = ch
        widths = {la.shape[1] for la, _ in pairs}
        m = (kind, acc_dt, widths.pop() if len(widths) == 1 else None)
        if mode is None:
            mode = m
        elif mode != m:
            return None
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
    if abuf.numel != Mfull * lda or lda < K or bbuf.numel < K * ldb or ldb < Nfull:
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
    lib = R.load_library()
    sa, sb, sc = low.slots[abuf.index], low.slots[bbuf.index], low.slots[cbuf.index]
    a_off, b_off, c_off = i_lo * lda * 2, j_lo * 2, (i_lo * ldc + j_lo) * 2
    kind, acc_dt, width = mode
    from .lower import Launch, Plan
    aligned = not (M % GEMM_TILE_M or N % GEMM_TILE_N or K % GEMM_TILE_K) and lda == K and \
        ldb == Nfull
    if kind != "wide" or not aligned:
        # f16 block products (rounded per block), or a shape the aligned kernel does not take
        block_k = 0 if kind == "wide" else width
        if block_k is None or block_k % 16 or lda % 8 or ldb % 8 or \
                (a_off | b_off) % 16:
            return None

        def run_blocked(bufs, stream, status):
            d = R.KtirGemmBlockedDesc()
            d.a, d.b, d.c = bufs.base[sa] + a_off, bufs.base[sb] + b_off, bufs.base[sc] + c_off
            d.lda, d.ldb, d.ldc = lda, ldb, ldc
            d.m, d.n, d.k = M, N, K
            d.block_k = block_k
            d.acc_f16 = 1 if acc_dt == np.float16 else 0
            d.status = status
            R.check(lib.ktir_gemm_f16_blocked(C.byref(d), stream), "ktir_gemm_f16_blocked")
        plan = Plan("gemm", [Launch(run_blocked, "gemm_blocked")], [], status_check=True)
        plan.info.update(m=M, n=N, k=K, tiles=len(tiles), flops=2 * M * N * K, block_k=block_k,
                         acc=str(acc_dt))
        return plan

    def run(bufs, stream, status):
        d = R.KtirGemmDesc()
        d.a, d.b, d.c = bufs.base[sa] + a_off, bufs.base[sb] + b_off, bufs.base[sc] + c_off
        d.lda, d.ldb, d.ldc = lda, ldb, ldc
        d.m, d.n, d.k = M, N, K
        d.add_zero = 1
        d.status = status
        R.check(lib.ktir_gemm_f16(C.byref(d), stream), "ktir_gemm_f16")

    plan = Plan("gemm", [Launch(run, "gemm")], [], status_check=True)
    plan.info.update(m=M, n=N, k=K, tiles=len(tiles), flops=2 * M * N * K)
    return plan


def match_attention(low, stores: List[Store]):
    from .rewrite import match_attention_plan
    return match_attention_plan(low, stores)
