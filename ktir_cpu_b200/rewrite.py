"""The attention rewrite: online-softmax KV loops become one attention node.

A KTIR attention kernel walks K/V blocks in an ``scf.for`` whose iter_args
carry the running row max ``m``, row sum ``l`` and output accumulator ``acc``
(the pattern of examples/triton-ktir/paged_attention.mlir and of the causal
attention workload here).  Executed op by op that loop is dozens of small
tile ops per block; this pass recognises it structurally and lets the tracer
replace the whole loop with a single node, while still evaluating the
loop's scalar and addressing ops per iteration (so every K/V block's
location, the causal offsets and the scale come from the program itself).
The lowering then maps the normalised result ``acc / l`` onto the tcgen05
flash-attention kernel.

Recognised loop body (roles by dataflow, other ops must be scalar / view /
constant ops):

    K, V   = load(access tile), load(access tile)       (both depend on the iv)
    Kt     = transpose(extf K)                           permutation [1, 0]
    S      = matmul(Q, Kt) outs(zero)                    Q defined outside the loop
    Ss     = mulf S, scale                               scale: outer scalar
    Sm     = generic(Ss){ row = index 0 + a; col = index 1 + b;
                          select(cmpi sgt col, row), -inf, x }     (optional)
    mb     = reduce maxnumf(Sm)                          over dim 1
    m_new  = maxnumf m_i, mb
    P      = generic(Sm, m_new){ exp(x - m) }            row broadcast of m_new
    alpha  = generic(m_i, m_new){ exp(a - b) }
    l_new  = addf(mulf(l_i, alpha), reduce addf(P))
    acc_s  = generic(acc_i, alpha){ mulf }               row broadcast of alpha
    acc_n  = matmul(P, extf V) outs(acc_s)
    yield m_new, l_new, acc_n
"""

from __future__ import annotations

import os

from typing import Any, Dict, List, Optional

import numpy as np

from .ir import IRFunction, Operation, iter_ops

TILE_OPS_OK = {"arith.constant", "tensor.empty", "tensor.splat", "ktdp.construct_access_tile",
               "scf.yield"}


def _defs(ops: List[Operation]) -> Dict[str, Operation]:
    d = {}
    for op in ops:
        for r in op.results:
            d[r] = op
    return d


def _region_ops(op: Operation) -> List[str]:
    return [o.op_type for o in op.regions[0].ops] if op.regions else []


def _maps_dims(op: Operation) -> List[tuple]:
    return [tuple(e[1] for e in m.exprs if e[0] == "d") for m in op.attributes.get("indexing_maps", [])]


def match_attention_loop(loop: Operation) -> Optional[Dict[str, Any]]:
    if loop.op_type != "scf.for" or len(loop.attributes.get("iter_args", [])) != 3:
        return None
    body = loop.regions[0].ops
    iv = loop.attributes["iter_var"]
    it = loop.attributes["iter_args"]
    d = _defs(body)
    yld = body[-1] if body and body[-1].op_type == "scf.yield" else None
    if yld is None or len(yld.operands) != 3:
        return None
    roles: Dict[str, str] = {}

    def op_of(name):
        return d.get(name)

    # find the two matmuls: S (Q, Kt) and the PV accumulation (P, V)
    mms = [o for o in body if o.op_type == "linalg.matmul"]
    if len(mms) != 2:
        return None
    s_mm = pv_mm = None
    for mm in mms:
        outs = op_of(mm.operands[2]) if len(mm.operands) > 2 else None
        if outs is not None and outs.op_type == "linalg.generic":
            pv_mm = mm
        else:
            s_mm = mm
    if s_mm is None or pv_mm is None:
        return None
    q_name, kt_name = s_mm.operands[0], s_mm.operands[1]
    if q_name in d:
        return None  # Q must come from outside the loop
    tr = op_of(kt_name)
    if tr is None or tr.op_type != "linalg.transpose" or tr.attributes["permutation"] != [1, 0]:
        return None
    k_ext = op_of(tr.operands[0])
    if k_ext is None or k_ext.op_type != "arith.extf":
        return None
    k_load = op_of(k_ext.operands[0])
    if k_load is None or k_load.op_type != "ktdp.load":
        return None
    s0 = op_of(s_mm.operands[2]) if len(s_mm.operands) > 2 else None
    if s0 is None or s0.op_type not in ("arith.constant", "tensor.empty") or \
            (s0.op_type == "arith.constant" and float(s0.attributes.get("value", 1)) != 0.0):
        return None
    # scale
    s_name = s_mm.results[0]
    scale_op = next((o for o in body if o.op_type == "arith.mulf" and s_name in o.operands), None)
    if scale_op is None:
        return None
    scale_name = [x for x in scale_op.operands if x != s_name]
    if len(scale_name) != 1 or scale_name[0] in d:
        return None
    ss_name = scale_op.results[0]
    # optional causal mask
    mask = None
    sm_name = ss_name
    users = [o for o in body if ss_name in o.operands and o is not scale_op]
    gen = [o for o in users if o.op_type == "linalg.generic"]
    if gen:
        g = gen[0]
        if g.operands[0] != ss_name or g.attributes["n_ins"] != 1:
            return None
        seq = [o.op_type for o in g.regions[0].ops]
        if seq != ["linalg.index", "linalg.index", "arith.addi", "arith.addi", "arith.cmpi",
                   "arith.select", "linalg.yield"]:
            return None
        rops = g.regions[0].ops
        idx = {rops[0].results[0]: rops[0].attributes["dim"],
               rops[1].results[0]: rops[1].attributes["dim"]}
        offs = {}
        for addi in rops[2:4]:
            a, b = addi.operands
            if a in idx:
                offs[addi.results[0]] = (idx[a], b)
            elif b in idx:
                offs[addi.results[0]] = (idx[b], a)
            else:
                return None
        cmpi = rops[4]
        if cmpi.attributes["predicate"] != "sgt":
            return None
        lhs, rhs = cmpi.operands[:2]
        if lhs not in offs or rhs not in offs or offs[lhs][0] != 1 or offs[rhs][0] != 0:
            return None
        sel = rops[5]
        x_arg = g.regions[0].args[0][0] if g.regions[0].args else None
        if sel.operands[0] != cmpi.results[0] or sel.operands[2] != x_arg:
            return None
        mask = {"koff": offs[lhs][1], "qoff": offs[rhs][1], "neg": sel.operands[1]}
        sm_name = g.results[0]
    # running max
    red_max = next((o for o in body if o.op_type == "linalg.reduce" and o.operands[0] == sm_name
                    and o.attributes.get("combiner") == "arith.maxnumf"), None)
    if red_max is None or red_max.attributes.get("dims") != [1]:
        return None
    mnew = next((o for o in body if o.op_type == "arith.maxnumf" and red_max.results[0] in o.operands),
                None)
    if mnew is None:
        return None
    m_i = [x for x in mnew.operands if x != red_max.results[0]]
    if len(m_i) != 1 or m_i[0] not in it:
        return None
    m_i = m_i[0]
    mn = mnew.results[0]

    def exp_sub_generic(o, a, b, maps):
        return (o.op_type == "linalg.generic" and o.operands[:2] == [a, b] and
                o.attributes["n_ins"] == 2 and _maps_dims(o)[:2] == maps and
                _region_ops(o) == ["arith.subf", "math.exp", "linalg.yield"])
    p_gen = next((o for o in body if exp_sub_generic(o, sm_name, mn, [(0, 1), (0,)])), None)
    a_gen = next((o for o in body if exp_sub_generic(o, m_i, mn, [(0,), (0,)])), None)
    if p_gen is None or a_gen is None:
        return None
    p_name, alpha = p_gen.results[0], a_gen.results[0]
    red_sum = next((o for o in body if o.op_type == "linalg.reduce" and o.operands[0] == p_name and
                    o.attributes.get("combiner") == "arith.addf"), None)
    if red_sum is None:
        return None
    lsc = next((o for o in body if o.op_type == "arith.mulf" and alpha in o.operands and
                any(x in it for x in o.operands)), None)
    if lsc is None:
        return None
    l_i = [x for x in lsc.operands if x != alpha][0]
    lnew = next((o for o in body if o.op_type == "arith.addf" and lsc.results[0] in o.operands and
                 red_sum.results[0] in o.operands), None)
    if lnew is None:
        return None
    accs = op_of(pv_mm.operands[2])
    if not (accs.operands[:2] and accs.operands[1] == alpha and accs.operands[0] in it and
            _region_ops(accs) == ["arith.mulf", "linalg.yield"] and
            _maps_dims(accs)[:2] == [(0, 1), (0,)]):
        return None
    acc_i = accs.operands[0]
    if pv_mm.operands[0] != p_name:
        return None
    v_ext = op_of(pv_mm.operands[1])
    if v_ext is None or v_ext.op_type != "arith.extf":
        return None
    v_load = op_of(v_ext.operands[0])
    if v_load is None or v_load.op_type != "ktdp.load":
        return None
    order = {m_i: mn, l_i: lnew.results[0], acc_i: pv_mm.results[0]}
    if [order.get(x) for x in it] != list(yld.operands):
        return None
    # every other body op must be scalar / addressing / constant work
    tile_ops = {id(o) for o in (k_load, v_load, k_ext, v_ext, tr, s_mm, scale_op, red_max, mnew,
                                p_gen, a_gen, red_sum, lsc, lnew, accs, pv_mm, s0)}
    if gen:
        tile_ops.add(id(gen[0]))
    for o in body:
        if id(o) in tile_ops:
            continue
        if o.op_type in ("arith.addi", "arith.muli", "arith.subi", "arith.divui", "arith.remui",
                         "arith.index_cast") or o.op_type in TILE_OPS_OK:
            continue
        return None
    return {
        "iv": iv, "iter_args": it, "m": m_i, "l": l_i, "acc": acc_i,
        "q": q_name, "k_load": k_load, "v_load": v_load, "scale": scale_name[0], "mask": mask,
        "tile_op_ids": tile_ops, "body": body,
    }


def attention_rewrites(func: IRFunction) -> Dict[int, Any]:
    """Map id(scf.for) -> tracer handler for every recognised attention loop."""
    out: Dict[int, Any] = {}
    for op in iter_ops(func.operations):
        info = match_attention_loop(op)
        if info is not None:
            out[id(op)] = _make_handler(info)
    return out


def _make_handler(info):
    def handler(tracer, op):
        from .trace import DataDependentError, Node, _concrete, _is_tile, _need_int
        core = tracer.core
        lb, ub, st = (_need_int(core.get(o), "scf.for bound") for o in op.operands[:3])
        inits = [core.get(o) for o in op.operands[3:]]
        names = info["iter_args"]
        for n, v in zip(names, inits):
            core.set(n, v)
            if _is_tile(v):
                core.track(n, v.nbytes)
        init = dict(zip(names, inits))
        m0, l0, a0 = init[info["m"]], init[info["l"]], init[info["acc"]]
        ok_init = (isinstance(m0, Node) and m0.kind == "const" and np.isneginf(float(m0.attrs["value"]))
                   and isinstance(l0, Node) and l0.kind == "const" and float(l0.attrs["value"]) == 0.0
                   and isinstance(a0, Node) and a0.kind == "const" and float(a0.attrs["value"]) == 0.0)
        q = core.get(info["q"])
        if not ok_init or not (isinstance(q, Node) and q.kind == "ew" and q.attrs.get("op") == "cast"):
            raise DataDependentError("attention loop with unsupported initial state")
        q_load = q.ins[0]
        scale = core.get(info["scale"])
        if not _concrete(scale):
            raise DataDependentError("attention scale depends on tile data")
        scale16 = float(np.float16(scale))      # float binops round scalar operands to f16
        k_tiles, v_tiles, offs = [], [], []
        body = info["body"]
        skip = info["tile_op_ids"]
        for i in range(lb, ub, max(st, 1)):
            core.push()
            core.set(info["iv"], i)
            for bop in body:
                if bop.op_type == "scf.yield":
                    continue
                if id(bop) in skip:
                    if bop is info["k_load"] or bop is info["v_load"]:
                        at = core.get(bop.operands[0])
                        ld = tracer.op_ktdp_load(bop)
                        (k_tiles if bop is info["k_load"] else v_tiles).append(ld)
                    continue
                if bop.op_type in ("tensor.empty", "tensor.splat", "arith.constant") and \
                        bop.result_types and "tensor<" in (bop.result_types[0] or ""):
                    continue
                tracer.run_op(bop)
            if info["mask"] is not None:
                offs.append((int(core.get(info["mask"]["qoff"])), int(core.get(info["mask"]["koff"]))))
            core.pop()
        bq, d = a0.shape
        attn = tracer.node("attention", (bq, d), np.float32, (q_load,),
                           {"k": k_tiles, "v": v_tiles, "scale": scale16,
                            "causal_offsets": offs if info["mask"] is not None else None})
        m = tracer.node("attn_out", (bq,), np.float32, (attn,), {"which": "m"})
        l_ = tracer.node("attn_out", (bq,), np.float32, (attn,), {"which": "l"})
        acc = tracer.node("attn_out", (bq, d), np.float32, (attn,), {"which": "acc"})
        res = {info["m"]: m, info["l"]: l_, info["acc"]: acc}
        for n in names:
            core.untrack(n)
            core.set(n, res[n])
            core.track(n, res[n].nbytes)
        out = [res[n] for n in names]
        return tuple(out)
    return handler


def attention_problem(stores, seq_hint=None):
    """The attention problem a list of stores computes, when every store is
    f16(acc / l) of an attention node over one [bh*seq, d] Q/K/V/O set:
    {q, k, v, o buffers, bq, d, causal, scale, seq, rows (query row of each
    unit)}, else None.  A causal problem's sequence length is taken from its
    last query block unless seq_hint gives it (a subset of the units, such as
    one GPU's share of a split, need not contain the last block)."""
    from .trace import Node, RectTarget
    if not stores:
        return None
    units = []
    for s in stores:
        t = s.target
        v = s.value
        if not isinstance(t, RectTarget) or t.dtype != np.float16 or len(t.shape) != 2:
            return None
        if not (isinstance(v, Node) and v.kind == "ew" and v.attrs.get("op") == "cast" and
                v.dtype == np.float16):
            return None
        dv = v.ins[0]
        if not (dv.kind == "ew" and dv.attrs.get("op") == "div"):
            return None
        a, b = dv.ins
        if not (a.kind == "bcast" and b.kind == "bcast" and a.attrs["map"] == (0, 1) and
                b.attrs["map"] == (0,)):
            return None
        acc, l_ = a.ins[0], b.ins[0]
        if not (acc.kind == "attn_out" and l_.kind == "attn_out" and acc.attrs["which"] == "acc"
                and l_.attrs["which"] == "l" and acc.ins[0] is l_.ins[0]):
            return None
        units.append((acc.ins[0], t))
    attn0, t0 = units[0]
    q0 = attn0.ins[0]
    bq, d = attn0.shape
    qbuf, kbuf, vbuf, obuf = q0.attrs["buf"], attn0.attrs["k"][0].attrs["buf"], \
        attn0.attrs["v"][0].attrs["buf"], t0.buf
    if d != 128 or obuf.index in (qbuf.index, kbuf.index, vbuf.index):
        return None
    ld = t0.strides[0]
    if ld != d or any(x.attrs["strides"] != (d, 1) for x in [q0]):
        return None
    rows = qbuf.numel // d
    causal = attn0.attrs["causal_offsets"] is not None
    scale = attn0.attrs["scale"]
    # infer seq from the causal offsets (last q block) or from the K sweep length
    seen = set()
    seq = None
    last_end = 0
    for attn, t in units:
        q = attn.ins[0]
        if attn.attrs["scale"] != scale or (attn.attrs["causal_offsets"] is not None) != causal:
            return None
        qrow = q.attrs["off"] // d
        if t.off // d != qrow or t.shape != (bq, d) or q.shape != (bq, d):
            return None
        ks, vs = attn.attrs["k"], attn.attrs["v"]
        if len(ks) != len(vs) or not ks:
            return None
        bk = ks[0].shape[0]
        krow0 = ks[0].attrs["off"] // d
        for i, (kl, vl) in enumerate(zip(ks, vs)):
            if kl.attrs["buf"] is not kbuf or vl.attrs["buf"] is not vbuf:
                return None
            if kl.attrs["off"] != vl.attrs["off"] or kl.attrs["off"] // d != krow0 + i * bk:
                return None
            if kl.shape != (bk, d) or kl.attrs["strides"] != (d, 1):
                return None
        if causal:
            offs = attn.attrs["causal_offsets"]
            qoff = offs[0][0]
            if any(o[0] != qoff or o[1] != i * bk for i, o in enumerate(offs)):
                return None
            if qrow - qoff != krow0 or len(ks) * bk != qoff + bq:
                return None
            last_end = max(last_end, qoff + bq)
            seq = seq_hint if seq_hint is not None else max(seq or 0, qoff + bq)
        else:
            seq_u = len(ks) * bk
            if seq is not None and seq != seq_u:
                return None
            seq = seq_u
        seen.add(qrow)
    if seq is None or seq % 128 or rows % seq or not scale > 0 or last_end > seq:
        return None
    return {"q": qbuf, "k": kbuf, "v": vbuf, "o": obuf, "bq": bq, "d": d, "causal": causal,
            "scale": scale, "seq": seq, "n_rows": rows, "rows": seen}


def match_attention_plan(low, stores):
    """All stores are f16(acc / l) of attention nodes that tile a [bh*seq, d]
    problem: whole heads (one GPU, or a split whose cores own whole heads) run
    the fused kernel over those heads; a split whose cores own stretches of
    every head's sequence runs the K/V ring across the GPUs."""
    import ctypes as C
    from . import runtime as R
    from .lower import Launch, Plan
    hint = None
    if low.shard is not None:
        whole = attention_problem(low.all_stores)
        hint = whole["seq"] if whole is not None else None
    prob = attention_problem(stores, hint)
    if prob is None:
        return None
    qbuf, kbuf, vbuf, obuf = prob["q"], prob["k"], prob["v"], prob["o"]
    bq, d, causal, scale, seq, seen = (prob[k] for k in ("bq", "d", "causal", "scale", "seq", "rows"))
    # the units must cover whole heads [h_lo, h_hi) (all heads, or a shard's)
    heads = sorted({q // seq for q in seen})
    h_lo, h_hi = heads[0], heads[-1] + 1
    if len(seen) * bq != (h_hi - h_lo) * seq or heads != list(range(h_lo, h_hi)):
        if low.shard is not None:
            from .ring import ring_attention_plan
            # KTIR_KV_EXCHANGE picks how the K/V shares travel (ring.EXCHANGES)
            return ring_attention_plan(low, prob,
                                       os.environ.get("KTIR_KV_EXCHANGE", "copy_overlap"))
        return None
    bh = h_hi - h_lo
    off = h_lo * seq * d * 2
    lib = R.load_library()
    sq, sk, sv, so = (low.slots[b.index] for b in (qbuf, kbuf, vbuf, obuf))

    def run(bufs, stream, status):
        dsc = R.KtirFmhaDesc()
        dsc.q, dsc.k, dsc.v, dsc.o = (bufs.base[sq] + off, bufs.base[sk] + off,
                                      bufs.base[sv] + off, bufs.base[so] + off)
        dsc.bh, dsc.seq, dsc.d = bh, seq, d
        dsc.scale = scale
        dsc.causal = 1 if causal else 0
        dsc.row_stride = d
        dsc.status = status
        R.check(lib.ktir_fmha_f16(C.byref(dsc), stream), "ktir_fmha_f16")
    plan = Plan("attention", [Launch(run, "fmha")], [], status_check=True)
    flops = 4 * bh * seq * seq * d // (2 if causal else 1)
    plan.info.update(bh=bh, seq=seq, d=d, causal=causal, scale=scale, flops=flops)
    if low.shard is not None:
        # a split reads only its heads' rows of Q, K and V: (buffer index, byte ranges)
        plan.info["upload_ranges"] = {b.index: [(off, bh * seq * d * 2)]
                                      for b in (qbuf, kbuf, vbuf)}
    return plan
