"""Attention split over the sequence across GPUs, K/V blocks passed in a ring.

A KTIR attention program whose cores own stretches of every head's sequence
(the benchmark's zigzag layout: query blocks b and nq-1-b of every head on
one core) is split across GPUs by contiguous core ranges.  Each GPU then
owns some 128-row query tiles of every head, and needs the K/V rows of every
earlier tile, most of which belong to other GPUs' query tiles.  The K/V rows
of a GPU's own tiles ("its share") are packed into one contiguous block of a
staging buffer that holds every GPU's share one after the other; in step t
each GPU adds the key tiles of share (rank - t) mod world to its queries
(the partial attention entry point, ktir_fmha_f16_part, carrying the
online-softmax state between steps), while NCCL sends that share on to the
next GPU and receives share (rank - t - 1) mod world from the previous one.
After world steps every GPU has added every key tile and writes its query
tiles of O.  The reference has no multi-device execution: its cores read
K/V from one simulated HBM (ktir_cpu/ops/memory_ops.py:438-587); the ring is
how the same reads reach a GPU that does not hold them.

The pure functions here (tile ownership, staging layout, step masks) are
the host logic, tested on CPU; ring_attention_plan builds the device plan.
"""

from __future__ import annotations

from typing import Dict, List, Optional, Sequence, Tuple

TILE = 128


def query_tiles(rows: Sequence[int], seq: int, bq: int) -> Optional[List[int]]:
    """The 128-row query tiles that a set of query-block row offsets covers,
    when every head covers the same tiles and every covered tile is whole;
    else None."""
    per_tile = TILE // bq if TILE % bq == 0 else 0
    if per_tile == 0:
        return None
    heads: Dict[int, Dict[int, int]] = {}
    for r in rows:
        h, off = divmod(r, seq)
        t = off // TILE
        heads.setdefault(h, {})
        heads[h][t] = heads[h].get(t, 0) + 1
    if not heads:
        return None
    sets = {tuple(sorted(d)) for d in heads.values()}
    if len(sets) != 1:
        return None
    if any(c != per_tile for d in heads.values() for c in d.values()):
        return None
    return list(next(iter(sets)))


def staging_layout(tiles_of: Sequence[Sequence[int]], n_tiles: int):
    """(kv_owner, kv_local, kv_tiles) for the staging buffer: key tile kt of a
    head lives in share kv_owner[kt] at local index kv_local[kt]; every share
    is kv_tiles tiles per head.  The shares must partition the tiles."""
    owner = [-1] * n_tiles
    local = [0] * n_tiles
    for s, tiles in enumerate(tiles_of):
        for i, t in enumerate(sorted(tiles)):
            if not 0 <= t < n_tiles or owner[t] != -1:
                raise ValueError(f"query tile {t} owned twice or out of range")
            owner[t], local[t] = s, i
    if -1 in owner:
        raise ValueError("the shares do not cover every query tile")
    return owner, local, max(len(t) for t in tiles_of)


def step_shares(rank: int, world: int) -> List[int]:
    """The share whose key tiles each step adds: share (rank - t) mod world at step t."""
    return [(rank - t) % world for t in range(world)]


def share_mask(tiles: Sequence[int]) -> int:
    m = 0
    for t in tiles:
        m |= 1 << t
    return m


EXCHANGES = ("gather", "allgather", "ring")


def ring_attention_plan(low, prob, exchange: str = "gather"):
    """Device plan for one rank (see the module docstring).

    exchange "gather": the rank packs its share (ktir_pack_kv) into the
    staging buffer ([world][K | V][head][tile][128][d] f16), one NCCL
    all-gather fills in the others' shares, then one attention kernel adds
    every key tile from the staging buffer (no carried state; the exchange
    has the GPU to itself).  The overlapped forms: step 0 adds the rank's own
    key tiles straight from the call's K and V while a high-priority comm
    stream packs and passes the shares, and the later steps add the other
    shares from the staging buffer, the softmax state carried between steps:
    "allgather" passes them with one NCCL all-gather, then one kernel for
    every other share; "ring" with world - 1 NCCL send/recv steps, each GPU
    forwarding the share it last received, one kernel per arrived share."""
    import ctypes as C

    import torch
    import torch.distributed as dist

    from . import runtime as R
    from .lower import Launch, Plan, core_range
    from .rewrite import attention_problem

    rank, world, group = low.shard
    seq, bq, d = prob["seq"], prob["bq"], prob["d"]
    if d != 128 or seq % TILE or seq > 32 * TILE or not prob["causal"]:
        return None
    n_tiles = seq // TILE
    bh = prob["n_rows"] // seq
    nx, ny, nz = low.trace.grid
    tiles_of = []
    for r in range(world):
        c0, c1 = core_range(r, world, nx * ny * nz)
        pr = attention_problem([s for s in low.all_stores if c0 <= s.core < c1], seq)
        if pr is None or pr["q"] is not prob["q"] or pr["k"] is not prob["k"]:
            return None
        tl = query_tiles(pr["rows"], seq, bq)
        if tl is None:
            return None
        tiles_of.append(tl)
    try:
        owner, local, kv_tiles = staging_layout(tiles_of, n_tiles)
    except ValueError:
        return None
    if len({len(t) for t in tiles_of}) != 1:
        return None                       # equal shares: NCCL all-gather and same-size sends
    mine = tiles_of[rank]
    dev = low.device
    share_rows = bh * kv_tiles * TILE
    row_bytes = d * 2
    kv_all = torch.empty(world * 2 * share_rows * d, dtype=torch.float16, device=dev)
    if exchange not in EXCHANGES:
        raise ValueError(f"K/V exchange {exchange!r}: expected one of {EXCHANGES}")
    # the overlapped forms carry the softmax state between their steps
    o_acc = ml = None
    if exchange != "gather":
        o_acc = torch.empty(bh * len(mine) * TILE * d, dtype=torch.float32, device=dev)
        ml = torch.empty(bh * len(mine) * TILE * 2, dtype=torch.float32, device=dev)
    lib = R.load_library()
    sq, sk, sv, so = (low.slots[b.index] for b in (prob["q"], prob["k"], prob["v"], prob["o"]))
    # high priority: the packing and NCCL kernels take their SMs ahead of the
    # attention kernel's CTAs, which would otherwise fill every SM first
    comm = (torch.cuda.Stream(dev, priority=-1) if dev.type == "cuda" and exchange != "gather"
            else None)
    own_mask = share_mask(mine)
    all_mask = share_mask(range(n_tiles))

    def desc(mask, first, last, staged):
        dsc = R.KtirFmhaPartDesc()
        dsc.bh, dsc.seq, dsc.d = bh, seq, d
        dsc.scale, dsc.causal = prob["scale"], 1
        dsc.n_qtiles = len(mine)
        dsc.key_mask = mask
        dsc.flags = (1 if first else 0) | (2 if last else 0)
        if o_acc is not None:
            dsc.o_acc, dsc.ml = o_acc.data_ptr(), ml.data_ptr()
        for i, qt in enumerate(mine):
            dsc.qtiles[i] = qt
        if staged:
            # K of share s at rows ((2s * bh + h) * kv_tiles + i) * 128, V one share later
            dsc.kv_tiles, dsc.kv_rows = kv_tiles, (2 * world - 1) * share_rows
            dsc.k = kv_all.data_ptr()
            dsc.v = kv_all.data_ptr() + share_rows * row_bytes
            for kt in range(n_tiles):
                dsc.kv_owner[kt], dsc.kv_local[kt] = 2 * owner[kt], local[kt]
        else:
            # the call's own K / V: tile kt of head h at row h * seq + kt * 128
            dsc.kv_tiles, dsc.kv_rows = n_tiles, bh * seq
            for kt in range(n_tiles):
                dsc.kv_owner[kt], dsc.kv_local[kt] = 0, kt
        return dsc

    shares = step_shares(rank, world)
    if exchange == "gather":
        steps = [desc(all_mask, True, True, True)]
    elif exchange == "ring":
        steps = [desc(own_mask, True, False, False)] + \
            [desc(share_mask(tiles_of[s]), False, t == world - 1, True)
             for t, s in enumerate(shares) if t > 0]
    else:
        steps = [desc(own_mask, True, False, False), desc(all_mask & ~own_mask, False, True, True)]
    nxt, prv = (rank + 1) % world, (rank - 1) % world
    if group is not None:
        nxt, prv = dist.get_global_rank(group, nxt), dist.get_global_rank(group, prv)

    def share(s):
        return kv_all[s * 2 * share_rows * d:(s + 1) * 2 * share_rows * d]

    def run(bufs, stream, status):
        compute = (torch.cuda.ExternalStream(stream.value, device=dev) if stream.value
                   else torch.cuda.default_stream(dev))
        if exchange == "gather":
            with torch.cuda.stream(compute):
                R.check(lib.ktir_pack_kv(C.c_void_p(share(rank).data_ptr()),
                                         C.c_void_p(bufs.base[sk]), C.c_void_p(bufs.base[sv]),
                                         bh, seq, d, own_mask, stream), "ktir_pack_kv")
                # the compute stream waits for the all-gather before the kernel
                dist.all_gather_into_tensor(kv_all, share(rank), group=group)
            k0 = steps[0]
            k0.q, k0.o, k0.status = bufs.base[sq], bufs.base[so], status
            R.check(lib.ktir_fmha_f16_part(C.byref(k0), stream), "ktir_fmha_f16_part")
            return
        # the comm stream starts after the previous execution's kernels, which
        # read the staging buffer it overwrites; its work is queued before the
        # first attention step so that it reaches the SMs first
        comm.wait_stream(compute)
        arrived = []
        with torch.cuda.stream(comm):
            cs = C.c_void_p(comm.cuda_stream)
            R.check(lib.ktir_pack_kv(C.c_void_p(share(rank).data_ptr()), C.c_void_p(bufs.base[sk]),
                                     C.c_void_p(bufs.base[sv]), bh, seq, d, own_mask, cs),
                    "ktir_pack_kv")
            if exchange == "ring":
                for t in range(world - 1):
                    ops = [dist.P2POp(dist.isend, share(shares[t]), nxt, group),
                           dist.P2POp(dist.irecv, share(shares[t + 1]), prv, group)]
                    for w in dist.batch_isend_irecv(ops):
                        w.wait()
                    ev = torch.cuda.Event()
                    ev.record(comm)
                    arrived.append(ev)
            else:
                dist.all_gather_into_tensor(kv_all, share(rank), group=group)
                ev = torch.cuda.Event()
                ev.record(comm)
                arrived.append(ev)
        k0 = steps[0]
        k0.q, k0.o, k0.k, k0.v, k0.status = (bufs.base[sq], bufs.base[so], bufs.base[sk],
                                              bufs.base[sv], status)
        R.check(lib.ktir_fmha_f16_part(C.byref(k0), stream), "ktir_fmha_f16_part")
        for ev, dsc in zip(arrived, steps[1:]):
            compute.wait_event(ev)
            dsc.q, dsc.o, dsc.status = bufs.base[sq], bufs.base[so], status
            R.check(lib.ktir_fmha_f16_part(C.byref(dsc), stream), "ktir_fmha_f16_part")

    plan = Plan("attention", [Launch(run, "kv_ring", len(steps) + 1)], [], status_check=True)
    plan.scratch.update(kv_all=kv_all, o_acc=o_acc, ml=ml, comm=comm)
    flops = 4 * bh * seq * seq * d // 2
    plan.info.update(bh=bh, seq=seq, d=d, causal=True, scale=prob["scale"], flops=flops,
                     ring=dict(tiles=tiles_of, kv_tiles=kv_tiles, exchange=exchange,
                               share_bytes=2 * share_rows * row_bytes))
    # this rank reads only its own query tiles and K/V share from the call's
    # tensors (the rest arrives over NVLink): (buffer index, byte ranges)
    ranges = []
    for qt in mine:
        for h in range(bh):
            ranges.append(((h * seq + qt * TILE) * row_bytes, TILE * row_bytes))
    plan.info["upload_ranges"] = {b.index: ranges for b in (prob["q"], prob["k"], prob["v"])}
    return plan
