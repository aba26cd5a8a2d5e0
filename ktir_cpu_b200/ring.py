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

When the program's cores form one ring per group of heads (the zigzag layout
with head groups), a GPU's cores serve one range of heads, and the GPUs that
serve the same heads form its exchange group: shares travel within each
group only (each group's ring indexed by the members' places in it), and
the groups exchange side by side.  The whole-sequence case above is one
group of every GPU.

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


def head_tiles(rows: Sequence[int], seq: int, bq: int) -> Optional[Tuple[int, int, List[int]]]:
    """(first head, end head, query tiles) when a set of query-block row
    offsets covers one contiguous range of heads, every head the same whole
    128-row tiles; else None."""
    tiles = query_tiles(rows, seq, bq)
    if tiles is None:
        return None
    heads = sorted({r // seq for r in rows})
    if heads != list(range(heads[0], heads[-1] + 1)):
        return None
    return heads[0], heads[-1] + 1, tiles


def exchange_group(spans: Sequence[Tuple[int, int, Sequence[int]]], rank: int) -> Optional[List[int]]:
    """The ranks whose query tiles share `rank`'s heads (its exchange group,
    in rank order), given every rank's (first head, end head, tiles).  Each
    rank needs the K/V rows of its own heads only, so K/V shares pass among
    the ranks of one group and never between groups.  None unless the ranks'
    head ranges are equal or disjoint."""
    lo, hi, _ = spans[rank]
    members = []
    for r, (l2, h2, _) in enumerate(spans):
        if (l2, h2) == (lo, hi):
            members.append(r)
        elif l2 < hi and lo < h2:
            return None                   # overlapping, unequal head ranges
    return members


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


def copy_schedule(pos: int, gsize: int, epoch: int) -> List[Tuple]:
    """The stream operations of one execution's copy exchange on the GPU at
    place `pos` of a group of `gsize`, in issue order (epochs count from 1,
    modulo 2^32):

      ("wait_taken", i, e - 1)  until member i has copied this GPU's share of
                                the previous execution (a flag in this GPU's
                                staging buffer, word 1 + i)
      ("pack",)                 this GPU's share into its staging buffer
      ("set_ready", e)          this GPU's "packed" flag (word 0)
      ("wait_ready", i, e)      until member i has packed its share
      ("copy", i)               member i's share into this GPU's buffer
      ("set_taken", i, e)       "copied" in member i's buffer (word 1 + pos)

    Other members are visited in ring order from this GPU."""
    e = epoch & 0xFFFFFFFF
    order = [(pos + t) % gsize for t in range(1, gsize)]
    ops: List[Tuple] = [("wait_taken", i, (e - 1) & 0xFFFFFFFF) for i in order]
    ops += [("pack",), ("set_ready", e)]
    for i in order:
        ops += [("wait_ready", i, e), ("copy", i), ("set_taken", i, e)]
    return ops


EXCHANGES = ("copy_overlap", "copy", "gather", "allgather", "ring")

# staging buffer of the copy exchanges: a 256-byte block of epoch flags (word 0:
# the epoch whose share this GPU has packed; word 1 + i: the epoch whose share
# member i of the group has copied out), then the shares
FLAG_BYTES = 256
FLAG_SPIN_LIMIT = 1 << 25          # polls of a flag wait (a short sleep each)


class PeerStaging:
    """This GPU's staging buffer (flags, then every member's K/V share),
    exported as a CUDA IPC handle, and the staging buffers of the other
    members of its exchange group mapped into this process.  Built by every
    rank of the process group at the same time (the handles travel in one
    all_gather_object)."""

    def __init__(self, lib, nbytes: int, members: Sequence[int], pos: int, group):
        import ctypes as C

        import torch.distributed as dist

        from . import runtime as R
        self.lib = lib
        self.base = None
        self.peer: Dict[int, int] = {}
        ptr = C.c_void_p()
        handle = (C.c_char * 64)()
        R.check(lib.ktir_ipc_alloc(FLAG_BYTES + nbytes, C.byref(ptr), handle), "ktir_ipc_alloc")
        self.base = ptr.value
        n = dist.get_world_size(group)
        handles = [None] * n
        dist.all_gather_object(handles, bytes(handle), group=group)
        for i, m in enumerate(members):
            if i != pos:
                p = C.c_void_p()
                R.check(lib.ktir_ipc_open(C.c_char_p(handles[m]), C.byref(p)), "ktir_ipc_open")
                self.peer[i] = p.value

    def close(self) -> None:
        import ctypes as C
        for p in self.peer.values():
            self.lib.ktir_ipc_close(C.c_void_p(p))
        self.peer = {}
        if self.base is not None:
            self.lib.ktir_ipc_free(C.c_void_p(self.base))
            self.base = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def ring_attention_plan(low, prob, exchange: str = "gather"):
    """Device plan for one rank (see the module docstring).

    exchange "copy_overlap" (the default on GPUs): step 0 adds the rank's own
    key tiles straight from the call's K and V while a high-priority comm
    stream packs the rank's share into its staging buffer, which the other
    members of its group have mapped (PeerStaging), flags it packed, and
    pulls every other member's share with the copy engines once that
    member's flag shows it packed (then flags the copy done in the member's
    buffer, so the member may pack over it next time); step 1 adds the
    other shares, the softmax state carried between the steps.  "copy": the
    same exchange, then one kernel over every key tile.  The NCCL forms:
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
    nx, ny, nz = low.trace.grid
    spans = []
    for r in range(world):
        c0, c1 = core_range(r, world, nx * ny * nz)
        pr = attention_problem([s for s in low.all_stores if c0 <= s.core < c1], seq)
        if pr is None or pr["q"] is not prob["q"] or pr["k"] is not prob["k"]:
            return None
        sp = head_tiles(pr["rows"], seq, bq)
        if sp is None:
            return None
        spans.append(sp)
    members = exchange_group(spans, rank)
    if members is None or len(members) < 2:
        return None
    # this rank's heads [h_lo, h_hi); its group's shares are indexed by the
    # members' places in the group
    h_lo, h_hi, _ = spans[rank]
    bh = h_hi - h_lo
    hoff = h_lo * seq * d * 2             # byte offset of head h_lo in Q, K, V, O
    tiles_of = [spans[m][2] for m in members]
    gsize, pos = len(members), members.index(rank)
    try:
        owner, local, kv_tiles = staging_layout(tiles_of, n_tiles)
    except ValueError:
        return None
    if len({len(t) for t in tiles_of}) != 1:
        return None                       # equal shares: NCCL all-gather and same-size sends
    mine = tiles_of[pos]
    dev = low.device
    share_rows = bh * kv_tiles * TILE
    row_bytes = d * 2
    share_bytes = 2 * share_rows * row_bytes
    if exchange not in EXCHANGES:
        raise ValueError(f"K/V exchange {exchange!r}: expected one of {EXCHANGES}")
    copies = exchange in ("copy", "copy_overlap")
    sizes = [len(exchange_group(spans, r) or ()) for r in range(world)]
    if copies and (dev.type != "cuda" or min(sizes) < 2 or max(sizes) > FLAG_BYTES // 4 - 1):
        # peer mappings need GPUs, every rank of the process group must take
        # part in the handle exchange, and the flag block holds one "copied"
        # word per member: plain NCCL otherwise
        exchange, copies = ("gather", False)
    lib = R.load_library()
    staging = kv_all = None
    if copies:
        staging = PeerStaging(lib, gsize * share_bytes, members, pos, group)
        kv_base = staging.base + FLAG_BYTES
    else:
        kv_all = torch.empty(gsize * 2 * share_rows * d, dtype=torch.float16, device=dev)
        kv_base = kv_all.data_ptr()
    # the overlapped forms carry the softmax state between their steps
    o_acc = ml = None
    if exchange not in ("gather", "copy"):
        o_acc = torch.empty(bh * len(mine) * TILE * d, dtype=torch.float32, device=dev)
        ml = torch.empty(bh * len(mine) * TILE * 2, dtype=torch.float32, device=dev)
    sq, sk, sv, so = (low.slots[b.index] for b in (prob["q"], prob["k"], prob["v"], prob["o"]))
    # high priority: the packing and NCCL kernels take their SMs ahead of the
    # attention kernel's CTAs, which would otherwise fill every SM first
    comm = (torch.cuda.Stream(dev, priority=-1)
            if dev.type == "cuda" and exchange not in ("gather", "copy") else None)
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
            dsc.kv_tiles, dsc.kv_rows = kv_tiles, (2 * gsize - 1) * share_rows
            dsc.k = kv_base
            dsc.v = kv_base + share_rows * row_bytes
            for kt in range(n_tiles):
                dsc.kv_owner[kt], dsc.kv_local[kt] = 2 * owner[kt], local[kt]
        else:
            # the call's own K / V: tile kt of head h at row h * seq + kt * 128
            dsc.kv_tiles, dsc.kv_rows = n_tiles, bh * seq
            for kt in range(n_tiles):
                dsc.kv_owner[kt], dsc.kv_local[kt] = 0, kt
        return dsc

    shares = step_shares(pos, gsize)
    if exchange in ("gather", "copy"):
        steps = [desc(all_mask, True, True, True)]
    elif exchange == "ring":
        steps = [desc(own_mask, True, False, False)] + \
            [desc(share_mask(tiles_of[s]), False, t == gsize - 1, True)
             for t, s in enumerate(shares) if t > 0]
    else:
        steps = [desc(own_mask, True, False, False), desc(all_mask & ~own_mask, False, True, True)]

    def global_rank(r):
        return r if group is None else dist.get_global_rank(group, r)
    peers = [global_rank(m) for m in members]
    nxt, prv = peers[(pos + 1) % gsize], peers[(pos - 1) % gsize]
    whole_group = gsize == world

    def share(s):
        return kv_all[s * 2 * share_rows * d:(s + 1) * 2 * share_rows * d]

    epoch = [0]

    def pull_shares(bufs, st, status):
        """The copy exchange of one execution on stream `st`: wait until every
        member has copied this GPU's previous share, pack the share, flag it
        packed, and for each other member (in ring order from this GPU) wait
        for its share, pull it with the copy engines and flag it copied."""
        e = epoch[0] = (epoch[0] + 1) & 0xFFFFFFFF
        flags = staging.base
        stp = C.c_void_p(status)

        def wait(addr, value):
            R.check(lib.ktir_flag_wait(C.c_void_p(addr), 1, 1, value, FLAG_SPIN_LIMIT, stp, st),
                    "ktir_flag_wait")
        for op in copy_schedule(pos, gsize, e):
            kind = op[0]
            if kind == "wait_taken":
                wait(flags + 4 * (1 + op[1]), op[2])
            elif kind == "pack":
                R.check(lib.ktir_pack_kv(C.c_void_p(kv_base + pos * share_bytes),
                                         C.c_void_p(bufs.base[sk] + hoff),
                                         C.c_void_p(bufs.base[sv] + hoff),
                                         bh, seq, d, own_mask, st), "ktir_pack_kv")
            elif kind == "set_ready":
                R.check(lib.ktir_flag_set(C.c_void_p(flags), op[1], st), "ktir_flag_set")
            elif kind == "wait_ready":
                wait(staging.peer[op[1]], op[2])
            elif kind == "copy":
                i = op[1]
                R.check(lib.ktir_copy_async(C.c_void_p(kv_base + i * share_bytes),
                                            C.c_void_p(staging.peer[i] + FLAG_BYTES + i * share_bytes),
                                            share_bytes, st), "ktir_copy_async")
            else:                                   # set_taken
                R.check(lib.ktir_flag_set(C.c_void_p(staging.peer[op[1]] + 4 * (1 + pos)), op[2],
                                          st), "ktir_flag_set")

    def gather_shares():
        """Every member's share into its place of kv_all: one all-gather when
        the group is the whole process group, else send/recv with each other
        member (the groups' exchanges run side by side)."""
        if whole_group:
            dist.all_gather_into_tensor(kv_all, share(pos), group=group)
            return
        ops = []
        for i, p in enumerate(peers):
            if i != pos:
                ops += [dist.P2POp(dist.isend, share(pos), p, group),
                        dist.P2POp(dist.irecv, share(i), p, group)]
        for w in dist.batch_isend_irecv(ops):
            w.wait()

    def run(bufs, stream, status):
        compute = (torch.cuda.ExternalStream(stream.value, device=dev) if stream.value
                   else torch.cuda.default_stream(dev))
        if exchange == "copy":
            pull_shares(bufs, stream, status)
            k0 = steps[0]
            k0.q, k0.o, k0.status = bufs.base[sq] + hoff, bufs.base[so] + hoff, status
            R.check(lib.ktir_fmha_f16_part(C.byref(k0), stream), "ktir_fmha_f16_part")
            return
        if exchange == "gather":
            with torch.cuda.stream(compute):
                R.check(lib.ktir_pack_kv(C.c_void_p(share(pos).data_ptr()),
                                         C.c_void_p(bufs.base[sk] + hoff),
                                         C.c_void_p(bufs.base[sv] + hoff),
                                         bh, seq, d, own_mask, stream), "ktir_pack_kv")
                # the compute stream waits for the exchange before the kernel
                gather_shares()
            k0 = steps[0]
            k0.q, k0.o, k0.status = bufs.base[sq] + hoff, bufs.base[so] + hoff, status
            R.check(lib.ktir_fmha_f16_part(C.byref(k0), stream), "ktir_fmha_f16_part")
            return
        # the comm stream starts after the previous execution's kernels, which
        # read the staging buffer it overwrites; its work is queued before the
        # first attention step so that it reaches the SMs first
        comm.wait_stream(compute)
        arrived = []
        with torch.cuda.stream(comm):
            cs = C.c_void_p(comm.cuda_stream)
            if copies:
                pull_shares(bufs, cs, status)
            else:
                R.check(lib.ktir_pack_kv(C.c_void_p(share(pos).data_ptr()),
                                         C.c_void_p(bufs.base[sk] + hoff),
                                         C.c_void_p(bufs.base[sv] + hoff), bh, seq, d, own_mask,
                                         cs), "ktir_pack_kv")
            if exchange == "ring":
                for t in range(gsize - 1):
                    ops = [dist.P2POp(dist.isend, share(shares[t]), nxt, group),
                           dist.P2POp(dist.irecv, share(shares[t + 1]), prv, group)]
                    for w in dist.batch_isend_irecv(ops):
                        w.wait()
                    ev = torch.cuda.Event()
                    ev.record(comm)
                    arrived.append(ev)
            else:
                if not copies:
                    gather_shares()
                ev = torch.cuda.Event()
                ev.record(comm)
                arrived.append(ev)
        k0 = steps[0]
        k0.q, k0.o, k0.k, k0.v, k0.status = (bufs.base[sq] + hoff, bufs.base[so] + hoff,
                                              bufs.base[sk] + hoff, bufs.base[sv] + hoff, status)
        R.check(lib.ktir_fmha_f16_part(C.byref(k0), stream), "ktir_fmha_f16_part")
        for ev, dsc in zip(arrived, steps[1:]):
            compute.wait_event(ev)
            dsc.q, dsc.o, dsc.status = bufs.base[sq] + hoff, bufs.base[so] + hoff, status
            R.check(lib.ktir_fmha_f16_part(C.byref(dsc), stream), "ktir_fmha_f16_part")

    plan = Plan("attention", [Launch(run, "kv_ring", len(steps) + 1)], [], status_check=True)
    plan.scratch.update(kv_all=kv_all, staging=staging, o_acc=o_acc, ml=ml, comm=comm)
    flops = 4 * bh * seq * seq * d // 2
    plan.info.update(bh=bh, seq=seq, d=d, causal=True, scale=prob["scale"], flops=flops,
                     ring=dict(tiles=tiles_of, kv_tiles=kv_tiles, exchange=exchange,
                               heads=(h_lo, h_hi), group=members, share_bytes=share_bytes))
    # this rank reads only its own query tiles and K/V share from the call's
    # tensors (the rest arrives over NVLink): (buffer index, byte ranges)
    ranges = []
    for qt in mine:
        for h in range(h_lo, h_hi):
            ranges.append(((h * seq + qt * TILE) * row_bytes, TILE * row_bytes))
    plan.info["upload_ranges"] = {b.index: ranges for b in (prob["q"], prob["k"], prob["v"])}
    return plan
