"""Host logic of the attention K/V ring, on CPU ranks (gloo).

A zigzag attention program is traced on the host; each rank's contiguous
core range gives its query tiles (ring.query_tiles), the staging layout and
the ring order follow (ring.staging_layout, ring.step_shares).  Two and four
gloo ranks then run the ring with NumPy in place of the kernel: each rank
packs its share of K/V, adds the key tiles of one share per step to its
queries while the shares travel rank to rank with send/recv, carries the
online-softmax state (max, sum, O) between steps, and must reproduce whole
causal attention for its query tiles.  With head groups (one ring of cores
per group of heads), each rank's heads give its exchange group
(ring.exchange_group) and the shares travel within that group only.  The
copy exchange's epoch-flag protocol (ring.copy_schedule) is run by 2-4
simulated members under random interleavings of their streams.
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from ktir_cpu_b200 import workloads as W
from ktir_cpu_b200.lower import core_range
from ktir_cpu_b200.ring import (exchange_group, head_tiles, query_tiles, share_mask,
                                 staging_layout, step_shares)

P = dict(batch=1, heads=2, seq=1024, dim=128, grid=8, groups=1)
# two head groups of two heads, each a ring of four cores: on four ranks every
# group's K/V shares pass between two ranks only
PG = dict(batch=1, heads=4, seq=1024, dim=128, grid=8, groups=2)
T = 128


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _spans_per_rank(world, params):
    """(first head, end head, query tiles) of each rank's core range, from the
    traced zigzag program."""
    from ktir_cpu_b200 import KTIRInterpreter
    from ktir_cpu_b200.rewrite import attention_problem, attention_rewrites
    from ktir_cpu_b200.trace import Tracer
    it = KTIRInterpreter(device=torch.device("cpu"))
    it.load(W.source("attention", **params))
    kw = W.inputs("attention", seed=0, **params)
    func, kw, ptrs, scalars, _ = it._bind("causal_attention", kw)
    tr = Tracer(func, it._space(ptrs), scalars, ptrs, rewrites=attention_rewrites(func)).run()
    seq = attention_problem(tr.stores)["seq"]
    out = []
    for r in range(world):
        c0, c1 = core_range(r, world, params["grid"])
        pr = attention_problem([s for s in tr.stores if c0 <= s.core < c1], seq)
        assert query_tiles(pr["rows"], seq, 64) == head_tiles(pr["rows"], seq, 64)[2]
        out.append(head_tiles(pr["rows"], seq, 64))
    return out


def _worker(rank, world, port, spans, params, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        kw = W.inputs("attention", seed=5, **params)
        seq, d = params["seq"], params["dim"]
        bh = params["batch"] * params["heads"]
        n_tiles = seq // T
        scale = float(np.float16(1.0 / np.sqrt(d)))
        members = exchange_group(spans, rank)
        pos, g = members.index(rank), len(members)
        h_lo, h_hi, _ = spans[rank]
        tiles_of = [spans[m][2] for m in members]
        owner, local, kv_tiles = staging_layout(tiles_of, n_tiles)
        qf, kf, vf = (kw[n].astype(np.float64).reshape(bh, seq, d)[h_lo:h_hi]
                      for n in ("q_ptr", "k_ptr", "v_ptr"))
        nh = h_hi - h_lo
        share = np.zeros((g, 2, nh, kv_tiles, T, d))        # the staging buffers (K, V)
        for i, t in enumerate(tiles_of[pos]):
            share[pos, 0, :, i] = kf[:, t * T:(t + 1) * T]
            share[pos, 1, :, i] = vf[:, t * T:(t + 1) * T]
        mine = tiles_of[pos]
        m = np.full((nh, len(mine), T), -np.inf)
        l_ = np.zeros((nh, len(mine), T))
        o = np.zeros((nh, len(mine), T, d))
        shares = step_shares(pos, g)
        nxt, prv = members[(pos + 1) % g], members[(pos - 1) % g]
        for t, s in enumerate(shares):
            mask = share_mask(tiles_of[s])
            for qi, qt in enumerate(mine):
                for kt in range(n_tiles):
                    if not (mask >> kt) & 1 or kt > qt:
                        continue
                    assert owner[kt] == s
                    kb = share[s, 0, :, local[kt]]
                    vb = share[s, 1, :, local[kt]]
                    sc = np.einsum("hqd,hkd->hqk", qf[:, qt * T:(qt + 1) * T], kb) * scale
                    if kt == qt:
                        sc = np.where(np.triu(np.ones((T, T), bool), 1), -np.inf, sc)
                    mn = np.maximum(m[:, qi], sc.max(-1))
                    a = np.exp(m[:, qi] - mn)
                    p = np.exp(sc - mn[..., None])
                    l_[:, qi] = l_[:, qi] * a + p.sum(-1)
                    o[:, qi] = o[:, qi] * a[..., None] + np.einsum("hqk,hkd->hqd", p, vb)
                    m[:, qi] = mn
            if t < g - 1:
                # pass share s on within the group, take share shares[t + 1]
                # from the previous member
                send = torch.from_numpy(share[s].copy())
                recv = torch.empty_like(send)
                reqs = [dist.isend(send, nxt), dist.irecv(recv, prv)]
                for rq in reqs:
                    rq.wait()
                share[shares[t + 1]] = recv.numpy()
        q.put((rank, h_lo, h_hi, mine, o / l_[..., None]))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,params,groups", [(2, P, [[0, 1]] * 2),
                                                 (4, P, [[0, 1, 2, 3]] * 4),
                                                 (4, PG, [[0, 1], [0, 1], [2, 3], [2, 3]])],
                         ids=["ring2", "ring4", "head_groups_4ranks"])
def test_ring_steps_reproduce_whole_attention(world, params, groups):
    spans = _spans_per_rank(world, params)
    assert [exchange_group(spans, r) for r in range(world)] == groups
    n_tiles = params["seq"] // T
    for members in {tuple(g) for g in groups}:
        tiles_of = [spans[m][2] for m in members]
        assert sorted(t for tl in tiles_of for t in tl) == list(range(n_tiles))
        # zigzag: every rank owns the same amount of causal work
        work = {sum(t + 1 for t in tl) for tl in tiles_of}
        assert len(work) == 1, tiles_of
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, spans, params, q))
             for r in range(world)]
    for p in procs:
        p.start()
    try:
        got = [q.get(timeout=120) for _ in range(world)]
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert all(p.exitcode == 0 for p in procs)
    kw = W.inputs("attention", seed=5, **params)
    seq, d = params["seq"], params["dim"]
    bh = params["batch"] * params["heads"]
    qf, kf, vf = (kw[n].astype(np.float64).reshape(bh, seq, d) for n in ("q_ptr", "k_ptr", "v_ptr"))
    s = np.einsum("hqd,hkd->hqk", qf, kf) * float(np.float16(1.0 / np.sqrt(d)))
    s = np.where(np.triu(np.ones((seq, seq), bool), 1), -np.inf, s)
    e = np.exp(s - s.max(-1, keepdims=True))
    want = np.einsum("hqk,hkd->hqd", e / e.sum(-1, keepdims=True), vf)
    covered = np.zeros((bh, seq // T), bool)
    for rank, h_lo, h_hi, mine, o in got:
        for qi, qt in enumerate(mine):
            np.testing.assert_allclose(o[:, qi], want[h_lo:h_hi, qt * T:(qt + 1) * T],
                                       rtol=1e-9, atol=1e-12)
            covered[h_lo:h_hi, qt] = True
    assert covered.all()


def test_exchange_group_rejects_overlapping_head_ranges():
    assert exchange_group([(0, 2, [0]), (0, 2, [1]), (2, 4, [0, 1])], 2) == [2]
    assert exchange_group([(0, 2, [0]), (1, 3, [1])], 0) is None
    assert head_tiles([0, 64, 1024, 1088, 3072, 3136], 1024, 64) is None   # heads 0, 1, 3


def test_staging_layout_rejects_overlaps_and_gaps():
    with pytest.raises(ValueError):
        staging_layout([[0, 3], [1, 3]], 4)
    with pytest.raises(ValueError):
        staging_layout([[0, 3], [1]], 4)
    owner, local, kv = staging_layout([[0, 3], [1, 2]], 4)
    assert owner == [0, 1, 1, 0] and local == [0, 0, 1, 1] and kv == 2
    assert step_shares(1, 4) == [1, 0, 3, 2]
    assert query_tiles([0, 64, 448, 192], 512, 64) is None          # a half tile
    assert query_tiles([0, 64, 512, 576], 512, 64) == [0]           # two heads, tile 0


def _reached(flag: int, value: int) -> bool:
    """The device wait's test: flag has reached value, modulo 2^32."""
    d = (flag - value) & 0xFFFFFFFF
    return d < 0x80000000


@pytest.mark.parametrize("gsize,first", [(2, 1), (3, 1), (4, 1), (2, 0xFFFFFFFE), (3, 0xFFFFFFFD)])
def test_copy_exchange_schedule_never_blocks_and_never_reads_a_share_being_packed(gsize, first):
    """The copy exchange's flag protocol (ring.copy_schedule), run by every
    member of a group over several executions under random interleavings of
    their streams: every wait ends, and every pull of a share reads the
    owner's pack of the same execution, with no later pack of that owner
    between the start and the end of the pull.  Epochs may wrap past 2^32."""
    import random
    from ktir_cpu_b200.ring import copy_schedule
    n_exec = 6
    epochs = [(first + k) & 0xFFFFFFFF for k in range(n_exec)]
    for seed in range(200):
        rng = random.Random(seed)
        prev = (first - 1) & 0xFFFFFFFF
        ready = [prev] * gsize                      # word 0 of each member's buffer
        taken = [[prev] * gsize for _ in range(gsize)]   # taken[owner][reader]
        packed = [None] * gsize                     # the epoch each owner's share holds
        ops = []
        for r in range(gsize):
            seq_r = []
            for e in epochs:
                for op in copy_schedule(r, gsize, e):
                    if op[0] == "copy":
                        # a pull takes time: other streams may move in between
                        seq_r += [("copy_start", op[1], e), ("copy_end", op[1], e)]
                    elif op[0] == "pack":
                        seq_r.append(("pack", e))
                    else:
                        seq_r.append(op)
            ops.append(seq_r)
        pc = [0] * gsize
        pulling = {}                                 # (reader, owner) -> epoch read at start

        def runnable(r):
            if pc[r] >= len(ops[r]):
                return False
            op = ops[r][pc[r]]
            if op[0] == "wait_taken":
                return _reached(taken[r][op[1]], op[2])
            if op[0] == "wait_ready":
                return _reached(ready[op[1]], op[2])
            return True

        while any(pc[r] < len(ops[r]) for r in range(gsize)):
            cand = [r for r in range(gsize) if runnable(r)]
            assert cand, f"seed {seed}: every remaining stream waits ({pc})"
            r = rng.choice(cand)
            op = ops[r][pc[r]]
            pc[r] += 1
            if op[0] == "pack":
                assert all(o != r for (_, o) in pulling), "a share packed while it is pulled"
                packed[r] = op[1]
            elif op[0] == "set_ready":
                ready[r] = op[1]
            elif op[0] == "copy_start":
                pulling[(r, op[1])] = packed[op[1]]
            elif op[0] == "copy_end":
                start = pulling.pop((r, op[1]))
                assert start == op[2] == packed[op[1]], "pulled a share of another execution"
            elif op[0] == "set_taken":
                taken[op[1]][r] = op[2]
