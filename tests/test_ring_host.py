"""Host logic of the attention K/V ring, on CPU ranks (gloo).

A zigzag attention program is traced on the host; each rank's contiguous
core range gives its query tiles (ring.query_tiles), the staging layout and
the ring order follow (ring.staging_layout, ring.step_shares).  Two and four
gloo ranks then run the ring with NumPy in place of the kernel: each rank
packs its share of K/V, adds the key tiles of one share per step to its
queries while the shares travel rank to rank with send/recv, carries the
online-softmax state (max, sum, O) between steps, and must reproduce whole
causal attention for its query tiles.
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
from ktir_cpu_b200.ring import query_tiles, share_mask, staging_layout, step_shares

P = dict(batch=1, heads=2, seq=1024, dim=128, grid=8)
T = 128


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _tiles_per_rank(world):
    """Query tiles of each rank's core range, from the traced zigzag program."""
    from ktir_cpu_b200 import KTIRInterpreter
    from ktir_cpu_b200.rewrite import attention_problem, attention_rewrites
    from ktir_cpu_b200.trace import Tracer
    it = KTIRInterpreter(device=torch.device("cpu"))
    it.load(W.source("attention", **P))
    kw = W.inputs("attention", seed=0, **P)
    func, kw, ptrs, scalars, _ = it._bind("causal_attention", kw)
    tr = Tracer(func, it._space(ptrs), scalars, ptrs, rewrites=attention_rewrites(func)).run()
    seq = attention_problem(tr.stores)["seq"]
    out = []
    for r in range(world):
        c0, c1 = core_range(r, world, P["grid"])
        pr = attention_problem([s for s in tr.stores if c0 <= s.core < c1], seq)
        out.append(query_tiles(pr["rows"], seq, 64))
    return out


def _worker(rank, world, port, tiles_of, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        kw = W.inputs("attention", seed=5, **P)
        seq, d = P["seq"], P["dim"]
        bh = P["batch"] * P["heads"]
        n_tiles = seq // T
        scale = float(np.float16(1.0 / np.sqrt(d)))
        owner, local, kv_tiles = staging_layout(tiles_of, n_tiles)
        qf, kf, vf = (kw[n].astype(np.float64).reshape(bh, seq, d) for n in ("q_ptr", "k_ptr", "v_ptr"))
        share = np.zeros((world, 2, bh, kv_tiles, T, d))       # the staging buffers (K, V)
        for i, t in enumerate(tiles_of[rank]):
            share[rank, 0, :, i] = kf[:, t * T:(t + 1) * T]
            share[rank, 1, :, i] = vf[:, t * T:(t + 1) * T]
        mine = tiles_of[rank]
        m = np.full((bh, len(mine), T), -np.inf)
        l_ = np.zeros((bh, len(mine), T))
        o = np.zeros((bh, len(mine), T, d))
        shares = step_shares(rank, world)
        nxt, prv = (rank + 1) % world, (rank - 1) % world
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
            if t < world - 1:
                # pass share s on, take share shares[t + 1] from the previous rank
                send = torch.from_numpy(share[s].copy())
                recv = torch.empty_like(send)
                reqs = [dist.isend(send, nxt), dist.irecv(recv, prv)]
                for rq in reqs:
                    rq.wait()
                share[shares[t + 1]] = recv.numpy()
        q.put((rank, mine, o / l_[..., None]))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_ring_steps_reproduce_whole_attention(world):
    tiles_of = _tiles_per_rank(world)
    n_tiles = P["seq"] // T
    assert sorted(t for tl in tiles_of for t in tl) == list(range(n_tiles))
    # zigzag: every rank owns the same amount of causal work
    work = {sum(t + 1 for t in tl) for tl in tiles_of}
    assert len(work) == 1, tiles_of
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, tiles_of, q)) for r in range(world)]
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
    kw = W.inputs("attention", seed=5, **P)
    seq, d = P["seq"], P["dim"]
    bh = P["batch"] * P["heads"]
    qf, kf, vf = (kw[n].astype(np.float64).reshape(bh, seq, d) for n in ("q_ptr", "k_ptr", "v_ptr"))
    s = np.einsum("hqd,hkd->hqk", qf, kf) * float(np.float16(1.0 / np.sqrt(d)))
    s = np.where(np.triu(np.ones((seq, seq), bool), 1), -np.inf, s)
    e = np.exp(s - s.max(-1, keepdims=True))
    want = np.einsum("hqk,hkd->hqd", e / e.sum(-1, keepdims=True), vf)
    for rank, mine, o in got:
        for qi, qt in enumerate(mine):
            np.testing.assert_allclose(o[:, qi], want[:, qt * T:(qt + 1) * T], rtol=1e-9, atol=1e-12)


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
