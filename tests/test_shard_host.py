"""Host logic of splitting one call's core grid across GPUs, on CPU ranks (gloo).

The sharded gather -> +1 -> scatter plan gives each rank a contiguous chunk
of table rows (lower.row_shard); the rank counts, for each of its rows, how
many units (of every core) name the row, and applies f that many times to
its rows.  No counts cross ranks: every rank reads the whole index tensor.
Here gloo ranks run that decomposition with NumPy in place of the two
kernels, the whole table assembled from the ranks' row chunks, and must
reproduce the oracle's sequential, unit-by-unit result exactly.
"""

import os
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from ktir_cpu_b200 import workloads as W
from ktir_cpu_b200.lower import core_range, row_shard

P = dict(rows=96, cols=8, n_idx=512, grid=4, chunk=32)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        kw = W.inputs("gather_add", seed=21, **P)
        table, idx = kw["table_ptr"], kw["idx_ptr"]
        r0, r1, _ = row_shard(rank, world, P["rows"])
        counts = np.zeros(P["rows"], np.int64)
        # every unit of every core, only the rows this rank owns
        for s in range(0, P["n_idx"], P["chunk"]):
            for r in np.unique(idx[s:s + P["chunk"]]):
                if r0 <= r < r1:
                    counts[int(r)] += 1
        assert not counts[:r0].any() and not counts[r1:].any()
        mine = table[r0:r1].copy()
        for i in range(r1 - r0):
            for _ in range(int(counts[r0 + i])):
                mine[i] = (mine[i] + np.float16(1.0)).astype(np.float16)
        parts = [None] * world
        dist.all_gather_object(parts, (r0, mine))
        if rank == 0:
            out = np.empty_like(table)
            for a, block in parts:
                out[a:a + len(block)] = block
            q.put(out)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_sharded_gather_rmw_matches_sequential_semantics(world):
    from oracle.interp import OracleInterpreter
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    ora = OracleInterpreter()
    ora.load(W.source("gather_add", **P))
    want = ora.execute_function("gather_add", **W.inputs("gather_add", seed=21, **P))["table_ptr"]
    assert np.array_equal(got, want)


def test_row_shards_partition_the_table():
    for n in (1, 7, 96, 1 << 20):
        for world in (1, 2, 3, 8):
            spans = [row_shard(r, world, n) for r in range(world)]
            chunk = spans[0][2]
            assert chunk * world >= n and all(c == chunk for _, _, c in spans)
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(spans[i][1] == spans[i + 1][0] for i in range(world - 1))
            assert all(a == min(n, r * chunk) for r, (a, _, _) in enumerate(spans))


def test_core_ranges_partition_the_grid():
    for n in (1, 7, 32, 64):
        for world in (1, 2, 3, 8):
            spans = [core_range(r, world, n) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(spans[i][1] == spans[i + 1][0] for i in range(world - 1))
