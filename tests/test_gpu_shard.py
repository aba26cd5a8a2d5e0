"""One call's core grid split across two or four GPUs (one process per GPU, NCCL),
against the oracle.  Each rank executes its contiguous range of cores and
the ranks combine their writes, so every rank returns the whole result,
which must equal the single-GPU (oracle) result.  The attention cases cover
cores that own whole heads (no exchange) and cores that own zigzag stretches
of every head's sequence (K/V shares passed between the GPUs: gathered before
one attention kernel, or passed while the first step runs, by all-gather or
by send/recv, or pulled from the other GPUs' mapped staging buffers by the
copy engines, KTIR_KV_EXCHANGE), and cores in rings per group of heads (on two
GPUs each GPU owns whole groups; on four, the two GPUs of a group exchange).
Skipped with fewer GPUs than a case splits over."""

import os
import socket
from datetime import timedelta

import pytest

from golden_util import assert_contraction, assert_matches, contraction_mag
from ktir_cpu_b200 import workloads as W

pytestmark = pytest.mark.gpu

_ATT = dict(batch=1, heads=4, seq=512, dim=128, grid=4, groups=1)
# two head groups, each a ring of four cores: on four GPUs each group's K/V
# shares pass between the two GPUs that serve it
_ATTG = dict(batch=1, heads=4, seq=512, dim=128, grid=8, groups=2)
CASES = [("softmax", dict(rows=256, cols=1024, grid=8, chunk=32), 1e-2, None, 2),
         ("gather_add", dict(rows=4096, cols=128, n_idx=16384, grid=8, chunk=1024), None, None, 2),
         ("gemm", dict(m=512, n=512, k=512, grid=(4, 2)), 1e-2, None, 2),
         ("attention", dict(_ATT, layout="heads"), 1e-2, None, 2),
         ("attention", _ATT, 1e-2, "gather", 2),
         ("attention", _ATT, 1e-2, "allgather", 2),
         ("attention", _ATT, 1e-2, "ring", 2),
         ("attention", _ATT, 1e-2, "copy", 2),
         ("attention", _ATT, 1e-2, "copy_overlap", 2),
         ("attention", _ATTG, 1e-2, None, 2),
         ("attention", _ATTG, 1e-2, "gather", 4),
         ("attention", _ATTG, 1e-2, "ring", 4),
         ("attention", _ATTG, 1e-2, "copy_overlap", 4)]
IDS = ["softmax", "gather_add", "gemm", "attention_heads", "attention_ring_gather",
       "attention_ring_allgather", "attention_ring_sendrecv", "attention_peer_copy",
       "attention_peer_copy_overlap", "attention_head_groups_2gpu",
       "attention_head_groups_4gpu_gather", "attention_head_groups_4gpu_sendrecv",
       "attention_head_groups_4gpu_peer_copy"]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, name, p, exchange, q):
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    if exchange:
        os.environ["KTIR_KV_EXCHANGE"] = exchange
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=timedelta(seconds=60))
    try:
        from ktir_cpu_b200 import KTIRInterpreter
        interp = KTIRInterpreter(device=dev, shard=(rank, world, None))
        interp.load(W.source(name, **p))
        kw = W.inputs(name, seed=3, **p)
        # twice: the second call reuses the plan, its staging buffers and
        # (with the peer copies) the epoch flags the first call left
        for _ in range(2):
            out = interp.execute_function(W.FUNC[name], **{k: v.copy() for k, v in kw.items()})
        torch.cuda.synchronize(dev)
        plan = interp.last_executable.plan
        q.put((rank, plan.kind, [l.kind for l in plan.launches], out))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("name,p,tol,exchange,world", CASES, ids=IDS)
def test_gpu_shards_merge_to_oracle(name, p, tol, exchange, world):
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    from oracle.interp import OracleInterpreter
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, name, p, exchange, q))
             for r in range(world)]
    for pr in procs:
        pr.start()
    try:
        got = [q.get(timeout=300) for _ in range(world)]
    finally:
        for pr in procs:
            pr.join(timeout=60)
            if pr.is_alive():
                pr.kill()
    assert all(pr.exitcode == 0 for pr in procs)
    kw = W.inputs(name, seed=3, **p)
    ora = OracleInterpreter()
    ora.load(W.source(name, **p))
    want = ora.execute_function(W.FUNC[name], **{k: v.copy() for k, v in kw.items()})
    kinds = {kind for _, kind, _, _ in got}
    assert len(kinds) == 1 and kinds != {"generic"}, kinds
    if exchange is not None:
        assert all(launches == ["kv_ring"] for _, _, launches, _ in got)
    elif name == "attention":
        # cores of each GPU own whole heads: no exchange
        assert all(launches == ["fmha"] for _, _, launches, _ in got)
    mags = contraction_mag(f"{name}_seq{p.get('seq', 0)}", kw) or {}
    for rank, _, _, out in got:
        for k, w in want.items():
            if k in mags:
                assert_contraction(f"rank {rank} {name}:{k}", out[k], w, mags[k], tol)
            else:
                assert_matches(f"rank {rank} {name}:{k}", out[k], w, tol)
