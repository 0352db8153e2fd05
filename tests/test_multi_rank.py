"""Multi-rank host logic on CPU (gloo, world size 2).

The prefill path shards without a data-path collective: independent
batches per rank (weak scaling) or disjoint KV-head groups of one long
prefill (strong scaling).  These tests check, on two gloo ranks, that the
head split covers every KV head exactly once and that the reported time is
the max over ranks, as bench.py computes it.
"""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import bench
        w = bench.make_workload("paged_long")
        hk, hq = w.local_heads(rank, world)
        heads = torch.arange(rank * hk, (rank + 1) * hk)
        gathered = [torch.zeros(hk, dtype=torch.long) for _ in range(world)]
        dist.all_gather(gathered, heads)
        elapsed = torch.tensor([10.0 + rank], dtype=torch.float64)   # rank 1 is the slow one
        dist.all_reduce(elapsed, op=dist.ReduceOp.MAX)
        if rank == 0:
            q.put((torch.cat(gathered).tolist(), hq, float(elapsed)))
    finally:
        dist.destroy_process_group()


@pytest.mark.slow
def test_head_split_and_max_time_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    heads, hq, elapsed = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert sorted(heads) == list(range(8))   # every KV head on exactly one rank
    assert hq == 32                          # 4 KV heads x GQA 8 per rank
    assert elapsed == 11.0                   # time is the max over ranks


def test_head_split_rejects_non_divisor():
    import bench
    w = bench.make_workload("paged_long")
    with pytest.raises(SystemExit):
        w.local_heads(0, 3)
