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


def _cp_worker(rank, world, port, q):
    """Context-parallel host logic: gather a chunk-sharded int8 pool and the
    zig-zag suffix K/V over gloo; both must equal the unsharded originals."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from kvboost_b200 import context_parallel as cp
        from kvboost_b200.paged import DeviceBlockAllocator
        H, D, C, Sq = 2, 64, 5, 16                      # 5 chunks of 128 tokens, 16-row suffix
        g = torch.Generator().manual_seed(7)
        pool = torch.randint(-127, 128, (C * 8, 2, H, 16, D), generator=g, dtype=torch.int8)
        ks = torch.rand(C * 8, H, 16, generator=g)
        vs = torch.rand(C * 8, H, D, generator=g)
        local = cp.make_shard_allocator(C, world, H, D, "cpu")
        for slot, c in enumerate(cp.local_chunk_slots(C, world, rank)):
            dst = slice(slot * 8, slot * 8 + 8)
            local.pools[0][dst] = pool[c * 8:c * 8 + 8]
            local.k_scale[0][dst] = ks[c * 8:c * 8 + 8]
            local.v_scale[0][dst] = vs[c * 8:c * 8 + 8]
        full = DeviceBlockAllocator(1, H, D, world * local.num_blocks, device="cpu")
        cp.gather_pool(local, full)
        table = torch.tensor(cp.gathered_block_table(C, world))
        ok_pool = (torch.equal(full.pools[0][table], pool) and torch.equal(full.k_scale[0][table], ks)
                   and torch.equal(full.v_scale[0][table], vs))
        kfull = torch.randn(1, H, Sq, D, generator=g)
        vfull = torch.randn(1, H, Sq, D, generator=g)
        rows = torch.cat([torch.arange(s, e) for s, e in cp.zigzag_chunks(Sq, world, rank)])
        k2, v2 = cp.gather_suffix_kv(kfull[:, :, rows], vfull[:, :, rows], Sq)
        ok_kv = torch.equal(k2, kfull) and torch.equal(v2, vfull)
        flags = torch.tensor([int(ok_pool), int(ok_kv)])
        dist.all_reduce(flags, op=dist.ReduceOp.MIN)
        if rank == 0:
            q.put(flags.tolist())
    finally:
        dist.destroy_process_group()


@pytest.mark.slow
def test_context_parallel_gathers_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_cp_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    flags = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert flags == [1, 1]


def test_zigzag_chunks_cover_and_balance():
    from kvboost_b200 import context_parallel as cp
    for world in (1, 2, 4, 8):
        q_len = 2048
        spans = [sp for r in range(world) for sp in cp.zigzag_chunks(q_len, world, r)]
        covered = sorted(i for s, e in spans for i in range(s, e))
        assert covered == list(range(q_len))
        # causal work of rank r ~ sum of its rows' key counts: equal across ranks
        work = [sum(e * (e + 1) // 2 - s * (s + 1) // 2 for s, e in cp.zigzag_chunks(q_len, world, r))
                for r in range(world)]
        assert max(work) == min(work)
        idx = cp.zigzag_token_index(q_len, world)
        assert sorted(idx.tolist()) == list(range(q_len))


def test_lpt_partition_covers_and_balances():
    from kvboost_b200.sharding import lpt_partition, request_cost
    import bench
    w = bench.make_workload("varlen_d96")
    costs = [request_cost(a, b, w.Hq, w.Hkv, w.D) for a, b in zip(w.sq, w.skv)]
    for world in (1, 2, 4, 8):
        parts = lpt_partition(costs, world)
        assert sorted(i for p in parts for i in p) == list(range(len(costs)))
        loads = [sum(costs[i] for i in p) for p in parts]
        # longest-first placement: the slowest rank within 4/3 of the average share,
        # or held up by one request alone
        assert max(loads) <= max(sum(costs) / world * 4 / 3, max(costs)) + 1e-12
    assert lpt_partition([3.0, 1.0, 2.0], 2) == [[0], [1, 2]]
    assert lpt_partition([1.0, 1.0], 4) == [[0], [1], [], []]


def _varlen_shard_rank(rank, world, out):
    import bench
    w = bench.make_workload("varlen_d96")
    total = w.flops()
    w.shard(rank, world)
    out[rank] = (w.sq, w.skv, w.flops(), w.work(), total, w.scaling, w.tokens())


def test_varlen_shards_agree_across_ranks():
    """Each rank derives its share on its own; together they are the batch."""
    import bench
    full = bench.make_workload("varlen_d96")
    out = {}
    for r in range(4):
        _varlen_shard_rank(r, 4, out)
    pairs = sorted((a, b) for r in range(4) for a, b in zip(out[r][0], out[r][1]))
    assert pairs == sorted(zip(full.sq, full.skv))
    assert abs(sum(out[r][2] for r in range(4)) - full.flops()) < 1e-3 * full.flops()
    for r in range(4):
        assert abs(out[r][3] * 4 - full.flops()) < 1e-6 * full.flops()
        assert out[r][5] == "strong" and out[r][6] == sum(full.sq)
