"""Two GPUs: the context-parallel reuse prefill across real ranks.

Skipped unless at least two B200s are visible.  Each rank holds a round-robin
shard of a 1152-token int8 paged prefix and the suffix K/V of its zig-zag
query rows; both gather paths (NCCL all-gather, and the dequantise kernel
reading the peers' symmetric-memory shards over NVLink) must give every rank's
rows the result of the unsharded paged prefill, which each rank can compute
because all shards are generated from one seed.  The peers path orders the
shard writes with ``kvb_peer_barrier``; a barrier one rank skips makes the
other's give up within its limit and report ``KVB_STATUS_PEER_WAIT``.
"""

import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, q):
    from datetime import timedelta
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=timedelta(seconds=60))
    try:
        from kvboost_b200 import context_parallel as cp
        from kvboost_b200.paged import (DeviceBlockAllocator, block_table_tensor,
                                        paged_prefill_attention, quantize_chunk_int8)
        Hq, Hkv, D, C, Sq = 16, 2, 128, 9, 512
        P = C * 128
        g = torch.Generator().manual_seed(31)
        full = DeviceBlockAllocator(1, Hkv, D, C * 8, device=dev)
        chunks = []
        for c in range(C):
            k = torch.randn(1, Hkv, 128, D, generator=g).to(torch.bfloat16).half().to(dev)
            v = torch.randn(1, Hkv, 128, D, generator=g).to(torch.bfloat16).half().to(dev)
            chunks.append(quantize_chunk_int8(k, v))
            full.write_chunk_int8(0, list(range(c * 8, c * 8 + 8)), *chunks[c])
        qf = torch.randn(1, Hq, Sq, D, generator=g).to(torch.bfloat16).to(dev)
        kf = torch.randn(1, Hkv, Sq, D, generator=g).to(torch.bfloat16).to(dev)
        vf = torch.randn(1, Hkv, Sq, D, generator=g).to(torch.bfloat16).to(dev)
        ref, _ = paged_prefill_attention(qf, kf, vf, full, 0,
                                         block_table_tensor([list(range(C * 8))], dev), P)
        rows = torch.cat([torch.arange(s, e) for s, e in cp.zigzag_chunks(Sq, world, rank)]).to(dev)
        ql, kl, vl = (t[:, :, rows].contiguous() for t in (qf, kf, vf))

        shards = cp.PeerShardBuffer(C, world, Hkv, D, Sq, torch.bfloat16, dev, symmetric=True)
        for slot, c in enumerate(cp.local_chunk_slots(C, world, rank)):
            shards.alloc.write_chunk_int8(0, list(range(slot * 8, slot * 8 + 8)), *chunks[c])
        shards.suffix_k.copy_(kl[0])
        shards.suffix_v.copy_(vl[0])
        torch.cuda.synchronize()
        o_peer = cp.cp_reuse_prefill_peers(ql, shards, P, rank)

        local = cp.make_shard_allocator(C, world, Hkv, D, dev)
        for slot, c in enumerate(cp.local_chunk_slots(C, world, rank)):
            local.write_chunk_int8(0, list(range(slot * 8, slot * 8 + 8)), *chunks[c])
        gathered = DeviceBlockAllocator(1, Hkv, D, world * local.num_blocks, device=dev)
        o_nccl = cp.cp_reuse_prefill(ql, kl, vl, local, gathered, P, Sq)
        torch.cuda.synchronize()
        want = ref[:, :, rows]
        from kvboost_b200 import _lib, ops
        status = ops.read_status(dev)            # the peer barrier passed on every rank
        err = torch.tensor([(o_peer.float() - want.float()).abs().max().item(),
                            (o_nccl.float() - want.float()).abs().max().item(), float(status)],
                           device=dev)
        dist.all_reduce(err, op=dist.ReduceOp.MAX)
        # A rank that does not come to a barrier (a failure made on the host, between
        # steps, with nothing of its own in flight): the other rank's barrier kernel
        # gives up after its limit and reports it in the status word.
        missed = 0
        if rank == 0:
            shards.barrier(timeout_ms=100)
            torch.cuda.synchronize()
            missed = ops.read_status(dev) & _lib.KVB_STATUS_PEER_WAIT
        dist.barrier()
        if rank == 0:
            q.put(err.tolist() + [missed])
        dist.barrier()
    except Exception as e:  # report, then let the group time out the peer if it waits
        q.put(repr(e))
        raise
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs two B200s")
def test_context_parallel_two_gpus():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = q.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
    assert isinstance(res, list), res
    assert max(res[:2]) <= 2e-2, res
    assert res[2] == 0, res          # no barrier gave up while both ranks took part
    assert res[3] != 0, res          # the lone rank's barrier reported the missing peer
    assert all(p.exitcode == 0 for p in procs)
