"""GPU parity of the int8 paged reuse prefill (KIVI int8 prefix in 16-token blocks).

The cached prefix is KIVI-int8 quantised per 128-token chunk, stored in
16-token blocks of a device pool at a seeded random permutation of block ids,
and attended to together with the suffix's own fresh K/V.  The oracle is the
reference's host path restated: dequantise (``float16(q * scale)``), gather by
the block table, cast to the compute dtype, concatenate, bottom-right causal
attention.  Tolerances: max-abs 2e-2 (bf16), 1e-2 (fp16), LSE 2e-3.
"""

import math

import numpy as np
import pytest
import torch

from oracle import attention as oattn
from oracle import kv_quant as oq
from oracle import paged as opaged

pytestmark = pytest.mark.gpu
TOL = {torch.bfloat16: 2e-2, torch.float16: 1e-2}


@pytest.fixture(autouse=True)
def _gpu():
    if not torch.cuda.is_available() or torch.cuda.get_device_capability()[0] != 10:
        pytest.skip("needs an sm_100 (B200) device")
    from kvboost_b200 import ops
    ops.read_status(torch.device("cuda"))
    yield


def test_gpu_quantiser_matches_reference_bit_exact():
    """quantize_chunk_int8 on the GPU == the reference's _quantize_int8 (kv_quantize.py:73-100)."""
    from kvboost_b200.paged import quantize_chunk_int8
    g = torch.Generator().manual_seed(3)
    for H, L, D in ((2, 128, 128), (8, 128, 64), (1, 100, 96)):
        k = torch.randn(1, H, L, D, generator=g).to(torch.bfloat16).to(torch.float16)
        v = (torch.randn(1, H, L, D, generator=g) * 3).to(torch.float16)
        kq, ks, vq, vs = quantize_chunk_int8(k.cuda(), v.cuda())
        rk, rks, rv, rvs = oq.quantize_int8(k.numpy(), v.numpy())
        assert np.array_equal(kq.cpu().numpy(), rk) and np.array_equal(vq.cpu().numpy(), rv)
        assert np.array_equal(ks.cpu().numpy().view(np.uint16), rks.view(np.uint16))
        assert np.array_equal(vs.cpu().numpy().view(np.uint16), rvs.view(np.uint16))


def _oracle_prefix(alloc, tbl, P):
    pool = alloc.pools[0].cpu().numpy()
    ks = alloc.k_scale16[0].cpu().numpy()
    vs = alloc.v_scale16[0].cpu().numpy()
    return opaged.dequant_gather(pool, ks, vs, tbl, P, 16)   # float16 [H, P, D]


def _run_case(B, Hq, Hkv, D, chunk_sets, Sq, dtype, seed, num_blocks=512, rows=None,
              fused_only=False, heads=None):
    from kvboost_b200.paged import (DeviceBlockAllocator, block_table_tensor,
                                    paged_prefill_attention, quantize_chunk_int8)
    g = torch.Generator().manual_seed(seed + 1)
    # one pool shared by the batch, chunks stored at a seeded permutation of block ids
    total = sum((L + 15) // 16 for cs in chunk_sets for L in cs)
    assert total <= num_blocks
    perm = torch.randperm(num_blocks, generator=g).tolist()
    alloc = DeviceBlockAllocator(1, Hkv, D, num_blocks)
    tables, pos = [], 0
    for cs in chunk_sets:
        tb = []
        for L in cs:
            n = (L + 15) // 16
            ids = perm[pos:pos + n]
            pos += n
            k = torch.randn(1, Hkv, L, D, generator=g).to(torch.float16)
            v = torch.randn(1, Hkv, L, D, generator=g).to(torch.float16)
            alloc.write_chunk_int8(0, ids, *quantize_chunk_int8(k.cuda(), v.cuda()))
            tb.extend(ids)
        tables.append(tb)
    prefix = [sum(cs) for cs in chunk_sets]
    P = max(prefix)
    q = torch.randn(B, Hq, Sq, D, generator=g).to(dtype)
    kn = torch.randn(B, Hkv, Sq, D, generator=g).to(dtype)
    vn = torch.randn(B, Hkv, Sq, D, generator=g).to(dtype)
    bt = block_table_tensor(tables, "cuda")
    pl = torch.tensor(prefix, dtype=torch.int32, device="cuda")
    o, lse = paged_prefill_attention(q.cuda(), kn.cuda(), vn.cuda(), alloc, 0, bt, P,
                                     prefix_lens=pl, softmax_scale=1.0 / math.sqrt(D),
                                     fused_only=fused_only)
    torch.cuda.synchronize()
    from kvboost_b200 import ops
    assert ops.read_status(torch.device("cuda")) == 0
    for b in range(B):
        kp, vp = _oracle_prefix(alloc, tables[b], prefix[b]) if prefix[b] else (
            np.zeros((Hkv, 0, D), np.float16), np.zeros((Hkv, 0, D), np.float16))
        # the reference casts the float16 dequantised K/V to the model dtype
        kp = torch.from_numpy(kp).to(dtype).float().numpy()
        vp = torch.from_numpy(vp).to(dtype).float().numpy()
        k_all = np.concatenate([kp, kn[b].float().numpy()], axis=1)[None]
        v_all = np.concatenate([vp, vn[b].float().numpy()], axis=1)[None]
        qb = q[b:b + 1].float().numpy()
        ob = o[b:b + 1].float().cpu().numpy()
        lb = lse[b:b + 1].cpu().numpy()
        if rows is not None:  # the last `rows` queries only (same bottom-right offsets)
            qb, ob, lb = qb[:, :, -rows:], ob[:, :, -rows:], lb[:, :, -rows:]
        if heads is not None:  # whole GQA groups [h0, h1) of query heads, every row
            h0, h1 = heads
            g = Hq // Hkv
            assert h0 % g == 0 and h1 % g == 0
            qb, ob, lb = qb[:, h0:h1], ob[:, h0:h1], lb[:, h0:h1]
            k_all, v_all = k_all[:, h0 // g:h1 // g], v_all[:, h0 // g:h1 // g]
        o_ref, l_ref = oattn.attention(qb, k_all, v_all, 1.0 / math.sqrt(D), True,
                                       compute_dtype=np.float32)
        err = np.abs(ob - o_ref).max()
        assert err <= TOL[dtype], f"batch {b}: max-abs {err}"
        assert np.abs(lb - l_ref).max() <= 2e-3


# fused: gather + dequantise inside the attention kernel's load stage;
# materialised: one dequantise pass into a workspace, then the dense kernel.
STRATEGIES = [pytest.param(True, id="fused"), pytest.param(False, id="auto")]


@pytest.mark.parametrize("fused_only", STRATEGIES)
def test_paged_config5_shape_reduced(fused_only):
    """GQA 8, D128, bf16: 8 cached chunks at a random block permutation + 200 new tokens."""
    _run_case(1, 16, 2, 128, [[128] * 8], 200, torch.bfloat16, seed=5, fused_only=fused_only)


@pytest.mark.parametrize("fused_only", STRATEGIES)
def test_paged_ragged_batch(fused_only):
    """Per-sequence prefixes: full chunks, a partial last chunk, and no prefix at all."""
    _run_case(3, 8, 2, 128, [[128, 128, 128], [128, 100], []], 330, torch.bfloat16, seed=6,
              fused_only=fused_only)


@pytest.mark.parametrize("fused_only", STRATEGIES)
@pytest.mark.parametrize("D,dtype", [(64, torch.float16), (96, torch.float16), (128, torch.float16),
                                     (64, torch.bfloat16)])
def test_paged_head_dims(D, dtype, fused_only):
    _run_case(2, 16, 2, D, [[128] * 3, [128] * 2], 277, dtype, seed=D, fused_only=fused_only)


def test_paged_suffix_shorter_than_tile_mha():
    _run_case(1, 4, 4, 128, [[128] * 5], 16, torch.bfloat16, seed=9)


@pytest.mark.parametrize("fused_only", STRATEGIES)
def test_paged_config5_full_size_last_rows(fused_only):
    """The full 32K-prefix paged workload on one GPU: P=32768 int8 prefix in an 8192-block pool, 2048 new
    tokens, Hq 64 / Hkv 8, D 128; the last 64 query rows of every head are checked."""
    _run_case(1, 64, 8, 128, [[128] * 256], 2048, torch.bfloat16, seed=50, num_blocks=8192,
              rows=64, fused_only=fused_only)


@pytest.mark.parametrize("fused_only", STRATEGIES)
def test_paged_config5_full_size_whole_group(fused_only):
    """The full 32K-prefix paged workload (P 32768 int8 in an 8192-block pool at a seeded
    permutation, 2048 new tokens, Hq 64 / Hkv 8, D 128, bf16): every one of the 2048 query
    rows of one whole GQA group (8 query heads over KV head 5) against the oracle."""
    _run_case(1, 64, 8, 128, [[128] * 256], 2048, torch.bfloat16, seed=51, num_blocks=8192,
              heads=(40, 48), fused_only=fused_only)


@pytest.mark.parametrize("fused_only", STRATEGIES)
def test_bad_block_id_is_reported_not_read(fused_only):
    from kvboost_b200 import ops
    from kvboost_b200.paged import DeviceBlockAllocator, paged_prefill_attention
    alloc = DeviceBlockAllocator(1, 2, 64, 8)
    bt = torch.tensor([[0, 99]], dtype=torch.int32, device="cuda")  # 99 is outside the pool
    q = torch.randn(1, 16, 256, 64, device="cuda", dtype=torch.bfloat16)
    kn = torch.randn(1, 2, 256, 64, device="cuda", dtype=torch.bfloat16)
    o, _ = paged_prefill_attention(q, kn, kn.clone(), alloc, 0, bt, 32, fused_only=fused_only)
    torch.cuda.synchronize()
    assert ops.read_status(torch.device("cuda")) & 16
    assert torch.isfinite(o.float()).all()


def test_context_parallel_emulated_two_ranks():
    """Chunk-sharded pool gathered (here by concatenation, as the NCCL all-gather lays
    it out) + zig-zag query split: each rank's rows equal the unsharded paged prefill."""
    from kvboost_b200 import context_parallel as cp
    from kvboost_b200.paged import (DeviceBlockAllocator, block_table_tensor,
                                    paged_prefill_attention, quantize_chunk_int8)
    world, Hq, Hkv, D, C, Sq = 2, 16, 2, 128, 9, 512
    P = C * 128
    g = torch.Generator().manual_seed(21)
    full = DeviceBlockAllocator(1, Hkv, D, C * 8)
    for c in range(C):
        k = torch.randn(1, Hkv, 128, D, generator=g).to(torch.bfloat16).half()
        v = torch.randn(1, Hkv, 128, D, generator=g).to(torch.bfloat16).half()
        full.write_chunk_int8(0, list(range(c * 8, c * 8 + 8)), *quantize_chunk_int8(k.cuda(), v.cuda()))
    q = torch.randn(1, Hq, Sq, D, generator=g).to(torch.bfloat16).cuda()
    kn = torch.randn(1, Hkv, Sq, D, generator=g).to(torch.bfloat16).cuda()
    vn = torch.randn(1, Hkv, Sq, D, generator=g).to(torch.bfloat16).cuda()
    ref, _ = paged_prefill_attention(q, kn, vn, full, 0,
                                     block_table_tensor([list(range(C * 8))], "cuda"), P)
    # what the all-gather of the per-rank shards produces
    nb = cp.shard_chunks(C, world) * 8
    gathered = DeviceBlockAllocator(1, Hkv, D, world * nb)
    for r in range(world):
        for slot, c in enumerate(cp.local_chunk_slots(C, world, r)):
            src, dst = slice(c * 8, c * 8 + 8), slice(r * nb + slot * 8, r * nb + slot * 8 + 8)
            gathered.pools[0][dst] = full.pools[0][src]
            gathered.k_scale[0][dst] = full.k_scale[0][src]
            gathered.v_scale[0][dst] = full.v_scale[0][src]
    out = torch.empty_like(q)
    for r in range(world):
        rows = torch.cat([torch.arange(s, e) for s, e in cp.zigzag_chunks(Sq, world, r)]).cuda()
        o_local = cp.cp_rank_prefill(q[:, :, rows].contiguous(), gathered, kn, vn, P, Sq, world, r)
        out[:, :, rows] = o_local
    torch.cuda.synchronize()
    assert (out.float() - ref.float()).abs().max().item() <= TOL[torch.bfloat16]


def _pool_with_chunks(Hkv, D, chunk_sets, seed, num_blocks=256):
    """A one-layer int8 pool holding each sequence's chunks at a seeded permutation."""
    from kvboost_b200.paged import DeviceBlockAllocator, quantize_chunk_int8
    g = torch.Generator().manual_seed(seed)
    perm = torch.randperm(num_blocks, generator=g).tolist()
    alloc = DeviceBlockAllocator(1, Hkv, D, num_blocks)
    tables, pos = [], 0
    for cs in chunk_sets:
        tb = []
        for L in cs:
            ids = perm[pos:pos + (L + 15) // 16]
            pos += len(ids)
            k = torch.randn(1, Hkv, L, D, generator=g).to(torch.float16)
            v = torch.randn(1, Hkv, L, D, generator=g).to(torch.float16)
            alloc.write_chunk_int8(0, ids, *quantize_chunk_int8(k.cuda(), v.cuda()))
            tb.extend(ids)
        tables.append(tb)
    return alloc, tables, max(sum(cs) for cs in chunk_sets)


def test_materialize_matches_oracle_gather():
    """kvb_paged_materialize: prefix dequantised through the block table + suffix, rows
    past the end zero up to the next 128."""
    from kvboost_b200.paged import block_table_tensor, paged_materialize
    alloc, tables, P = _pool_with_chunks(2, 64, [[128, 128, 100], [128]], seed=33)
    kn = torch.randn(2, 2, 40, 64).to(torch.float16).cuda()
    vn = torch.randn(2, 2, 40, 64).to(torch.float16).cuda()
    plens = torch.tensor([356, 128], dtype=torch.int32, device="cuda")
    bt = block_table_tensor(tables, "cuda")
    K, V = paged_materialize(alloc, 0, bt, 356, kn, vn, prefix_lens=plens)
    torch.cuda.synchronize()
    for b, Pb in enumerate([356, 128]):
        pre = _oracle_prefix(alloc, tables[b], Pb)            # float16 [H, P, D] K then V
        Kb = K[b].float().cpu().numpy()
        Vb = V[b].float().cpu().numpy()
        assert np.array_equal(Kb[:, :Pb], pre[0].astype(np.float32))
        assert np.array_equal(Vb[:, :Pb], pre[1].astype(np.float32))
        assert np.array_equal(Kb[:, Pb:Pb + 40], kn[b].float().cpu().numpy())
        pad_end = (Pb + 40 + 127) // 128 * 128
        assert not Kb[:, Pb + 40:pad_end].any() and not Vb[:, Pb + 40:pad_end].any()


def test_context_parallel_peer_shards_emulated():
    """The fused gather: two ranks' shard buffers (here both in this GPU's memory) read in
    place by kvb_paged_materialize_peers; each rank's zig-zag rows equal the unsharded
    paged prefill, and the dense K/V equal the NCCL-path layout bit for bit."""
    from kvboost_b200 import context_parallel as cp
    from kvboost_b200.paged import (DeviceBlockAllocator, block_table_tensor,
                                    paged_materialize, paged_prefill_attention,
                                    quantize_chunk_int8)
    world, Hq, Hkv, D, C, Sq = 2, 16, 2, 128, 9, 512
    P = C * 128
    g = torch.Generator().manual_seed(23)
    chunks = []
    full = DeviceBlockAllocator(1, Hkv, D, C * 8)
    for c in range(C):
        k = torch.randn(1, Hkv, 128, D, generator=g).to(torch.bfloat16).half().cuda()
        v = torch.randn(1, Hkv, 128, D, generator=g).to(torch.bfloat16).half().cuda()
        qz = quantize_chunk_int8(k, v)
        chunks.append(qz)
        full.write_chunk_int8(0, list(range(c * 8, c * 8 + 8)), *qz)
    q = torch.randn(1, Hq, Sq, D, generator=g).to(torch.bfloat16).cuda()
    kn = torch.randn(1, Hkv, Sq, D, generator=g).to(torch.bfloat16).cuda()
    vn = torch.randn(1, Hkv, Sq, D, generator=g).to(torch.bfloat16).cuda()
    ref, _ = paged_prefill_attention(q, kn, vn, full, 0,
                                     block_table_tensor([list(range(C * 8))], "cuda"), P)
    shards = [cp.PeerShardBuffer(C, world, Hkv, D, Sq, torch.bfloat16, "cuda", symmetric=False)
              for _ in range(world)]
    for r, sh in enumerate(shards):
        for slot, c in enumerate(cp.local_chunk_slots(C, world, r)):
            sh.alloc.write_chunk_int8(0, list(range(slot * 8, slot * 8 + 8)), *chunks[c])
        rows = torch.cat([torch.arange(s, e) for s, e in cp.zigzag_chunks(Sq, world, r)]).cuda()
        sh.suffix_k.copy_(kn[0][:, rows])
        sh.suffix_v.copy_(vn[0][:, rows])
    bases = [sh.buf.data_ptr() for sh in shards]
    table = block_table_tensor([cp.gathered_block_table(C, world)], "cuda")
    K, V = cp.materialize_from_peers(bases, shards[0].shard_blocks, shards[0].zz_rows, Hkv, D,
                                     torch.bfloat16, table, P, Sq, world * shards[0].shard_blocks)
    K_ref, V_ref = paged_materialize(full, 0, block_table_tensor([list(range(C * 8))], "cuda"),
                                     P, kn, vn)
    torch.cuda.synchronize()
    assert torch.equal(K, K_ref) and torch.equal(V, V_ref)
    out = torch.empty_like(q)
    for r in range(world):
        rows = torch.cat([torch.arange(s, e) for s, e in cp.zigzag_chunks(Sq, world, r)]).cuda()
        out[:, :, rows] = cp.zigzag_prefill(q[:, :, rows].contiguous(), K, V, P, Sq, world, r)
    torch.cuda.synchronize()
    assert (out.float() - ref.float()).abs().max().item() <= TOL[torch.bfloat16]
