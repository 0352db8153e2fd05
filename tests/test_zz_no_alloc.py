"""GPU: ``kvb_paged_prefill_fwd_noalloc`` against ``kvb_paged_prefill_fwd`` and the oracle.

The no-allocation entry point keeps the dequantised prefix in the library's
static per-device scratch instead of a workspace the caller allocates.  On two
calls in a row (the second reuses the scratch the first wrote) it must agree
with the existing entry point and with the oracle (the reference's host path:
dequantise, gather by the block table, bottom-right causal attention) within
the paged tests' tolerance; a small ragged call after a large one must not see
the large call's rows left in the scratch; it must allocate no device memory
after its first call, and reject requests larger than the scratch.  The file
name sorts last so it also runs after every other test.
"""

import math

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
TOL = {torch.bfloat16: 2e-2, torch.float16: 1e-2}


@pytest.fixture(autouse=True)
def _gpu():
    if not torch.cuda.is_available() or torch.cuda.get_device_capability()[0] != 10:
        pytest.skip("needs an sm_100 (B200) device")
    from kvboost_b200 import ops
    ops.read_status(torch.device("cuda"))      # start from a clear status word
    yield
    assert ops.read_status(torch.device("cuda")) == 0


def _case(B, Hq, Hkv, D, prefixes, Sq, dtype, seed, num_blocks=512):
    """Pool with each sequence's prefix at a seeded permutation of block ids."""
    from kvboost_b200.paged import DeviceBlockAllocator, block_table_tensor, quantize_chunk_int8
    g = torch.Generator().manual_seed(seed)
    perm = torch.randperm(num_blocks, generator=g).tolist()
    alloc = DeviceBlockAllocator(1, Hkv, D, num_blocks)
    tables, pos = [], 0
    for P in prefixes:
        tb = []
        for c0 in range(0, P, 128):
            L = min(128, P - c0)
            ids = perm[pos:pos + (L + 15) // 16]
            pos += len(ids)
            k = torch.randn(1, Hkv, L, D, generator=g).to(torch.float16)
            v = torch.randn(1, Hkv, L, D, generator=g).to(torch.float16)
            alloc.write_chunk_int8(0, ids, *quantize_chunk_int8(k.cuda(), v.cuda()))
            tb.extend(ids)
        tables.append(tb)
    q = torch.randn(B, Hq, Sq, D, generator=g).to(dtype).cuda()
    kn = torch.randn(B, Hkv, Sq, D, generator=g).to(dtype).cuda()
    vn = torch.randn(B, Hkv, Sq, D, generator=g).to(dtype).cuda()
    bt = block_table_tensor(tables, "cuda")
    plens = (torch.tensor(prefixes, dtype=torch.int32, device="cuda")
             if len(set(prefixes)) > 1 else None)
    return q, kn, vn, alloc, bt, max(prefixes), plens, tables


def _oracle(q, kn, vn, alloc, tables, prefixes, dtype):
    """O and LSE of the reference's host path for every sequence (float32)."""
    from oracle import attention as oattn
    from oracle import paged as opaged
    pool = alloc.pools[0].cpu().numpy()
    ks = alloc.k_scale16[0].cpu().numpy()
    vs = alloc.v_scale16[0].cpu().numpy()
    D = q.shape[-1]
    outs, lses = [], []
    for b, P in enumerate(prefixes):
        H = kn.shape[1]
        kp, vp = (opaged.dequant_gather(pool, ks, vs, tables[b], P, 16) if P else   # float16
                  (np.zeros((H, 0, D), np.float16), np.zeros((H, 0, D), np.float16)))  # [H, P, D]
        kp = torch.from_numpy(kp).to(dtype).float().numpy()              # to the model dtype
        vp = torch.from_numpy(vp).to(dtype).float().numpy()
        k_all = np.concatenate([kp, kn[b].float().cpu().numpy()], axis=1)[None]
        v_all = np.concatenate([vp, vn[b].float().cpu().numpy()], axis=1)[None]
        o, l = oattn.attention(q[b:b + 1].float().cpu().numpy(), k_all, v_all,
                               1.0 / math.sqrt(D), True, compute_dtype=np.float32)
        outs.append(o[0])
        lses.append(l[0])
    return np.stack(outs), np.stack(lses)


@pytest.mark.parametrize("B,Hq,Hkv,D,prefixes,Sq,dtype", [
    (2, 16, 4, 128, [768, 768], 256, torch.bfloat16),     # existing path also materialises
    (2, 8, 8, 64, [640, 256], 100, torch.float16),        # existing path fused, ragged prefixes
    (1, 12, 4, 96, [1000], 300, torch.bfloat16),          # odd GQA group, partial chunk
])
def test_noalloc_matches_existing_entry_point(B, Hq, Hkv, D, prefixes, Sq, dtype):
    from kvboost_b200.ops import status_word
    from kvboost_b200.paged import paged_prefill_attention, paged_prefill_attention_noalloc
    q, kn, vn, alloc, bt, P, plens, tables = _case(B, Hq, Hkv, D, prefixes, Sq, dtype,
                                                   seed=B * 100 + D)
    ref, ref_lse = paged_prefill_attention(q, kn, vn, alloc, 0, bt, P, prefix_lens=plens)
    st = status_word(q.device)
    outs = [torch.full_like(q, float("nan")) for _ in range(2)]
    lses = [torch.full((B, Hq, Sq), float("nan"), device="cuda") for _ in range(2)]
    for o, l in zip(outs, lses):      # two calls in a row over the same scratch
        paged_prefill_attention_noalloc(q, kn, vn, alloc, 0, bt, P, o, lse=l, prefix_lens=plens,
                                        status=st)
    torch.cuda.synchronize()
    o_or, l_or = _oracle(q, kn, vn, alloc, tables, prefixes, dtype)
    for o, l in zip(outs, lses):
        assert torch.isfinite(o).all()
        assert (o.float() - ref.float()).abs().max().item() <= TOL[dtype]
        assert (l - ref_lse).abs().max().item() <= 2e-3
        assert np.abs(o.float().cpu().numpy() - o_or).max() <= TOL[dtype]
        assert np.abs(l.cpu().numpy() - l_or).max() <= 2e-3


def test_noalloc_small_ragged_call_after_large_call():
    """The scratch keeps the last call's rows.  A large call (B 4, long prefixes)
    fills most of it; a smaller call with ragged prefixes that follows must read
    only what it wrote itself: equal to the existing entry point and the oracle."""
    from kvboost_b200.ops import status_word
    from kvboost_b200.paged import paged_prefill_attention, paged_prefill_attention_noalloc
    big = _case(4, 16, 4, 128, [3072, 2944, 3072, 2000], 256, torch.bfloat16, seed=11,
                num_blocks=1024)
    q, kn, vn, alloc, bt, P, plens, _ = big
    out = torch.empty_like(q)
    st = status_word(q.device)
    paged_prefill_attention_noalloc(q, kn, vn, alloc, 0, bt, P, out, prefix_lens=plens, status=st)
    prefixes = [300, 0, 1100]
    q, kn, vn, alloc, bt, P, plens, tables = _case(3, 8, 2, 128, prefixes, 77, torch.bfloat16,
                                                   seed=12)
    small = torch.full_like(q, float("nan"))
    paged_prefill_attention_noalloc(q, kn, vn, alloc, 0, bt, P, small, prefix_lens=plens,
                                    status=st)
    ref, _ = paged_prefill_attention(q, kn, vn, alloc, 0, bt, P, prefix_lens=plens)
    torch.cuda.synchronize()
    assert torch.isfinite(small).all()
    assert (small.float() - ref.float()).abs().max().item() <= TOL[torch.bfloat16]
    o_or, _ = _oracle(q, kn, vn, alloc, tables, prefixes, torch.bfloat16)
    assert np.abs(small.float().cpu().numpy() - o_or).max() <= TOL[torch.bfloat16]


def test_noalloc_allocates_nothing_after_setup():
    from kvboost_b200.paged import paged_prefill_attention_noalloc
    q, kn, vn, alloc, bt, P, plens, _ = _case(1, 8, 2, 128, [1024], 512, torch.bfloat16, seed=7)
    out = torch.empty_like(q)
    paged_prefill_attention_noalloc(q, kn, vn, alloc, 0, bt, P, out)   # first call: setup
    torch.cuda.synchronize()
    reserved = torch.cuda.memory_reserved()
    free0, _ = torch.cuda.mem_get_info()
    for _ in range(3):
        paged_prefill_attention_noalloc(q, kn, vn, alloc, 0, bt, P, out)
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert torch.cuda.memory_reserved() == reserved
    assert free1 == free0


def test_noalloc_rejects_requests_beyond_scratch():
    """4 x 8 KV heads x round_up(4096 + 128, 128) x D128 needs 66 MiB > 32 MiB: refused
    before any launch (the block table's ids are all valid regardless)."""
    from kvboost_b200 import _lib
    from kvboost_b200.paged import DeviceBlockAllocator, paged_prefill_attention_noalloc
    B, Hq, Hkv, D, Sq, P = 4, 8, 8, 128, 128, 4096
    alloc = DeviceBlockAllocator(1, Hkv, D, 16)
    bt = torch.zeros(B, P // 16, dtype=torch.int32, device="cuda")
    q = torch.randn(B, Hq, Sq, D, device="cuda").to(torch.bfloat16)
    kn = torch.randn(B, Hkv, Sq, D, device="cuda").to(torch.bfloat16)
    vn = torch.randn_like(kn)
    out = torch.zeros_like(q)
    need = 2 * B * Hkv * ((P + Sq + 127) // 128 * 128) * D * 2
    assert need > _lib.KVB_NOALLOC_SCRATCH_BYTES
    with pytest.raises(RuntimeError, match="static scratch holds 33554432"):
        paged_prefill_attention_noalloc(q, kn, vn, alloc, 0, bt, P, out)
    torch.cuda.synchronize()
    assert out.abs().sum().item() == 0      # nothing ran
