"""Quantise-on-store and CacheBlend kernels against the oracle (and the reference's
own fixtures), through the C ABI.

* ``kvb_quantize_store``: pool bytes, float16 scales and their float32 copies
  bit-exact with ``oracle.kv_quant.quantize_int8_model_dtype`` then the block
  layout of ``write_chunk_int8``; the reference's fixtures
  (``tests/golden/kv_quant_model_dtypes.npz``) reproduced directly.
* ``kvb_cacheblend_fwd``: deviations within 1e-5 of the float64 oracle; the
  selection exactly the oracle's selection rule applied to the kernel's own
  deviations (ties included) and the reference's decided positions on its
  fixtures; the patch an exact row copy.
"""

import os

import numpy as np
import pytest
import torch

from oracle import cacheblend as ocb
from oracle import kv_quant as oq

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def _f32(t: torch.Tensor) -> np.ndarray:
    return t.float().cpu().numpy()


def _expected_pool(alloc, layer, blocks, key, val, dtype_name):
    """Oracle quantisation laid out as write_chunk_int8 lays it out (the pool
    rows, the per-token K scales and the per-block V scales of those blocks)."""
    kq, ks, vq, vs = oq.quantize_int8_model_dtype(_f32(key), _f32(val), dtype_name)
    H, S, D = key.shape
    n = len(blocks)
    pad = lambda a, last: np.concatenate(   # noqa: E731
        [a, np.zeros((H, n * 16 - S, last), a.dtype)], axis=1).reshape(H, n, 16, last).transpose(1, 0, 2, 3)
    pool = np.stack([pad(kq, D), pad(vq, D)], axis=1)                      # [n, 2, H, 16, D]
    kscale = pad(ks.reshape(H, S, 1), 1)[..., 0]                           # [n, H, 16]
    vscale = np.broadcast_to(vs.reshape(1, H, D), (n, H, D))
    return pool, kscale, vscale


def _check_layer(alloc, layer, blocks, key, val, dtype_name):
    pool, kscale, vscale = _expected_pool(alloc, layer, blocks, key, val, dtype_name)
    idx = torch.tensor(blocks, device=alloc.device)
    got_pool = alloc.pools[layer][idx].cpu().numpy()
    assert np.array_equal(got_pool, pool)
    got_ks = alloc.k_scale16[layer][idx].cpu().numpy()
    got_vs = alloc.v_scale16[layer][idx].cpu().numpy()
    assert np.array_equal(got_ks.view(np.uint16), kscale.astype(np.float16).view(np.uint16))
    assert np.array_equal(got_vs.view(np.uint16), np.ascontiguousarray(vscale).astype(np.float16).view(np.uint16))
    assert np.array_equal(alloc.k_scale[layer][idx].cpu().numpy(), got_ks.astype(np.float32))
    assert np.array_equal(alloc.v_scale[layer][idx].cpu().numpy(), got_vs.astype(np.float32))


@pytest.mark.parametrize("dt,D,S,mag", [
    (torch.bfloat16, 128, 128, 1.0), (torch.bfloat16, 64, 100, 1e-3), (torch.bfloat16, 96, 33, 50.0),
    (torch.float16, 128, 128, 1.0), (torch.float16, 128, 77, 1e-3), (torch.float16, 64, 16, 3.0)])
def test_quantize_store_bit_exact(dt, D, S, mag):
    from kvboost_b200.paged import DeviceBlockAllocator
    L, H = 3, 2
    g = torch.Generator().manual_seed(S * 7 + D)
    alloc = DeviceBlockAllocator(L, H, D, 64)
    alloc.allocate(5)                                   # not the first blocks
    blocks = alloc.allocate((S + 15) // 16)
    keys = [(torch.randn(1, H, S, D, generator=g) * mag).to(dt) for _ in range(L)]
    vals = [(torch.randn(1, H, S, D, generator=g) * mag * 2).to(dt) for _ in range(L)]
    keys[1][0, 0, S // 2] = 0                           # an all-zero K row
    vals[2][0, 1, :, 3] = 0                             # an all-zero V channel
    alloc.store_chunk_int8(blocks, [k.cuda() for k in keys], [v.cuda() for v in vals])
    torch.cuda.synchronize()
    name = "bf16" if dt == torch.bfloat16 else "f16"
    for layer in range(L):
        _check_layer(alloc, layer, blocks, keys[layer][0], vals[layer][0], name)


def test_quantize_store_model_cache_strides():
    """Sources laid out as a model's cache holds them: [1, H, S, D] views of a
    [1, S, H, D] projection (row stride H*D, head stride D)."""
    from kvboost_b200.paged import DeviceBlockAllocator
    L, H, S, D = 2, 4, 128, 128
    g = torch.Generator().manual_seed(3)
    alloc = DeviceBlockAllocator(L, H, D, 32)
    blocks = alloc.allocate(8)
    raw_k = [torch.randn(1, S, H, D, generator=g).to(torch.bfloat16).cuda() for _ in range(L)]
    raw_v = [torch.randn(1, S, H, D, generator=g).to(torch.bfloat16).cuda() for _ in range(L)]
    keys = [t.transpose(1, 2) for t in raw_k]
    vals = [t.transpose(1, 2) for t in raw_v]
    assert keys[0].stride() == (S * H * D, D, H * D, 1)
    alloc.store_chunk_int8(blocks, keys, vals)
    torch.cuda.synchronize()
    for layer in range(L):
        _check_layer(alloc, layer, blocks, keys[layer][0].cpu(), vals[layer][0].cpu(), "bf16")


@pytest.mark.parametrize("i", range(5))
def test_quantize_store_reproduces_reference_fixture(i):
    from kvboost_b200.paged import DeviceBlockAllocator
    d = np.load(os.path.join(GOLDEN, "kv_quant_model_dtypes.npz"))
    p = f"b{i}/"
    dt = torch.bfloat16 if int(d[p + "dtype"]) == 1 else torch.float16
    key = torch.from_numpy(d[p + "key"].view(np.int16)).view(dt)[0]
    val = torch.from_numpy(d[p + "val"].view(np.int16)).view(dt)[0]
    H, S, D = key.shape
    n = (S + 15) // 16
    alloc = DeviceBlockAllocator(1, H, D, n + 3)
    blocks = alloc.allocate(n)
    alloc.store_chunk_int8(blocks, key[None].cuda(), val[None].cuda())
    torch.cuda.synchronize()
    idx = torch.tensor(blocks)
    pool = alloc.pools[0].cpu()[idx]                                  # [n, 2, H, 16, D]
    kq = pool[:, 0].permute(1, 0, 2, 3).reshape(H, n * 16, D)[:, :S].numpy()
    vq = pool[:, 1].permute(1, 0, 2, 3).reshape(H, n * 16, D)[:, :S].numpy()
    assert np.array_equal(kq, d[p + "key_q"][0])
    assert np.array_equal(vq, d[p + "val_q"][0])
    ks = alloc.k_scale16[0].cpu()[idx].permute(1, 0, 2).reshape(H, n * 16)[:, :S].numpy()
    assert np.array_equal(ks.view(np.uint16), d[p + "key_scale"][0, :, :, 0])
    vs = alloc.v_scale16[0].cpu()[idx].numpy()
    for b in range(n):
        assert np.array_equal(vs[b].view(np.uint16), d[p + "val_scale"][0, :, 0, :])


def test_quantize_store_then_paged_gather_dequantises():
    """The stored chunk read back through the paged gather kernel equals the
    oracle's dequantisation (q * scale rounded once to the compute dtype)."""
    from kvboost_b200.paged import DeviceBlockAllocator, block_table_tensor, paged_materialize
    H, S, D = 2, 256, 128
    g = torch.Generator().manual_seed(11)
    key = torch.randn(1, H, S, D, generator=g).to(torch.float16)
    val = torch.randn(1, H, S, D, generator=g).to(torch.float16)
    alloc = DeviceBlockAllocator(1, H, D, 40)
    blocks = alloc.allocate(16)
    alloc.store_chunk_int8(blocks, key.cuda(), val.cuda())
    empty = torch.empty(1, H, 0, D, dtype=torch.float16, device="cuda")
    K, V = paged_materialize(alloc, 0, block_table_tensor([blocks], "cuda"), S, empty, empty)
    kq, ks, vq, vs = oq.quantize_int8_model_dtype(_f32(key[0]), _f32(val[0]), "f16")
    assert np.array_equal(K[0, :, :S].cpu().numpy().view(np.uint16),
                          oq.dequantize_int8(kq, ks).view(np.uint16))
    assert np.array_equal(V[0, :, :S].cpu().numpy().view(np.uint16),
                          oq.dequantize_int8(vq, vs).view(np.uint16))


# ── CacheBlend ────────────────────────────────────────────────────────────────

def _blend_inputs(L, H, S, D, dt, seed, mags=None):
    g = torch.Generator().manual_seed(seed)
    if mags is None:
        mags = torch.rand(S, generator=g) * 1.5
    ck = torch.randn(L, H, S, D, generator=g)
    cv = torch.randn(L, H, S, D, generator=g)
    fk = ck + mags.view(1, 1, S, 1) * torch.randn(L, H, S, D, generator=g)
    fv = torch.randn(L, H, S, D, generator=g)
    return [t.to(dt) for t in (ck, cv, fk, fv)]


@pytest.mark.parametrize("dt,L,H,S,D,ratio,min_dev", [
    (torch.bfloat16, 4, 2, 300, 128, 0.15, 0.01),
    (torch.float16, 3, 8, 1500, 64, 0.2, 0.05),
    (torch.bfloat16, 36, 2, 3072, 128, 0.15, 0.01),
    (torch.bfloat16, 2, 1, 33, 96, 0.5, 0.3),
])
def test_cacheblend_matches_oracle(dt, L, H, S, D, ratio, min_dev):
    from kvboost_b200.cacheblend import cacheblend_fwd
    ck, cv, fk, fv = _blend_inputs(L, H, S, D, dt, seed=S + L)
    want_dev = ocb.deviation(_f32(ck), _f32(fk))
    gck, gcv, gfk, gfv = (t.cuda() for t in (ck, cv, fk, fv))
    dev, sel, cnt = cacheblend_fwd(gck, gcv, gfk, gfv, ratio, min_dev, patch=True)
    torch.cuda.synchronize()
    dev = dev.cpu().numpy()
    assert np.abs(dev - want_dev).max() <= 1e-5
    k = ocb.num_select(S, ratio)
    want_sel = ocb.select(dev, k, min_dev)                   # the rule, on the kernel's deviations
    n = int(cnt.item())
    assert sel.cpu().tolist() == want_sel + [-1] * (k - len(want_sel))
    assert n == len(want_sel)
    # the oracle's own deviations choose the same set unless the k-th is a near-tie
    ref_sel = ocb.select(want_dev, k, min_dev)
    if ref_sel != want_sel:
        kth = np.sort(want_dev[want_dev > min_dev])[::-1][len(ref_sel) - 1]
        diff = set(ref_sel) ^ set(want_sel)
        assert all(abs(want_dev[i] - kth) <= 2e-5 for i in diff)
    pk, pv = ocb.patch(_f32(ck), _f32(cv), _f32(fk), _f32(fv), want_sel)
    assert np.array_equal(_f32(gck), pk)
    assert np.array_equal(_f32(gcv), pv)


def test_cacheblend_ties_take_lowest_positions():
    """Positions with bit-identical K rows have bit-identical deviations: the
    kernel takes the lowest ones first, across several 1024-position tiles."""
    from kvboost_b200.cacheblend import cacheblend_fwd
    L, H, S, D = 2, 2, 5000, 64
    g = torch.Generator().manual_seed(5)
    row_c = torch.randn(L, H, 1, D, generator=g)
    row_f = row_c + 0.7 * torch.randn(L, H, 1, D, generator=g)
    ck = row_c.expand(L, H, S, D).clone()
    fk = row_f.expand(L, H, S, D).clone()
    strong = torch.tensor([17, 1500, 4999])
    fk[:, :, strong] = -ck[:, :, strong]                     # deviation 2: always chosen
    ck, fk = ck.to(torch.bfloat16).cuda(), fk.to(torch.bfloat16).cuda()
    dev, sel, cnt = cacheblend_fwd(ck, None, fk, None, 0.1, 0.01, patch=False)
    k = ocb.num_select(S, 0.1)
    got = sel.cpu().tolist()
    assert int(cnt.item()) == k
    assert got == sorted(strong.tolist() + [i for i in range(S) if i not in set(strong.tolist())][:k - 3])
    assert got == ocb.select(dev.cpu().numpy(), k, 0.01)


def test_cacheblend_none_above_threshold_and_fewer_than_k():
    from kvboost_b200.cacheblend import cacheblend_fwd
    L, H, S, D = 2, 2, 200, 128
    mags = torch.full((S,), 1e-3)
    ck, cv, fk, fv = _blend_inputs(L, H, S, D, torch.bfloat16, 9, mags)
    gck = ck.cuda()
    dev, sel, cnt = cacheblend_fwd(gck, cv.cuda(), fk.cuda(), fv.cuda(), 0.15, 0.01)
    assert int(cnt.item()) == 0 and sel.cpu().tolist() == [-1] * 30
    assert torch.equal(gck.cpu(), ck)                        # nothing patched
    mags[[3, 50, 199]] = 2.0
    ck, cv, fk, fv = _blend_inputs(L, H, S, D, torch.bfloat16, 9, mags)
    dev, sel, cnt = cacheblend_fwd(ck.cuda(), cv.cuda(), fk.cuda(), fv.cuda(), 0.15, 0.01)
    assert int(cnt.item()) == 3 and sel.cpu().tolist()[:4] == [3, 50, 199, -1]


@pytest.mark.parametrize("case", ["spread_f32", "none_above_f32", "few_above_f32", "gapped_bf16",
                                  "zero_row_f32"])
def test_cacheblend_reproduces_reference_fixture(case):
    """The reference's decided positions (float32 cases run here in bfloat16 /
    float16 would reorder rounding-level ties, so they run as float16 after a check
    that the fixture's gaps are wide enough)."""
    from kvboost_b200.cacheblend import cacheblend_fwd
    d = np.load(os.path.join(GOLDEN, "cacheblend.npz"))
    p = case + "/"
    L, H, S, D, is_bf16 = d[p + "meta"].tolist()
    if is_bf16:
        ck = torch.from_numpy(d[p + "cached_k"].view(np.int16)).view(torch.bfloat16)
        fk = torch.from_numpy(d[p + "fresh_k"].view(np.int16)).view(torch.bfloat16)
    else:
        ck = torch.from_numpy(d[p + "cached_k"]).to(torch.float16)
        fk = torch.from_numpy(d[p + "fresh_k"]).to(torch.float16)
    ratio, min_dev = float(d[p + "ratio"]), float(d[p + "min_dev"])
    dev, sel, cnt = cacheblend_fwd(ck.cuda(), None, fk.cuda(), None, ratio, min_dev, patch=False)
    n = int(cnt.item())
    want = d[p + "patched_positions"].tolist()
    if not is_bf16:   # float16 rounding of float32 inputs: a choice within 1e-3 of the k-th may move
        dv = dev.cpu().numpy()
        got = sel.cpu().tolist()[:n]
        for i in set(got) ^ set(want):
            assert abs(dv[i] - np.sort(dv)[::-1][len(want) - 1]) < 1e-3
        return
    assert sel.cpu().tolist()[:n] == want


def test_many_layers_one_launch():
    """100 layers (the pointer tables near the kernels' 128-layer limit) in one launch
    each: quantise-on-store bit-exact, CacheBlend equal to the oracle's rule."""
    from kvboost_b200.cacheblend import cacheblend_fwd
    from kvboost_b200.paged import DeviceBlockAllocator
    L, H, S, D = 100, 1, 40, 64
    g = torch.Generator().manual_seed(100)
    alloc = DeviceBlockAllocator(L, H, D, 8)
    blocks = alloc.allocate(3)
    keys = [torch.randn(1, H, S, D, generator=g).to(torch.bfloat16) for _ in range(L)]
    vals = [torch.randn(1, H, S, D, generator=g).to(torch.bfloat16) for _ in range(L)]
    alloc.store_chunk_int8(blocks, [k.cuda() for k in keys], [v.cuda() for v in vals])
    torch.cuda.synchronize()
    for layer in (0, 57, 99):
        _check_layer(alloc, layer, blocks, keys[layer][0], vals[layer][0], "bf16")
    ck, cv, fk, fv = _blend_inputs(L, H, S, D, torch.bfloat16, 77)
    gck, gcv = ck.cuda(), cv.cuda()
    dev, sel, cnt = cacheblend_fwd(gck, gcv, fk.cuda(), fv.cuda(), 0.2, 0.01)
    dv = dev.cpu().numpy()
    assert np.abs(dv - ocb.deviation(_f32(ck), _f32(fk))).max() <= 1e-5
    want = ocb.select(dv, ocb.num_select(S, 0.2), 0.01)
    assert sel.cpu().tolist()[:int(cnt.item())] == want
    pk, pv = ocb.patch(_f32(ck), _f32(cv), _f32(fk), _f32(fv), want)
    assert np.array_equal(_f32(gck), pk) and np.array_equal(_f32(gcv), pv)


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
def test_batched_store_matches_oracle(dt):
    """Several chunks of ragged lengths in one kvb_quantize_store_batch launch."""
    from kvboost_b200.paged import DeviceBlockAllocator
    L, H, D = 4, 2, 128
    g = torch.Generator().manual_seed(21)
    alloc = DeviceBlockAllocator(L, H, D, 64)
    alloc.allocate(3)
    lens = [128, 100, 33, 16, 128]
    chunks, cpu = [], []
    for S in lens:
        blocks = alloc.allocate((S + 15) // 16)
        ks = [torch.randn(1, H, S, D, generator=g).to(dt) for _ in range(L)]
        vs = [torch.randn(1, H, S, D, generator=g).to(dt) for _ in range(L)]
        chunks.append((blocks, [k.cuda() for k in ks], [v.cuda() for v in vs]))
        cpu.append((blocks, ks, vs))
    alloc.store_chunks_int8(chunks)
    torch.cuda.synchronize()
    name = "bf16" if dt == torch.bfloat16 else "f16"
    for blocks, ks, vs in cpu:
        for layer in range(L):
            _check_layer(alloc, layer, blocks, ks[layer][0], vs[layer][0], name)


@pytest.mark.parametrize("D", [64, 128])
def test_batched_store_flags_bad_block_and_skips_it(D):
    """A block id outside the pool is skipped on the device (never written) and
    reported in the status word; the chunk's other blocks are still stored
    (head_dim 128 takes the shared-memory-staged kernel, 64 the other one)."""
    from kvboost_b200 import _lib, ops
    from kvboost_b200.paged import DeviceBlockAllocator
    L, H, S = 2, 2, 48
    g = torch.Generator().manual_seed(22)
    alloc = DeviceBlockAllocator(L, H, D, 8)
    ops.read_status(torch.device("cuda"))                     # start from 0
    ks = [torch.randn(1, H, S, D, generator=g).to(torch.bfloat16) for _ in range(L)]
    vs = [torch.randn(1, H, S, D, generator=g).to(torch.bfloat16) for _ in range(L)]
    alloc.store_chunks_int8([([5, 8 + 3, 6], [k.cuda() for k in ks], [v.cuda() for v in vs])])
    status = ops.read_status(torch.device("cuda"))
    assert status & _lib.KVB_STATUS_BAD_BLOCK
    kq, _, _, _ = oq.quantize_int8_model_dtype(_f32(ks[0][0]), _f32(vs[0][0]), "bf16")
    pool = alloc.pools[0].cpu().numpy()
    assert np.array_equal(pool[5, 0].reshape(H, 16, D), kq[:, :16])
    assert np.array_equal(pool[6, 0].reshape(H, 16, D), kq[:, 32:48])
