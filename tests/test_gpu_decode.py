"""GPU: split-key decode attention (``kvb_decode_fwd``) against the oracle.

Decode (one query per head) and the selective-recompute seams (up to 16
queries per head) over long key ranges: the query heads of a GQA group are
packed into one tile's rows and the keys are split over CTAs, then merged by
LSE.  Tolerances as everywhere: max-abs 2e-2 (bf16), 1e-2 (fp16), LSE 2e-3.
"""

import math

import numpy as np
import pytest
import torch

from oracle import attention as oattn

pytestmark = pytest.mark.gpu
TOL = {torch.bfloat16: 2e-2, torch.float16: 1e-2}


@pytest.fixture(autouse=True)
def _gpu():
    if not torch.cuda.is_available() or torch.cuda.get_device_capability()[0] != 10:
        pytest.skip("needs an sm_100 (B200) device")
    from kvboost_b200 import ops
    ops.read_status(torch.device("cuda"))
    yield
    assert ops.read_status(torch.device("cuda")) == 0


def _case(B, Hq, Hkv, Sq, Skv, D, dtype, seed, splits=None, top_left=False, causal=True):
    from kvboost_b200.ops import decode_attention
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, Hq, Sq, D, generator=g).to(dtype)
    k = torch.randn(B, Hkv, Skv, D, generator=g).to(dtype)
    v = torch.randn(B, Hkv, Skv, D, generator=g).to(dtype)
    o, lse = decode_attention(q.cuda(), k.cuda(), v.cuda(), 1.0 / math.sqrt(D), causal,
                              num_splits=splits, top_left=top_left)
    torch.cuda.synchronize()
    if top_left:
        o_ref, lse_ref = oattn.attention(q.float().numpy(), k.float().numpy(), v.float().numpy(),
                                         1.0 / math.sqrt(D), causal, compute_dtype=np.float32,
                                         top_left=True)
    else:
        o_ref, lse_ref = oattn.attention(q.float().numpy(), k.float().numpy(), v.float().numpy(),
                                         1.0 / math.sqrt(D), causal, compute_dtype=np.float32)
    assert np.abs(o.float().cpu().numpy() - o_ref).max() <= TOL[dtype]
    assert np.abs(lse.cpu().numpy() - lse_ref).max() <= 2e-3
    return o


@pytest.mark.parametrize("Skv", [1, 100, 129, 4097])
@pytest.mark.parametrize("D,dtype", [(128, torch.bfloat16), (64, torch.float16),
                                     (96, torch.bfloat16)])
def test_decode_one_query(Skv, D, dtype):
    _case(3, 16, 2, 1, Skv, D, dtype, seed=Skv + D)


@pytest.mark.parametrize("Hq,Hkv,Sq", [(16, 2, 16), (32, 2, 8), (32, 2, 16), (8, 8, 16),
                                       (12, 4, 5)])
def test_seam_queries(Hq, Hkv, Sq):
    _case(2, Hq, Hkv, Sq, 1500, 128, torch.bfloat16, seed=Hq * Sq)


def test_split_counts_agree():
    a = _case(1, 16, 2, 4, 3000, 128, torch.bfloat16, seed=5, splits=1)
    b = _case(1, 16, 2, 4, 3000, 128, torch.bfloat16, seed=5, splits=7)
    c = _case(1, 16, 2, 4, 3000, 128, torch.bfloat16, seed=5, splits=64)
    assert (a.float() - b.float()).abs().max().item() <= 2e-2
    assert (a.float() - c.float()).abs().max().item() <= 2e-2


def test_top_left_and_noncausal():
    _case(1, 8, 2, 6, 900, 64, torch.float16, seed=8, top_left=True)
    _case(1, 8, 2, 6, 900, 64, torch.float16, seed=9, causal=False)


def test_hf_layout_single_query():
    """HF hands [B, S, H, D] storage viewed as [B, H, S, D]; one query row per head."""
    from kvboost_b200.ops import decode_attention
    g = torch.Generator().manual_seed(3)
    q = torch.randn(2, 1, 16, 128, generator=g).to(torch.bfloat16).cuda().transpose(1, 2)
    k = torch.randn(2, 700, 2, 128, generator=g).to(torch.bfloat16).cuda().transpose(1, 2)
    v = torch.randn(2, 700, 2, 128, generator=g).to(torch.bfloat16).cuda().transpose(1, 2)
    out = torch.empty(2, 1, 16, 128, dtype=torch.bfloat16, device="cuda").transpose(1, 2)
    o, lse = decode_attention(q, k, v, out=out)
    torch.cuda.synchronize()
    o_ref, _ = oattn.attention(q.float().cpu().numpy(), k.float().cpu().numpy(),
                               v.float().cpu().numpy(), 1.0 / math.sqrt(128), True,
                               compute_dtype=np.float32)
    assert np.abs(o.float().cpu().numpy() - o_ref).max() <= 2e-2


@pytest.mark.parametrize("Hq,Hkv,Sq,D,dtype", [(4, 2, 6, 64, torch.float16), (32, 2, 1, 96, torch.float16),
                                                (16, 1, 1, 128, torch.bfloat16), (2, 2, 16, 128, torch.bfloat16)])
def test_small_groups_masks(Hq, Hkv, Sq, D, dtype):
    """Packed groups of 1-16 rows per KV head: bottom-right, top-left and no mask."""
    _case(2, Hq, Hkv, Sq, 777, D, dtype, seed=Hq + Sq)
    _case(1, Hq, Hkv, Sq, 300, D, dtype, seed=Hq + Sq + 1, top_left=True)
    _case(1, Hq, Hkv, Sq, 300, D, dtype, seed=Hq + Sq + 2, causal=False)


def test_one_query_split_counts_agree():
    a = _case(2, 16, 2, 1, 3000, 128, torch.bfloat16, seed=15, splits=1)
    b = _case(2, 16, 2, 1, 3000, 128, torch.bfloat16, seed=15, splits=5)
    c = _case(2, 16, 2, 1, 3000, 128, torch.bfloat16, seed=15, splits=24)
    assert (a.float() - b.float()).abs().max().item() <= 2e-2
    assert (a.float() - c.float()).abs().max().item() <= 2e-2


@pytest.mark.parametrize("B,Hq,Hkv,Sq,Skv,D,dtype,splits", [
    (2, 32, 4, 64, 1500, 128, torch.bfloat16, None),   # 512 packed rows: two tile pairs
    (1, 16, 2, 100, 2000, 128, torch.bfloat16, 3),     # 800 rows: last pair 32 rows
    (1, 4, 4, 300, 2100, 96, torch.float16, None),     # MHA, 300 rows: 256 + 44
    (2, 8, 2, 80, 700, 64, torch.float16, 1),          # one split: merge of one partial
])
def test_packed_tile_pairs(B, Hq, Hkv, Sq, Skv, D, dtype, splits):
    """More packed rows than one CTA's two tiles: CTAs per (tile pair, key split),
    every row's partials merged by the merge launch."""
    _case(B, Hq, Hkv, Sq, Skv, D, dtype, seed=Sq + Skv, splits=splits)
    _case(1, Hq, Hkv, Sq, Skv, D, dtype, seed=Sq + 1, splits=splits, top_left=True)
    _case(1, Hq, Hkv, Sq, Skv, D, dtype, seed=Sq + 2, splits=splits, causal=False)


@pytest.mark.parametrize("B,Hq,Hkv,Sq,Skv,layout", [
    (8, 16, 2, 16, 4096, "bhsd"),     # selective-recompute seam shape of the Qwen2.5-3B architecture
    (2, 32, 8, 64, 6000, "bshd"),     # short reuse suffix, HF output layout
    (1, 32, 32, 16, 8192, "bhsd"),    # MHA short suffix (short varlen requests)
])
def test_prefill_routes_short_suffix(B, Hq, Hkv, Sq, Skv, layout):
    """prefill_attention sends short suffixes over long prefixes to the split-key
    kernel (split_key_plan); results as the oracle, output in the asked layout."""
    from kvboost_b200.ops import prefill_attention, split_key_plan
    assert split_key_plan(B, Hq, Hkv, Sq, Skv)[0]
    g = torch.Generator().manual_seed(Sq * B)
    q = torch.randn(B, Hq, Sq, 128, generator=g).to(torch.bfloat16)
    k = torch.randn(B, Hkv, Skv, 128, generator=g).to(torch.bfloat16)
    v = torch.randn(B, Hkv, Skv, 128, generator=g).to(torch.bfloat16)
    o, lse = prefill_attention(q.cuda(), k.cuda(), v.cuda(), None, True, out_layout=layout)
    torch.cuda.synchronize()
    if layout == "bshd":
        assert o.shape == (B, Sq, Hq, 128) and o.is_contiguous()
        o = o.transpose(1, 2)
    o_ref, lse_ref = oattn.attention(q.float().numpy(), k.float().numpy(), v.float().numpy(),
                                     1.0 / math.sqrt(128), True, compute_dtype=np.float32)
    assert np.abs(o.float().cpu().numpy() - o_ref).max() <= 2e-2
    assert np.abs(lse.cpu().numpy() - lse_ref).max() <= 2e-3


@pytest.mark.parametrize("B,Hq,Hkv,Sq,Skv,D,dtype,splits", [
    (2, 8, 2, 3, 5000, 64, torch.float16, 5),      # ring of 4: two stages per slot
    (1, 4, 1, 16, 3333, 96, torch.bfloat16, 3),    # odd split count: last CTA's second slot empty
    (3, 16, 2, 8, 2600, 128, torch.bfloat16, 2),   # one CTA per group, both slots busy
    (1, 8, 1, 4, 891, 128, torch.bfloat16, 4),     # 7 tiles: last CTA's slots take 2 and 1
    (2, 8, 2, 1, 4097, 96, torch.bfloat16, 16),    # 11 splits: last CTA's second slot empty
])
def test_dual_key_ranges(B, Hq, Hkv, Sq, Skv, D, dtype, splits):
    """Packed rows within one tile: each CTA's two slots stream two key splits."""
    _case(B, Hq, Hkv, Sq, Skv, D, dtype, seed=Skv, splits=splits)
    _case(1, Hq, Hkv, Sq, Skv, D, dtype, seed=Skv + 1, splits=splits, causal=False)
