"""Pin the CPU oracle against golden vectors produced by the reference itself.

The fixtures in ``tests/golden/`` were made by ``tests/golden/make_golden.py``
running KVBoost's own code (SDPA dispatch, KIVI int8, the paged allocator,
chunk hashing).  These tests need no GPU and no reference checkout.
"""

import json
import math
import os

import numpy as np
import pytest

from oracle import attention as oattn
from oracle import hashing as ohash
from oracle import kv_quant as oq
from oracle import paged as opaged


def _load(golden_dir, name):
    return np.load(os.path.join(golden_dir, name))


def _vals(arr, dtype_code):
    """Stored 16-bit floats are raw bit patterns; return their exact float32 values."""
    if dtype_code == 0:
        return arr.astype(np.float32)
    if dtype_code == 1:
        return oq.bf16_bits_to_f32(arr)
    return arr.view(np.float16).astype(np.float32)


ATTN_CASES = [
    "square_causal_f32", "square_noncausal_f32", "seq1_f32", "cross_noncausal_f32",
    "reuse_gqa4_f32", "reuse_gqa4_bf16", "reuse_mha_d96_f16", "square_d64_bf16",
    "suffix_longer_than_prefix_bf16",
]


@pytest.mark.parametrize("case", ATTN_CASES)
def test_attention_oracle_matches_reference(golden_dir, case):
    d = _load(golden_dir, "attention.npz")
    B, Hq, Hkv, Sq, Skv, D, causal, dt = d[case + "/meta"].tolist()
    q, k, v, o_ref = (_vals(d[f"{case}/{n}"], dt) for n in "qkvo")
    o, lse = oattn.attention(q, k, v, 1.0 / math.sqrt(D), bool(causal))
    # The reference output was rounded to the input dtype by SDPA; the oracle
    # computes in float64.  fp32 agrees to 1e-5, 16-bit outputs to one ulp-ish.
    tol = {0: 1e-5, 1: 2e-2, 2: 4e-3}[dt]
    assert o.shape == o_ref.shape
    assert np.max(np.abs(o - o_ref)) <= tol
    assert np.all(np.isfinite(lse))


def test_offset_mask_is_hf_tril():
    m = oattn.visible_mask(3, 7, True)
    expect = np.tril(np.ones((3, 7), dtype=bool), k=4)
    assert np.array_equal(m, expect)
    assert np.array_equal(oattn.visible_mask(5, 5, True), np.tril(np.ones((5, 5), dtype=bool)))


def test_lse_matches_definition():
    rng = np.random.default_rng(0)
    q = rng.standard_normal((1, 2, 5, 16))
    k = rng.standard_normal((1, 2, 9, 16))
    v = rng.standard_normal((1, 2, 9, 16))
    _, lse = oattn.attention(q, k, v, 0.25, True)
    s = np.einsum("bhqd,bhkd->bhqk", q, k) * 0.25
    s = np.where(oattn.visible_mask(5, 9, True), s, -np.inf)
    ref = np.log(np.exp(s).sum(-1))
    assert np.allclose(lse, ref, atol=1e-6)


def test_empty_rows_give_zero_and_neg_inf():
    q = np.ones((1, 1, 4, 8))
    k = np.ones((1, 1, 2, 8))
    v = np.ones((1, 1, 2, 8))
    o, lse = oattn.attention(q, k, v, 1.0, True)  # q_len > kv_len: first 2 rows see nothing
    assert np.all(o[0, 0, :2] == 0) and np.all(np.isneginf(lse[0, 0, :2]))
    assert np.all(np.isfinite(lse[0, 0, 2:]))


@pytest.mark.parametrize("i", [0, 1, 2])
def test_int8_quant_bit_exact(golden_dir, i):
    d = _load(golden_dir, "kv_quant.npz")
    p = f"q{i}/"
    key_q, key_scale, val_q, val_scale = oq.quantize_int8(d[p + "key"], d[p + "val"])
    assert np.array_equal(key_q, d[p + "key_q"])
    assert np.array_equal(key_scale.view(np.uint16), d[p + "key_scale"].view(np.uint16))
    assert np.array_equal(val_q, d[p + "val_q"])
    assert np.array_equal(val_scale.view(np.uint16), d[p + "val_scale"].view(np.uint16))
    kd = oq.dequantize_int8(d[p + "key_q"], d[p + "key_scale"])
    vd = oq.dequantize_int8(d[p + "val_q"], d[p + "val_scale"])
    assert np.array_equal(kd.view(np.uint16), d[p + "key_deq"].view(np.uint16))
    assert np.array_equal(vd.view(np.uint16), d[p + "val_deq"].view(np.uint16))


def test_block_tables_bit_exact(golden_dir):
    with open(os.path.join(golden_dir, "paged_tables.json")) as f:
        t = json.load(f)
    a = opaged.AllocatorModel(40)
    m = opaged.MapperModel(a, 16)
    assert m.load_chunk("c1", 128) == t["load_c1"]
    assert m.load_chunk("c2", 100) == t["load_c2"]
    assert m.load_chunk("c1", 128) == t["reload_c1"]
    assert m.build_block_table([("c1", 128), ("c2", 100), ("c3", 40)]) == t["build_c1_c2_c3"]
    m.on_evict("c2")
    assert a.allocate(3) == t["after_evict_alloc3"]
    shared = a.fork(t["load_c1"][:2])
    assert a.ensure_writable(shared[0]) == t["cow_first"]
    # append 20 tokens at slot 128 of c1's table: one new block, CoW on shared ids
    table, off = opaged.append_slots(a, list(t["load_c1"]), 128, 20, 16)
    assert table == t["append_20_after_128"] and off == t["append_new_offset"]
    assert len(a.free_list) == t["free_blocks_end"]
    assert a.free_list == t["free_list_end"]


def test_read_kv_gather_exact(golden_dir):
    d = _load(golden_dir, "paged.npz")
    k, v = opaged.gather(d["read/pool"], d["read/table"].tolist(), 100)
    assert np.array_equal(k, d["read/k"]) and np.array_equal(v, d["read/v"])


def test_paged_attention_topleft(golden_dir):
    d = _load(golden_dir, "paged.npz")
    table = d["read/table"].tolist()
    hist_k, hist_v = [], []
    for tb, n in ((table, 100), (table[:3], 37), ([], 0)):
        if n:
            k, v = opaged.gather(d["read/pool"], tb, n)
        else:
            k = v = np.zeros((3, 0, 16), np.float32)
        hist_k.append(k)
        hist_v.append(v)
    o = oattn.paged_attention_topleft(d["pattn/q"], hist_k, hist_v, causal=True)
    assert np.max(np.abs(o - d["pattn/o"])) < 1e-5


def test_hashes_and_split_bit_exact(golden_dir):
    with open(os.path.join(golden_dir, "hashes.json")) as f:
        h = json.load(f)
    for c in h["content"]:
        assert ohash.content_hash(c["ids"]) == c["hash"]
    ids = h["chained_ids"]
    parent = None
    spans = ohash.fixed_split(ids)
    assert len(spans) == len(h["chained"])
    for (s, e, sl), c in zip(spans, h["chained"]):
        assert (s, e) == (c["start"], c["end"]) and c["parent"] == parent
        parent = ohash.chained_hash(sl, parent)
        assert parent == c["hash"]
    for sp in h["splits"]:
        assert [(s, e) for s, e, _ in ohash.fixed_split(list(range(sp["n"])))] == [tuple(x) for x in sp["spans"]]


def test_flop_count_config2():
    # 4 * 128 * 32 * 4 * (256*896 + 256*257/2) = 17.19 GFLOP
    f = oattn.attention_flops([256] * 4, [1152] * 4, 32, 128)
    assert f == 4 * 128 * 32 * 4 * (256 * 896 + 256 * 257 // 2)


@pytest.mark.parametrize("i", range(5))
def test_int8_quant_model_dtype_bit_exact(golden_dir, i):
    """Quantise-on-store arithmetic in the model's dtype (bf16, f16) == the reference."""
    d = _load(golden_dir, "kv_quant_model_dtypes.npz")
    p = f"b{i}/"
    code = int(d[p + "dtype"])
    name = "bf16" if code == 1 else "f16"
    key, val = _vals(d[p + "key"], code), _vals(d[p + "val"], code)
    key_q, key_scale, val_q, val_scale = oq.quantize_int8_model_dtype(key, val, name)
    assert np.array_equal(key_q, d[p + "key_q"])
    assert np.array_equal(val_q, d[p + "val_q"])
    assert np.array_equal(key_scale.view(np.uint16), d[p + "key_scale"])
    assert np.array_equal(val_scale.view(np.uint16), d[p + "val_scale"])
    kd = oq.dequantize_int8(key_q, key_scale)
    vd = oq.dequantize_int8(val_q, val_scale)
    assert np.array_equal(kd.view(np.uint16), d[p + "key_deq"])
    assert np.array_equal(vd.view(np.uint16), d[p + "val_deq"])


def test_quant_scale_division_single_rounding():
    """For every finite non-negative 16-bit value a, round(a / 127) == round(a * (1/127))
    in float32 and the oracle's rounding matches torch's CPU kernel (the one the
    reference runs)."""
    import torch
    for dt, name, top in ((torch.bfloat16, "bf16", 0x7F80), (torch.float16, "f16", 0x7C00)):
        a = torch.arange(0, top, dtype=torch.int32).to(torch.int16).view(dt)
        want = (a / 127.0).float().numpy()
        af = a.float().numpy()
        got = oq._round_to(af / np.float32(127.0), name)
        assert np.array_equal(got, want)
        assert np.array_equal(oq._round_to(af * (np.float32(1) / np.float32(127)), name), want)


CB_CASES = ["spread_f32", "none_above_f32", "few_above_f32", "gapped_bf16", "zero_row_f32"]


@pytest.mark.parametrize("case", CB_CASES)
def test_cacheblend_selection_matches_reference(golden_dir, case):
    from oracle import cacheblend as ocb
    d = _load(golden_dir, "cacheblend.npz")
    p = case + "/"
    L, H, S, D, is_bf16 = d[p + "meta"].tolist()
    code = 1 if is_bf16 else 0
    ck, fk = _vals(d[p + "cached_k"], code), _vals(d[p + "fresh_k"], code)
    assert ck.shape == (L, H, S, D)
    dev = ocb.deviation(ck, fk)
    k = ocb.num_select(S, float(d[p + "ratio"]))
    got = ocb.select(dev, k, float(d[p + "min_dev"]))
    assert got == d[p + "patched_positions"].tolist()


def _torch_vals(arr, dtype_code):
    import torch
    if dtype_code == 0:
        return torch.from_numpy(arr.astype(np.float32))
    t = torch.from_numpy(arr.astype(np.uint16).view(np.int16).copy())
    return t.view(torch.bfloat16 if dtype_code == 1 else torch.float16)


@pytest.mark.parametrize("case", ATTN_CASES)
def test_timed_cpu_path_reproduces_reference_bits(golden_dir, case):
    """``oracle.sdpa_ref`` (what the CPU baseline and the reference arm of the bench
    time) reproduces the reference dispatcher's outputs bit for bit."""
    import torch
    from oracle import sdpa_ref
    d = _load(golden_dir, "attention.npz")
    B, Hq, Hkv, Sq, Skv, D, causal, dt = d[case + "/meta"].tolist()
    q, k, v = (_torch_vals(d[f"{case}/{n}"], dt) for n in "qkv")
    if causal:
        o = sdpa_ref.reuse_prefill(q, k, v, 1.0 / math.sqrt(D))
    else:
        rep = Hq // Hkv
        o = sdpa_ref.kvboost_flash_attn_cpu(q, k.repeat_interleave(rep, 1),
                                            v.repeat_interleave(rep, 1), 1.0 / math.sqrt(D),
                                            False)
    ref = _torch_vals(d[case + "/o"], dt)
    assert o.dtype == ref.dtype and torch.equal(o, ref)
