"""GPU parity: the sm_100a kernels against the pinned CPU oracle.

Tolerances are the ones stated for this path: max-abs 2e-2 on bfloat16
attention outputs, 1e-2 on float16 outputs; LSE (float32) within 2e-3.
Inputs are i.i.d. N(0, 1) from seeded torch generators, as in the configs
the reference is measured on.
"""

import math
import os

import numpy as np
import pytest
import torch

from oracle import attention as oattn
from oracle import kv_quant as oq

pytestmark = pytest.mark.gpu

TOL = {torch.bfloat16: 2e-2, torch.float16: 1e-2}
LSE_TOL = 2e-3


def _need_gpu():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    major, minor = torch.cuda.get_device_capability()
    if major != 10:
        pytest.skip("needs an sm_100 (B200) device")


@pytest.fixture(autouse=True)
def _gpu_and_status():
    _need_gpu()
    from kvboost_b200 import ops
    ops.read_status(torch.device("cuda"))
    yield
    torch.cuda.synchronize()
    assert ops.read_status(torch.device("cuda")) == 0, "a device-side wait gave up"


def _rand(shape, dtype, gen):
    return torch.randn(*shape, generator=gen).to(dtype)


def _check(o_gpu, lse_gpu, q, k, v, scale, causal, dtype, top_left=False):
    o_ref, lse_ref = oattn.attention(q.float().numpy(), k.float().numpy(), v.float().numpy(),
                                     scale, causal, compute_dtype=np.float32, top_left=top_left)
    o = o_gpu.float().cpu().numpy()
    err = np.max(np.abs(o - o_ref)) if o.size else 0.0
    assert err <= TOL[dtype], f"max-abs {err:.4g} > {TOL[dtype]}"
    if lse_gpu is not None:
        lse = lse_gpu.cpu().numpy()
        fin = np.isfinite(lse_ref)
        assert np.array_equal(np.isfinite(lse), fin)
        if fin.any():
            lerr = np.max(np.abs(lse[fin] - lse_ref[fin]))
            assert lerr <= LSE_TOL, f"lse max-abs {lerr:.4g}"
    return err


def _run(B, Hq, Hkv, Sq, Skv, D, dtype, causal=True, seed=0, top_left=False):
    from kvboost_b200.ops import prefill_attention
    g = torch.Generator().manual_seed(seed)
    q = _rand((B, Hq, Sq, D), dtype, g)
    k = _rand((B, Hkv, Skv, D), dtype, g)
    v = _rand((B, Hkv, Skv, D), dtype, g)
    scale = 1.0 / math.sqrt(D)
    o, lse = prefill_attention(q.cuda(), k.cuda(), v.cuda(), scale, causal, top_left=top_left)
    torch.cuda.synchronize()
    return _check(o, lse, q, k, v, scale, causal, dtype, top_left)


def test_config1_causal_op_full_size():
    """B2, 16 heads, S=1024, D=64, bf16, q_len == kv_len, seed 0."""
    _run(2, 16, 16, 1024, 1024, 64, torch.bfloat16)


def test_config2_prefix_reuse_full_size():
    """B4, Hq32/Hkv8, D128, bf16: 7 cached chunks (896) + 256-token suffix."""
    _run(4, 32, 8, 256, 1152, 128, torch.bfloat16)


@pytest.mark.parametrize("D", [64, 96, 128])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_head_dims_and_dtypes(D, dtype):
    _run(1, 4, 2, 200, 456, D, dtype, seed=D)


@pytest.mark.parametrize("Sq,Skv", [(1, 1), (1, 300), (16, 16), (100, 100), (130, 130),
                                     (128, 1024), (129, 257), (257, 2049), (64, 64 + 896)])
def test_tails_and_offsets(Sq, Skv):
    _run(2, 4, 4, Sq, Skv, 128, torch.bfloat16, seed=Sq * 7 + Skv)


@pytest.mark.parametrize("causal", [False, True])
def test_noncausal_and_causal(causal):
    _run(1, 8, 2, 77, 333, 64, torch.float16, causal=causal, seed=3)


@pytest.mark.parametrize("D,dtype,Sq,Skv,causal,top_left", [
    (128, torch.bfloat16, 100, 900, True, False),
    (96, torch.float16, 128, 1000, True, False),
    (64, torch.bfloat16, 37, 37, True, False),
    (128, torch.float16, 50, 60, True, False),      # fewer keys than one half-tile
    (128, torch.bfloat16, 20, 700, False, False),
    (96, torch.bfloat16, 90, 400, True, True),
    (64, torch.float16, 128, 129, True, False),
])
def test_single_query_tile_mha(D, dtype, Sq, Skv, causal, top_left):
    """CTAs holding a single query tile (MHA: no second tile for the slot pair)."""
    _run(1, 6, 6, Sq, Skv, D, dtype, causal=causal, top_left=top_left, seed=D + Sq + Skv)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_single_tile_running_max_raises_late(dtype):
    """The exact path (max raise + O rescale) in a CTA with one query tile."""
    from kvboost_b200.ops import prefill_attention
    g = torch.Generator().manual_seed(18)
    B, H, Sq, Skv, D = 1, 2, 90, 1100, 128
    q = _rand((B, H, Sq, D), dtype, g)
    ramp = torch.linspace(0.05, 3.0, Skv).view(1, 1, Skv, 1)
    k = (torch.randn(B, H, Skv, D, generator=g) * ramp).to(dtype)
    v = _rand((B, H, Skv, D), dtype, g)
    k[0, 1, 1000] = (q[0, 1, 7].float() * 0.9).to(dtype)
    k[0, 0, 600] = (q[0, 0, 2].float() * 0.9).to(dtype)
    o, lse = prefill_attention(q.cuda(), k.cuda(), v.cuda(), 1.0 / math.sqrt(D), True)
    torch.cuda.synchronize()
    o_ref, lse_ref = oattn.attention(q.float().numpy(), k.float().numpy(), v.float().numpy(),
                                     1.0 / math.sqrt(D), True, compute_dtype=np.float32)
    assert np.max(np.abs(o.float().cpu().numpy() - o_ref)) <= TOL[dtype]
    assert np.max(np.abs(lse.cpu().numpy() - lse_ref)) <= LSE_TOL


def test_top_left_alignment():
    """SDPA's is_causal alignment (used by the reference's paged path)."""
    _run(1, 4, 2, 40, 200, 128, torch.bfloat16, causal=True, top_left=True, seed=9)


def test_gqa_ratio_8():
    _run(1, 64, 8, 256, 640, 128, torch.bfloat16, seed=5)


def test_rows_without_keys():
    """q_len > kv_len: leading rows see no key -> O = 0, LSE = -inf."""
    _run(1, 2, 1, 200, 72, 64, torch.bfloat16, seed=11)


def test_empty_kv():
    from kvboost_b200.ops import prefill_attention
    q = torch.randn(1, 2, 5, 64, device="cuda", dtype=torch.bfloat16)
    k = torch.randn(1, 2, 0, 64, device="cuda", dtype=torch.bfloat16)
    o, lse = prefill_attention(q, k, k.clone(), 0.125, True)
    torch.cuda.synchronize()
    assert torch.all(o == 0) and torch.all(torch.isneginf(lse))


def test_hf_strided_layout():
    """HF hands [B, S, H, D] storage viewed as [B, H, S, D]; no copies needed."""
    from kvboost_b200.ops import prefill_attention
    g = torch.Generator().manual_seed(21)
    B, Hq, Hkv, Sq, Skv, D = 2, 16, 2, 96, 480, 128
    q = _rand((B, Sq, Hq, D), torch.bfloat16, g)
    k = _rand((B, Skv, Hkv, D), torch.bfloat16, g)
    v = _rand((B, Skv, Hkv, D), torch.bfloat16, g)
    qv, kv_, vv = (t.cuda().transpose(1, 2) for t in (q, k, v))
    o, lse = prefill_attention(qv, kv_, vv, 1.0 / math.sqrt(D), True, out_layout="bshd")
    torch.cuda.synchronize()
    assert o.shape == (B, Sq, Hq, D) and o.is_contiguous()
    _check(o.transpose(1, 2), lse, q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2),
           1.0 / math.sqrt(D), True, torch.bfloat16)


def test_varlen_config4_shape():
    """Varlen fp16 D=96 MHA: suffixes in [16, 512], prefixes multiples of 128 (reduced count)."""
    from kvboost_b200.ops import prefill_attention_varlen
    g = torch.Generator().manual_seed(4)
    n, H, D = 12, 32, 96
    sq = torch.randint(16, 513, (n,), generator=g).tolist()
    pre = (torch.randint(0, 17, (n,), generator=g) * 128).tolist()
    skv = [a + b for a, b in zip(sq, pre)]
    cu_q = np.concatenate([[0], np.cumsum(sq)]).astype(np.int32)
    cu_k = np.concatenate([[0], np.cumsum(skv)]).astype(np.int32)
    q = _rand((int(cu_q[-1]), H, D), torch.float16, g)
    k = _rand((int(cu_k[-1]), H, D), torch.float16, g)
    v = _rand((int(cu_k[-1]), H, D), torch.float16, g)
    o, lse = prefill_attention_varlen(q.cuda(), k.cuda(), v.cuda(),
                                      torch.from_numpy(cu_q).cuda(), torch.from_numpy(cu_k).cuda(),
                                      max(sq), max(skv), 1.0 / math.sqrt(D), True)
    torch.cuda.synchronize()
    o_ref, lse_ref = oattn.attention_varlen(q.float().numpy(), k.float().numpy(), v.float().numpy(),
                                            cu_q, cu_k, 1.0 / math.sqrt(D), True,
                                            compute_dtype=np.float32)
    assert np.max(np.abs(o.float().cpu().numpy() - o_ref)) <= TOL[torch.float16]
    assert np.max(np.abs(lse.cpu().numpy() - lse_ref)) <= LSE_TOL


def test_varlen_config4_full_size():
    """The whole varlen D96 batch as the bench draws it: 64 requests, suffixes U{16..512},
    prefixes 128 * U{0..64} (up to 8192 tokens), 32 heads MHA, fp16; every row of every
    head of every request against the oracle."""
    import bench
    from kvboost_b200.ops import prefill_attention_varlen
    w = bench.make_workload("varlen_d96")
    sq, skv, H, D = w.sq, w.skv, w.Hq, w.D
    assert len(sq) == 64 and max(w.pre) > 4096
    g = torch.Generator().manual_seed(404)
    cu_q = np.concatenate([[0], np.cumsum(sq)]).astype(np.int32)
    cu_k = np.concatenate([[0], np.cumsum(skv)]).astype(np.int32)
    q = _rand((int(cu_q[-1]), H, D), torch.float16, g)
    k = _rand((int(cu_k[-1]), H, D), torch.float16, g)
    v = _rand((int(cu_k[-1]), H, D), torch.float16, g)
    o, lse = prefill_attention_varlen(q.cuda(), k.cuda(), v.cuda(),
                                      torch.from_numpy(cu_q).cuda(), torch.from_numpy(cu_k).cuda(),
                                      max(sq), max(skv), 1.0 / math.sqrt(D), True)
    torch.cuda.synchronize()
    o_ref, lse_ref = oattn.attention_varlen(q.float().numpy(), k.float().numpy(), v.float().numpy(),
                                            cu_q, cu_k, 1.0 / math.sqrt(D), True,
                                            compute_dtype=np.float32)
    assert np.max(np.abs(o.float().cpu().numpy() - o_ref)) <= TOL[torch.float16]
    assert np.max(np.abs(lse.cpu().numpy() - lse_ref)) <= LSE_TOL


def test_golden_vectors_through_gpu(golden_dir):
    """The reference's own outputs (SDPA) on its own inputs, rerun on the GPU path."""
    from kvboost_b200.ops import prefill_attention
    d = np.load(os.path.join(golden_dir, "attention.npz"))
    for case in ("reuse_gqa4_bf16", "reuse_mha_d96_f16", "square_d64_bf16",
                 "suffix_longer_than_prefix_bf16"):
        B, Hq, Hkv, Sq, Skv, D, causal, dt = d[case + "/meta"].tolist()
        dtype = torch.bfloat16 if dt == 1 else torch.float16
        t = {n: torch.from_numpy(d[f"{case}/{n}"].astype(np.int16)).view(dtype) for n in "qkvo"}
        o, _ = prefill_attention(t["q"].cuda(), t["k"].cuda(), t["v"].cuda(), 1.0 / math.sqrt(D),
                                 bool(causal))
        torch.cuda.synchronize()
        err = (o.float().cpu() - t["o"].float()).abs().max().item()
        assert err <= TOL[dtype], f"{case}: {err}"


def test_reference_compat_op():
    """kvboost._flash_attn_cuda.flash_attn_fwd drop-in: same signature and outputs."""
    from kvboost_b200 import _flash_attn_cuda as fac
    g = torch.Generator().manual_seed(42)
    for dtype, (B, H, S, D) in ((torch.float16, (2, 8, 128, 128)), (torch.bfloat16, (1, 4, 64, 64))):
        Q, K, V = (_rand((B, H, S, D), dtype, g) for _ in range(3))
        O, L = fac.flash_attn_fwd(Q.cuda(), K.cuda(), V.cuda(), 1.0 / math.sqrt(D), True)
        torch.cuda.synchronize()
        assert O.shape == Q.shape and O.dtype == dtype and L.shape == (B, H, S)
        assert L.dtype == torch.float32
        _check(O, L, Q, K, V, 1.0 / math.sqrt(D), True, dtype)


def test_cabi_direct_call():
    """Call kvb_flash_attn_fwd through ctypes with raw pointers, as an FFI user would."""
    from kvboost_b200 import _lib
    lib = _lib.load()
    g = torch.Generator().manual_seed(1)
    B, H, S, D = 1, 2, 300, 96
    Q, K, V = (_rand((B, H, S, D), torch.bfloat16, g).cuda() for _ in range(3))
    O = torch.empty_like(Q)
    L = torch.empty(B, H, S, device="cuda", dtype=torch.float32)
    rc = lib.kvb_flash_attn_fwd(Q.data_ptr(), K.data_ptr(), V.data_ptr(), O.data_ptr(),
                                L.data_ptr(), B, H, S, D, _lib.KVB_DTYPE_BF16,
                                1.0 / math.sqrt(D), 1, torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib.kvb_last_error()
    torch.cuda.synchronize()
    _check(O, L, Q.cpu(), K.cpu(), V.cpu(), 1.0 / math.sqrt(D), True, torch.bfloat16)


def test_repeatable_bitwise():
    """Same inputs, same launch -> identical bits (no nondeterministic reductions)."""
    from kvboost_b200.ops import prefill_attention
    g = torch.Generator().manual_seed(8)
    q = _rand((2, 8, 300, 128), torch.bfloat16, g).cuda()
    k = _rand((2, 2, 900, 128), torch.bfloat16, g).cuda()
    v = _rand((2, 2, 900, 128), torch.bfloat16, g).cuda()
    o1, l1 = prefill_attention(q, k, v)
    o2, l2 = prefill_attention(q, k, v)
    torch.cuda.synchronize()
    assert torch.equal(o1, o2) and torch.equal(l1, l2)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_running_max_raises_late(dtype):
    """Scores that grow along the keys force the exact path (max raise + O rescale)."""
    from kvboost_b200.ops import prefill_attention
    g = torch.Generator().manual_seed(17)
    B, H, Sq, Skv, D = 1, 4, 130, 1000, 128
    q = _rand((B, H, Sq, D), dtype, g)
    ramp = torch.linspace(0.05, 3.0, Skv).view(1, 1, Skv, 1)
    k = (torch.randn(B, H, Skv, D, generator=g) * ramp).to(dtype)
    v = _rand((B, H, Skv, D), dtype, g)
    # one very strong key late in the sequence for query row 3
    k[0, 0, 900] = (q[0, 0, 3].float() * 0.9).to(dtype)
    o, lse = prefill_attention(q.cuda(), k.cuda(), v.cuda(), 1.0 / math.sqrt(D), True)
    torch.cuda.synchronize()
    _check(o, lse, q, k, v, 1.0 / math.sqrt(D), True, dtype)


def _varlen_case(sq, pre, H, D, dtype, causal, seed):
    from kvboost_b200.ops import prefill_attention_varlen
    g = torch.Generator().manual_seed(seed)
    skv = [a + b for a, b in zip(sq, pre)]
    cu_q = np.concatenate([[0], np.cumsum(sq)]).astype(np.int32)
    cu_k = np.concatenate([[0], np.cumsum(skv)]).astype(np.int32)
    q = _rand((int(cu_q[-1]), H, D), dtype, g)
    k = _rand((int(cu_k[-1]), H, D), dtype, g)
    v = _rand((int(cu_k[-1]), H, D), dtype, g)
    o, lse = prefill_attention_varlen(q.cuda(), k.cuda(), v.cuda(),
                                      torch.from_numpy(cu_q).cuda(), torch.from_numpy(cu_k).cuda(),
                                      max(sq), max(skv), 1.0 / math.sqrt(D), causal)
    torch.cuda.synchronize()
    o_ref, lse_ref = oattn.attention_varlen(q.float().numpy(), k.float().numpy(), v.float().numpy(),
                                            cu_q, cu_k, 1.0 / math.sqrt(D), causal,
                                            compute_dtype=np.float32)
    assert np.max(np.abs(o.float().cpu().numpy() - o_ref)) <= TOL[dtype]
    assert np.max(np.abs(lse.cpu().numpy() - lse_ref)) <= LSE_TOL


@pytest.mark.parametrize("D,dtype", [(96, torch.float16), (128, torch.bfloat16), (64, torch.float16)])
@pytest.mark.parametrize("causal", [True, False])
def test_varlen_lone_tiles_split_keys(D, dtype, causal):
    """Varlen MHA sequences whose last CTA holds one query tile over many key tiles:
    the CTA's two slots take the two halves of the key range and slot 0 merges them
    (single-tile sequences, the third tile of three, short key ranges that stay whole)."""
    sq = [16, 128, 1, 300, 100, 64, 40]
    pre = [2048, 1024, 3000, 1280, 256, 0, 640]
    _varlen_case(sq, pre, 4, D, dtype, causal, seed=D + int(causal))


@pytest.mark.parametrize("causal,top_left", [(True, False), (False, False), (True, True)])
def test_dense_odd_tiles_split_keys(causal, top_left):
    """Dense MHA with an odd query-tile count, through the prefill kernel: the last
    tile's CTA splits its keys over both slots."""
    from kvboost_b200.ops import prefill_attention
    g = torch.Generator().manual_seed(31)
    B, H, Sq, Skv, D = 2, 3, 300, 2100, 128
    q = _rand((B, H, Sq, D), torch.bfloat16, g)
    k = _rand((B, H, Skv, D), torch.bfloat16, g)
    v = _rand((B, H, Skv, D), torch.bfloat16, g)
    o, lse = prefill_attention(q.cuda(), k.cuda(), v.cuda(), 1.0 / math.sqrt(D), causal,
                               top_left=top_left, kernel="prefill")
    torch.cuda.synchronize()
    _check(o, lse, q, k, v, 1.0 / math.sqrt(D), causal, torch.bfloat16, top_left)
