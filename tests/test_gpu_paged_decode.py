"""GPU: paged attention over a 16-bit block pool (the reference's paged engine
pool) -- ``paged_attention_fwd`` against the oracle, and the
``install_paged_attention`` protocol decoding a small Qwen2 to the same greedy
tokens as stock SDPA with a dense cache."""

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


def _pool(dtype, lens, Hkv=3, D=64, seed=0):
    from kvboost_b200.paged import DeviceBlockAllocator
    g = torch.Generator().manual_seed(seed)
    a = DeviceBlockAllocator(1, Hkv, D, 64, dtype=dtype)
    tables, hist = [], []
    for n in lens:
        k = torch.randn(Hkv, n, D, generator=g).to(dtype)
        v = torch.randn(Hkv, n, D, generator=g).to(dtype)
        tb, _ = a.append_kv(0, [], 0, k.cuda(), v.cuda())
        tables.append(tb)
        hist.append((k.float().numpy(), v.float().numpy()))
    return a, tables, hist


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("Sq", [1, 5])
@pytest.mark.parametrize("top_left", [True, False])
def test_paged_attention_fwd_matches_oracle(dtype, Sq, top_left):
    from kvboost_b200.paged import paged_attention_fwd
    lens = [100, 37, 0]
    a, tables, hist = _pool(dtype, lens, seed=Sq + 3 * top_left)
    g = torch.Generator().manual_seed(9)
    q = torch.randn(3, 6, Sq, 64, generator=g).to(dtype)
    o = paged_attention_fwd(q.cuda(), a, tables, lens, 0, causal=True, top_left=top_left)
    torch.cuda.synchronize()
    qf = q.float().numpy()
    if top_left:
        ref = oattn.paged_attention_topleft(qf, [h[0] for h in hist], [h[1] for h in hist],
                                            causal=True, compute_dtype=np.float32)
    else:
        ref = np.zeros_like(qf)
        for b, n in enumerate(lens):
            if n:
                ref[b:b + 1], _ = oattn.attention(qf[b:b + 1], hist[b][0][None], hist[b][1][None],
                                                  1.0 / math.sqrt(64), Sq > 1,
                                                  compute_dtype=np.float32)
    assert np.abs(o.float().cpu().numpy() - ref).max() <= TOL[dtype]


def _tiny_qwen():
    from transformers import Qwen2Config, Qwen2ForCausalLM
    cfg = Qwen2Config(vocab_size=512, hidden_size=512, intermediate_size=1024,
                      num_hidden_layers=2, num_attention_heads=8, num_key_value_heads=2,
                      max_position_embeddings=2048, rms_norm_eps=1e-6, rope_theta=1e6,
                      tie_word_embeddings=False, attn_implementation="sdpa")
    torch.manual_seed(0)
    m = Qwen2ForCausalLM(cfg)
    with torch.no_grad():
        for name, p in m.named_parameters():
            p.normal_(0, 1.0 if "lm_head" in name else 0.02)
    return m.to("cuda", torch.bfloat16).eval()


def _greedy_dense(model, prompt, n):
    ids = torch.tensor([prompt], device="cuda")
    out = model(input_ids=ids, use_cache=True)
    cache, toks = out.past_key_values, [int(out.logits[0, -1].argmax())]
    for i in range(n - 1):
        out = model(input_ids=torch.tensor([[toks[-1]]], device="cuda"), past_key_values=cache,
                    position_ids=torch.tensor([[len(prompt) + i]], device="cuda"), use_cache=True)
        cache = out.past_key_values
        toks.append(int(out.logits[0, -1].argmax()))
    return toks


@pytest.mark.parametrize("top_left", [False, True])
def test_install_paged_attention_decodes_like_sdpa(top_left):
    from kvboost_b200.flash_attn_ext import install_paged_attention, uninstall_paged_attention
    from kvboost_b200.paged import DeviceBlockAllocator
    model = _tiny_qwen()
    g = torch.Generator().manual_seed(4)
    prompt = torch.randint(0, 512, (45,), generator=g).tolist()
    with torch.no_grad():
        want = _greedy_dense(model, prompt, 10)
        state = {"allocator": DeviceBlockAllocator(2, 2, 64, 32, dtype=torch.bfloat16),
                 "block_table": [], "_write_slot": 0, "top_left": top_left}
        assert install_paged_attention(model, state) == 2
        ids = torch.tensor([prompt], device="cuda")
        out = model(input_ids=ids, position_ids=torch.arange(len(prompt), device="cuda")[None],
                    use_cache=False)
        state["_write_slot"] += len(prompt)
        got = [int(out.logits[0, -1].argmax())]
        for _ in range(9):
            slot = state["_write_slot"]
            out = model(input_ids=torch.tensor([[got[-1]]], device="cuda"),
                        position_ids=torch.tensor([[slot]], device="cuda"), use_cache=False)
            state["_write_slot"] += 1
            got.append(int(out.logits[0, -1].argmax()))
        assert uninstall_paged_attention(model) == 2
    assert len(state["block_table"]) == (45 + 9 + 15) // 16
    # the prompt forward has q == kv (both masks coincide) and decode steps have one
    # query, so either alignment must decode exactly like the dense cache
    assert got == want
