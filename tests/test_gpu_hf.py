"""GPU: HF model attention routed through the patched registry to the sm_100a kernel.

A small random-init Qwen2 (the reference's model family) runs a full prefill
and a reuse prefill over cached ``past_key_values`` (HF's bottom-right bool
mask path).  Logits are compared with the same model on stock SDPA, and the
number of kernel calls is counted to prove the routing.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _need_gpu():
    if not torch.cuda.is_available() or torch.cuda.get_device_capability()[0] != 10:
        pytest.skip("needs an sm_100 (B200) device")


def _model(head_dim=64, layers=2):
    from transformers import Qwen2Config, Qwen2ForCausalLM
    heads, kv_heads = 8, 2
    cfg = Qwen2Config(vocab_size=1024, hidden_size=heads * head_dim, intermediate_size=1024,
                      num_hidden_layers=layers, num_attention_heads=heads,
                      num_key_value_heads=kv_heads, max_position_embeddings=4096,
                      rms_norm_eps=1e-6, rope_theta=1e6, attn_implementation="sdpa")
    torch.manual_seed(0)
    m = Qwen2ForCausalLM(cfg)
    with torch.no_grad():
        for p in m.parameters():
            p.normal_(0, 0.02)
    return m.to("cuda", torch.bfloat16).eval()


class _Counter:
    def __init__(self, monkeypatch):
        from kvboost_b200 import ops
        self.n = 0
        orig = ops.prefill_attention

        def wrapped(*a, **k):
            self.n += 1
            return orig(*a, **k)
        monkeypatch.setattr(ops, "prefill_attention", wrapped)


def _close(a, b):
    a, b = a.float(), b.float()
    cos = torch.nn.functional.cosine_similarity(a.flatten(), b.flatten(), dim=0).item()
    return cos, (a - b).abs().max().item(), b.abs().max().item()


@pytest.mark.parametrize("head_dim", [64, 128])
def test_full_and_reuse_prefill_match_sdpa(monkeypatch, head_dim):
    _need_gpu()
    from transformers import DynamicCache
    from kvboost_b200.flash_attn_ext import install_flash_attention, uninstall_flash_attention

    model = _model(head_dim)
    g = torch.Generator().manual_seed(1)
    prefix = torch.randint(0, 1024, (1, 384), generator=g).cuda()
    suffix = torch.randint(0, 1024, (1, 200), generator=g).cuda()

    with torch.no_grad():
        ref_full = model(torch.cat([prefix, suffix], 1)).logits
        pkv = DynamicCache()
        model(prefix, past_key_values=pkv, use_cache=True)
        ref_reuse = model(suffix, past_key_values=pkv, use_cache=True).logits

    counter = _Counter(monkeypatch)
    assert install_flash_attention(model) == 2
    with torch.no_grad():
        out_full = model(torch.cat([prefix, suffix], 1)).logits
        pkv = DynamicCache()
        model(prefix, past_key_values=pkv, use_cache=True)
        out_reuse = model(suffix, past_key_values=pkv, use_cache=True).logits
    assert counter.n == 3 * 2, "every layer of every forward must run on the kernel"
    uninstall_flash_attention(model)

    for out, ref in ((out_full, ref_full), (out_reuse, ref_reuse)):
        cos, err, scale = _close(out, ref)
        assert cos > 0.999 and err <= 2e-2 * max(1.0, scale), (cos, err, scale)
    # greedy next tokens agree at every position where the reference is not a near-tie
    top2 = ref_reuse.float().topk(2, dim=-1).values
    decisive = (top2[..., 0] - top2[..., 1]) > 1e-2
    agree = out_reuse.argmax(-1) == ref_reuse.argmax(-1)
    assert bool(agree[decisive].all())
