"""Host-side tests of the ``kvboost.flash_attn_ext`` drop-in (CPU only).

Mirrors the reference's ``tests/test_flash_attn.py`` (tier detection, CPU
numerics of the dispatch, install/uninstall on a toy module) and adds what
the reference never checked: that the patch really routes HF's attention
registry, and that masks are classified exactly.
"""

import math

import pytest
import torch
import torch.nn as nn
import torch.nn.functional as F

from kvboost_b200.flash_attn_ext import (
    _kvboost_flash_attn,
    classify_mask,
    flash_attention_available,
    get_tier,
    install_flash_attention,
    uninstall_flash_attention,
)


def make_qkv(B=2, H=4, S=64, D=64, dtype=torch.float32):
    torch.manual_seed(42)
    return (torch.randn(B, H, S, D, dtype=dtype), torch.randn(B, H, S, D, dtype=dtype),
            torch.randn(B, H, S, D, dtype=dtype))


class TestTierDetection:
    def test_get_tier_returns_string(self):
        assert get_tier() in ("kvboost_cuda", "torch_flash", "vanilla")

    def test_tier_is_kvboost_cuda_when_library_loads(self):
        assert get_tier() == "kvboost_cuda"
        assert flash_attention_available()


class TestCpuDispatch:
    """CPU tensors keep the reference's vanilla SDPA behaviour (its CPU tier)."""

    @pytest.mark.parametrize("causal", [True, False])
    @pytest.mark.parametrize("S", [1, 16, 100])
    def test_output_close_to_sdpa(self, causal, S):
        Q, K, V = make_qkv(B=1, H=2, S=S)
        out = _kvboost_flash_attn(Q, K, V, 0.125, causal)
        ref = F.scaled_dot_product_attention(Q, K, V, scale=0.125, is_causal=causal)
        assert torch.allclose(out, ref, atol=1e-5)


class TestMaskClassification:
    def test_bottom_right_bool(self):
        m = torch.ones(24, 88, dtype=torch.bool).tril(64)[None, None].expand(2, 1, 24, 88)
        assert classify_mask(m, 24, 88) is True

    def test_additive_float(self):
        keep = torch.ones(5, 9, dtype=torch.bool).tril(4)
        m = torch.zeros(1, 1, 5, 9).masked_fill(~keep, torch.finfo(torch.float32).min)
        assert classify_mask(m, 5, 9) is True

    def test_all_visible_decode_row(self):
        # for a single query the bottom-right mask *is* all-visible: either answer is exact
        m = torch.ones(3, 1, 1, 40, dtype=torch.bool)
        assert classify_mask(m, 1, 40) in (True, False)

    def test_all_visible_block(self):
        m = torch.ones(2, 1, 5, 40, dtype=torch.bool)
        assert classify_mask(m, 5, 40) is False

    def test_square_causal(self):
        m = torch.ones(8, 8, dtype=torch.bool).tril()
        assert classify_mask(m, 8, 8) is True

    def test_none(self):
        assert classify_mask(None, 4, 4) is None

    def test_padding_mask_rejected(self):
        m = torch.ones(2, 1, 6, 10, dtype=torch.bool).tril(4)
        m[1, :, :, :3] = False  # left padding in the second sequence
        with pytest.raises(NotImplementedError):
            classify_mask(m, 6, 10)

    def test_top_left_mask_rejected(self):
        m = torch.ones(4, 10, dtype=torch.bool).tril()
        with pytest.raises(NotImplementedError):
            classify_mask(m, 4, 10)

    def test_cache_follows_in_place_edits(self):
        m = torch.ones(1, 1, 3, 5, dtype=torch.bool).tril(2)
        assert classify_mask(m, 3, 5) is True
        m[0, 0, 0, 4] = True  # in-place edit bumps the version counter
        with pytest.raises(NotImplementedError):
            classify_mask(m, 3, 5)


class _ToyAttention(nn.Module):
    def __init__(self, embed_dim=64, num_heads=4):
        super().__init__()
        self.num_heads = num_heads
        self.head_dim = embed_dim // num_heads
        self.q_proj = nn.Linear(embed_dim, embed_dim, bias=False)
        self.k_proj = nn.Linear(embed_dim, embed_dim, bias=False)
        self.v_proj = nn.Linear(embed_dim, embed_dim, bias=False)
        self.out_proj = nn.Linear(embed_dim, embed_dim, bias=False)

    def forward(self, x):
        B, S, E = x.shape
        H, D = self.num_heads, self.head_dim
        Q = self.q_proj(x).view(B, S, H, D).transpose(1, 2)
        K = self.k_proj(x).view(B, S, H, D).transpose(1, 2)
        V = self.v_proj(x).view(B, S, H, D).transpose(1, 2)
        attn = F.scaled_dot_product_attention(Q, K, V, scale=1.0 / math.sqrt(D), is_causal=True)
        return self.out_proj(attn.transpose(1, 2).reshape(B, S, E))


class _ToyTransformer(nn.Module):
    def __init__(self):
        super().__init__()
        self.attention = _ToyAttention()

    def forward(self, x):
        return self.attention(x)


class TestModelPatching:
    def test_install_returns_count(self):
        assert install_flash_attention(_ToyTransformer()) == 1

    def test_install_and_uninstall_roundtrip(self):
        model = _ToyTransformer()
        torch.manual_seed(0)
        x = torch.randn(1, 8, 64)
        before = model(x).detach()
        install_flash_attention(model)
        assert torch.allclose(before, model(x).detach(), atol=1e-5)
        assert uninstall_flash_attention(model) == 1
        assert torch.allclose(before, model(x).detach(), atol=1e-5)

    def test_double_install_is_idempotent(self):
        model = _ToyTransformer()
        assert install_flash_attention(model) == 1
        assert install_flash_attention(model) == 0

    def test_uninstall_on_unpatched_model(self):
        assert uninstall_flash_attention(_ToyTransformer()) == 0


def _tiny_qwen2(device="cpu", dtype=torch.float32, layers=2):
    from transformers import Qwen2Config, Qwen2ForCausalLM
    cfg = Qwen2Config(vocab_size=128, hidden_size=256, intermediate_size=512,
                      num_hidden_layers=layers, num_attention_heads=4, num_key_value_heads=2,
                      max_position_embeddings=512, rms_norm_eps=1e-6, rope_theta=1e6,
                      attn_implementation="sdpa")
    torch.manual_seed(0)
    return Qwen2ForCausalLM(cfg).to(device=device, dtype=dtype).eval()


class TestRegistryRouting:
    """The patched forward must reach kvboost_attention_forward through HF's registry."""

    def test_patch_counts_hf_layers(self):
        model = _tiny_qwen2(layers=3)
        assert install_flash_attention(model) == 3
        assert uninstall_flash_attention(model) == 3

    def test_patched_forward_routes_to_kvboost(self):
        model = _tiny_qwen2()
        ids = torch.randint(0, 128, (1, 12))
        with torch.no_grad():
            ref = model(ids).logits
        install_flash_attention(model)
        # CPU tensors reaching the registry function prove the routing: it only runs on CUDA.
        with pytest.raises(RuntimeError, match="CUDA"):
            with torch.no_grad():
                model(ids)
        uninstall_flash_attention(model)
        with torch.no_grad():
            assert torch.allclose(model(ids).logits, ref)

    def test_registry_restored_after_forward(self):
        from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS
        before = dict(ALL_ATTENTION_FUNCTIONS._local_mapping)
        model = _tiny_qwen2()
        install_flash_attention(model)
        with pytest.raises(RuntimeError):
            with torch.no_grad():
                model(torch.randint(0, 128, (1, 4)))
        assert dict(ALL_ATTENTION_FUNCTIONS._local_mapping) == before
