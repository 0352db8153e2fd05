"""The engine's host logic against KVBoost's own ``InferenceEngine``, on the CPU.

Both engines run one small random-init Qwen2 on the CPU with HuggingFace's own
SDPA attention (the sm_100a hook is uninstalled here; the GPU replay of the
reference's decisions on the Qwen2.5-3B architecture is
``tests/test_gpu_engine_golden.py``).  With the same arithmetic on both sides,
every result must be identical: generated ids, ``cached_tokens``,
``prompt_tokens``, ``kv_reuse_ratio``, and the prefix-chained keys of the cached
chunks -- through ``warm``, ``generate`` with recompute "none" and "selective",
``cacheable_prefix_len``, the prefix-cache mode, ``generate_batch`` with ragged
suffixes (right-padded, no mask) and ``generate_many``
(``src/kvboost/engine.py:207-407``, ``:415-507``, ``:592-753``, ``:919-979``,
``src/kvboost/batch.py``).

The reference package comes from ``KVBOOST_REF_SRC`` or ``baseline/_ref``;
without either the test skips.
"""

import copy
import os
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def ref_engine_cls():
    for p in (os.environ.get("KVBOOST_REF_SRC"), os.path.join(ROOT, "baseline", "_ref")):
        if p and os.path.isfile(os.path.join(p, "kvboost", "engine.py")):
            sys.path.insert(0, p)
            try:
                from kvboost.engine import GenerationMode, InferenceEngine, RecomputeStrategy
            finally:
                sys.path.remove(p)
            return InferenceEngine, RecomputeStrategy, GenerationMode
    pytest.skip("the reference package is not available (KVBOOST_REF_SRC or baseline/_ref)")


class _Tok:
    eos_token_id = 997
    pad_token_id = 998
    eos_token = "<eos>"
    pad_token = "<pad>"

    def encode(self, text, add_special_tokens=True):
        return [int(t) for t in text.split()]

    def decode(self, ids, skip_special_tokens=True):
        return " ".join(str(int(i)) for i in ids)


def _text(ids):
    return " ".join(str(int(i)) for i in ids)


def _model():
    from transformers import Qwen2Config, Qwen2ForCausalLM
    cfg = Qwen2Config(vocab_size=1000, hidden_size=256, intermediate_size=512,
                      num_hidden_layers=3, num_attention_heads=8, num_key_value_heads=2,
                      max_position_embeddings=4096, rms_norm_eps=1e-6, rope_theta=1e6,
                      tie_word_embeddings=True, attn_implementation="sdpa")
    torch.manual_seed(0)
    m = Qwen2ForCausalLM(cfg)
    with torch.no_grad():
        for _, p in m.named_parameters():
            if p.dim() >= 2:
                p.normal_(0, 0.02)
    return m.to(torch.bfloat16).eval()


def test_engine_decisions_equal_reference_engine(ref_engine_cls):
    from kvboost_b200.engine import GenerationMode, KVBoost
    from kvboost_b200.flash_attn_ext import uninstall_flash_attention
    InferenceEngine, RefStrategy, RefMode = ref_engine_cls
    model = _model()
    ref = InferenceEngine(copy.deepcopy(model), _Tok(), max_cache_bytes=1 << 30,
                          recompute_strategy=RefStrategy.NONE, device="cpu")
    ours = KVBoost(copy.deepcopy(model), _Tok(), recompute_strategy="none", device="cpu")
    uninstall_flash_attention(ours.model)       # HF's own SDPA on the CPU, as the reference

    g = torch.Generator().manual_seed(7)
    draw = lambda n: torch.randint(0, 990, (n,), generator=g).tolist()
    prefix = draw(384)
    other = draw(300)

    def both(fn):
        r = fn(ref, RefStrategy, RefMode)
        o = fn(ours, type(ours.recompute_strategy), GenerationMode)
        r = r if isinstance(r, list) else [r]
        o = o if isinstance(o, list) else [o]
        assert [x.output_text for x in o] == [x.output_text for x in r]
        assert [x.cached_tokens for x in o] == [x.cached_tokens for x in r]
        assert [x.prompt_tokens for x in o] == [x.prompt_tokens for x in r]
        assert [x.kv_reuse_ratio for x in o] == pytest.approx([x.kv_reuse_ratio for x in r],
                                                              abs=0)
        assert [x.generated_tokens for x in o] == [x.generated_tokens for x in r]
        return o

    w_ref, w_ours = ref.warm(_text(prefix)), ours.warm(_text(prefix))
    assert (w_ours.chunks_stored, w_ours.chunk_boundary_aligned) == \
        (w_ref.chunks_stored, w_ref.chunk_boundary_aligned) == (3, True)

    def set_strategy(e, S, name):
        e.recompute_strategy = S(name)

    p1, p2, p3 = prefix + draw(90), prefix + draw(150), prefix + draw(200)
    both(lambda e, S, M: e.generate(_text(p1), max_new_tokens=10))
    both(lambda e, S, M: (set_strategy(e, S, "selective"),
                          e.generate(_text(p2), max_new_tokens=10))[1])
    both(lambda e, S, M: (set_strategy(e, S, "none"),
                          e.generate(_text(p3), max_new_tokens=6, cacheable_prefix_len=450))[1])
    # p3's chunks past token 450 were not stored: its repeat reuses only up to there
    both(lambda e, S, M: e.generate(_text(p3), max_new_tokens=6))
    p4 = p1 + draw(40)
    both(lambda e, S, M: e.generate(_text(p4), max_new_tokens=6, mode=M.PREFIX_CACHE))
    ragged = [prefix + draw(n) for n in (100, 37, 64)]
    both(lambda e, S, M: e.generate_batch([_text(p) for p in ragged], max_new_tokens=7))
    many = [prefix + draw(20), other + draw(10), prefix + draw(45), draw(64)]
    both(lambda e, S, M: e.generate_many([_text(p) for p in many], max_new_tokens=5))
    assert sorted(ours.store._chunks.keys()) == sorted(ref.cache_manager._hot.keys())
