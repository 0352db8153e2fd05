"""GPU: ``PagedEngine`` (the ``CPUPagedEngine`` drop-in) end to end.

* Greedy tokens equal ``KVBoost`` in CHUNK_KV_REUSE mode on the same cache
  contents (recompute "none", so both attend to the same prefix K/V; the paged
  engine reads it from the block pool, ``KVBoost`` from its dense cache).
* The pool's bookkeeping equals the oracle's replay of the reference engine's
  steps (``cpu_paged/cpu_engine.py:150-319``): chunks loaded through the mapper
  (forked when already loaded), the prompt's new tokens appended for every layer
  at the same slots, one slot per decode step, then the sequence's own blocks
  freed -- free list, reference counts and the sequence's block table all
  identical, over a first prompt, the same prompt again (now fully cached: the
  last token is re-fed and appended after the prefix) and a third prompt.
* The K/V the pool holds for the prompt's new tokens are the model's own.
"""

import copy

import pytest
import torch

from oracle import paged as opaged

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _gpu():
    if not torch.cuda.is_available() or torch.cuda.get_device_capability()[0] != 10:
        pytest.skip("needs an sm_100 (B200) device")
    from kvboost_b200 import ops
    ops.read_status(torch.device("cuda"))
    yield
    assert ops.read_status(torch.device("cuda")) == 0


def _model():
    from transformers import Qwen2Config, Qwen2ForCausalLM
    cfg = Qwen2Config(vocab_size=512, hidden_size=512, intermediate_size=1024,
                      num_hidden_layers=2, num_attention_heads=8, num_key_value_heads=2,
                      max_position_embeddings=4096, rms_norm_eps=1e-6, rope_theta=1e6,
                      tie_word_embeddings=False, attn_implementation="sdpa")
    torch.manual_seed(0)
    m = Qwen2ForCausalLM(cfg)
    with torch.no_grad():
        for name, p in m.named_parameters():
            p.normal_(0, 1.0 if "lm_head" in name else 0.02)  # decisive greedy choices
    return m.to("cuda", torch.bfloat16).eval()


class _Replay:
    """The reference engine's pool bookkeeping on the oracle's allocator."""

    def __init__(self, num_blocks, layers, bs=16):
        self.a = opaged.AllocatorModel(num_blocks)
        self.m = opaged.MapperModel(self.a, bs)
        self.layers, self.bs = layers, bs

    def generate(self, chunks, cached_len, n_live, new_tokens):
        table = self.m.build_block_table(chunks) if cached_len else []
        slot = cached_len
        n_app = n_live if n_live else 1              # a fully cached prompt re-feeds one token
        for _ in range(self.layers):                 # every layer writes the same slots
            t, _ = opaged.append_slots(self.a, table, slot, n_app, self.bs)
            table = t
        slot += n_app
        for _ in range(new_tokens - 1):              # one slot per decode step, all layers
            for _ in range(self.layers):
                table, _ = opaged.append_slots(self.a, table, slot, 1, self.bs)
            slot += 1
        own = table[(cached_len + self.bs - 1) // self.bs:]
        if own:
            self.a.free(own)
        return table


def test_paged_engine_tokens_and_block_tables():
    from kvboost_b200.engine import KVBoost, chained_hash, fixed_split
    from kvboost_b200.paged_engine import CPUPagedEngine, PagedEngine
    assert CPUPagedEngine is PagedEngine
    m = _model()
    m2 = copy.deepcopy(m)       # copied before either engine patches its modules
    paged = PagedEngine(m, None, recompute_strategy="none", num_blocks=256)
    dense = KVBoost(m2, None, recompute_strategy="none")
    g = torch.Generator().manual_seed(11)
    pre = torch.randint(0, 512, (384,), generator=g).tolist()
    p1 = pre + torch.randint(0, 512, (100,), generator=g).tolist()
    p3 = pre + torch.randint(0, 512, (57,), generator=g).tolist()
    for e in (paged, dense):
        assert e.warm(pre).chunks_stored == 3
    replay = _Replay(256, 2)
    keys = []
    parent = None
    for _, _, ids in fixed_split(pre):
        parent = chained_hash(ids, parent)
        keys.append(parent)

    r = paged.generate(p1, max_new_tokens=12)
    d = dense.generate(p1, max_new_tokens=12)
    assert r.cached_tokens == d.cached_tokens == 384 and r.generated_tokens == 12
    assert r.generated_ids == d.generated_ids
    a = torch.tensor(r.first_token_logits)
    b = torch.tensor(d.first_token_logits)
    assert torch.nn.functional.cosine_similarity(a, b, dim=0) > 0.999
    want = replay.generate([(k, 128) for k in keys], 384, 100, 12)
    assert paged.last_block_table == want
    assert paged.allocator._free == replay.a.free_list
    assert paged.allocator._ref_count == replay.a.ref

    # p1's 100-token tail is now a stored chunk: the repeat is fully cached
    tail_key = chained_hash(p1[384:], keys[-1])
    r2 = paged.generate(p1, max_new_tokens=5)
    assert r2.cached_tokens == 484 and r2.generated_tokens == 5
    want = replay.generate([(k, 128) for k in keys] + [(tail_key, 100)], 484, 0, 5)
    assert paged.last_block_table == want
    assert paged.allocator._free == replay.a.free_list
    assert paged.allocator._ref_count == replay.a.ref

    r3 = paged.generate(p3, max_new_tokens=7)
    d3 = dense.generate(p3, max_new_tokens=7)
    assert r3.generated_ids == d3.generated_ids
    want = replay.generate([(k, 128) for k in keys], 384, 57, 7)
    assert paged.last_block_table == want
    assert paged.allocator._free == replay.a.free_list
    st = paged.paged_stats()
    assert st["loaded_chunks"] == 4 and st["blocks_used_by_chunks"] == 3 * 8 + 7


def test_paged_engine_pool_holds_the_models_kv():
    """After a generate, the prompt's new tokens' K/V in the pool (their blocks are
    freed but not cleared) equal the model's K/V for those positions."""
    from kvboost_b200.paged_engine import PagedEngine
    m = _model()
    eng = PagedEngine(m, None, recompute_strategy="none", num_blocks=64)
    g = torch.Generator().manual_seed(5)
    pre = torch.randint(0, 512, (256,), generator=g).tolist()
    prompt = pre + torch.randint(0, 512, (40,), generator=g).tolist()
    eng.warm(pre)
    eng.generate(prompt, max_new_tokens=1)
    table = eng.last_block_table
    keys, values, cached, _ = eng._assemble(pre)
    assert cached == 256
    x = torch.tensor([prompt[256:]], device="cuda")
    pos = torch.arange(256, 296, device="cuda")[None]
    out = eng._forward(x, pos, eng._cache_from(keys, values))
    for layer, (k, v) in enumerate(eng._layers(out.past_key_values)):
        pk, pv = eng.allocator.read_kv(layer, table, 296)
        assert torch.equal(pk[:, 256:], k[0, :, 256:].to(pk.dtype))
        assert torch.equal(pv[:, 256:], v[0, :, 256:].to(pv.dtype))
