"""The model and tokenizer that the engine golden fixtures were made with.

The decoder is the Qwen2.5-3B architecture (36 layers, hidden 2048, 16 query /
2 KV heads, head dim 128, SiLU-gated MLP 11008, RMSNorm eps 1e-6, RoPE theta
1e6, vocabulary 151936, tied embeddings) with random weights: every matrix
N(0, 0.02) drawn in float32 on the CPU from its own generator (seeded by the
model seed and the matrix's index in ``named_parameters``) and rounded to
bfloat16, norms 1, biases 0.  Drawing on the CPU makes the weights the same on
any host with this torch build; the fixture
keeps a checksum of a few tensors so a host whose draw differs is reported as
such instead of as a token mismatch.

The tokenizer maps a prompt of space-separated integers to those token ids,
so text prompts reach both engines unchanged (the reference's engine needs a
tokenizer object; its ``encode`` / ``decode`` / ``eos_token_id`` /
``pad_token_id`` are all it uses).
"""

from __future__ import annotations

import torch

ARCH = dict(vocab_size=151936, hidden_size=2048, intermediate_size=11008,
            num_hidden_layers=36, num_attention_heads=16, num_key_value_heads=2,
            max_position_embeddings=32768, rms_norm_eps=1e-6, rope_theta=1e6,
            tie_word_embeddings=True)

EOS_ID = 151645
PAD_ID = 151643


class IntTokenizer:
    """Space-separated integer ids in, the same ids out."""

    eos_token_id = EOS_ID
    pad_token_id = PAD_ID
    eos_token = "<eos>"
    pad_token = "<pad>"

    def encode(self, text, add_special_tokens=True):
        return [int(t) for t in text.split()]

    def decode(self, ids, skip_special_tokens=True):
        return " ".join(str(int(i)) for i in ids)


def text(ids) -> str:
    return " ".join(str(int(i)) for i in ids)


def build_model(seed: int = 0):
    """The random-init decoder on the CPU in bfloat16 (about 6 GB)."""
    from transformers import Qwen2Config, Qwen2ForCausalLM
    from transformers.initialization import no_init_weights
    cfg = Qwen2Config(**ARCH, attn_implementation="sdpa")
    old = torch.get_default_dtype()
    torch.set_default_dtype(torch.bfloat16)
    try:
        with torch.device("cpu"), no_init_weights():   # every parameter is set below
            m = Qwen2ForCausalLM(cfg)
    finally:
        torch.set_default_dtype(old)
    from concurrent.futures import ThreadPoolExecutor
    params = list(m.named_parameters())

    def fill(i):
        name, p = params[i]
        with torch.no_grad():
            if p.dim() >= 2:   # its own generator: the draw does not depend on threading
                g = torch.Generator().manual_seed(seed * 100_003 + i)
                p.copy_(torch.empty(p.shape, dtype=torch.float32).normal_(0.0, 0.02, generator=g))
            else:   # RMSNorm weights 1, projection biases 0 (set, not left to HF's init)
                p.fill_(1.0 if name.endswith("norm.weight") else 0.0)

    with ThreadPoolExecutor(8) as ex:
        list(ex.map(fill, range(len(params))))
    return m.eval()


def weight_checksum(model) -> list:
    """Float64 sums over slices of a few weight matrices (exact for bfloat16 values)."""
    sd = dict(model.named_parameters())
    names = ["model.embed_tokens.weight", "model.layers.0.self_attn.q_proj.weight",
             "model.layers.17.mlp.gate_proj.weight", "model.layers.35.mlp.down_proj.weight"]
    return [float(sd[n].detach()[:64].double().sum()) for n in names]


def prompts():
    """The fixture's token ids: a 3072-token shared prefix (24 chunks of 128) and
    1024-token suffixes, uniform over the vocabulary, seeded."""
    import numpy as np
    g = np.random.default_rng(2026)
    V = ARCH["vocab_size"]
    # keep clear of the two special ids so a prompt never contains them
    draw = lambda n: [int(t) for t in g.integers(0, PAD_ID, n)]
    prefix = draw(3072)
    singles = [prefix + draw(1024) for _ in range(2)]
    batch = [prefix + draw(1024) for _ in range(8)]
    ragged = [prefix + draw(n) for n in (1024, 700, 333)]
    assert V > PAD_ID
    return prefix, singles, batch, ragged
