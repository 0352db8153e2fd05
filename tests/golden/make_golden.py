"""Generate golden vectors by running the KVBoost reference itself on the CPU.

Run from the repository root in a checkout that has the reference source
(``KVBOOST_REF_SRC`` points at its ``src`` directory)::

    KVBOOST_REF_SRC=<reference checkout>/src python tests/golden/make_golden.py

Writes ``tests/golden/*.npz`` / ``*.json``.  The fixtures are small (well
under 2 MB together) and are what ``tests/test_oracle_golden.py`` pins the
oracle against; the GPU parity tests then compare the CUDA path to the
pinned oracle.  Nothing at test time or on a GPU host needs the reference.

Reference entry points exercised (file:line in the KVBoost project):

* ``_kvboost_flash_attn`` CPU path -> SDPA (``flash_attn_ext.py:68-103``),
  called exactly as a reuse prefill reaches it: GQA expanded with
  ``repeat_interleave`` and HF's bottom-right boolean mask.
* ``quantize_kv`` / ``dequantize_kv`` int8 (``kv_quantize.py:73-109,194-222``).
* ``BlockAllocator`` / ``ChunkBlockMapper`` / ``append_kv_to_blocks`` /
  ``read_kv`` / ``paged_attention_fwd`` (``cpu_paged/``).
* ``chained_hash`` / ``content_hash_from_tokens`` (``models.py:131-148``) and
  ``ChunkRegistry`` fixed split (``chunk_registry.py:98-110``).
* ``quantize_kv`` on bfloat16 / float16 model K/V (the quantise-on-store
  fixtures) and ``CacheBlendRecompute._deviation_recompute``
  (``cacheblend.py:103-197``) with a preset full-context K/V.

``python tests/golden/make_golden.py blocks`` rewrites only the last two;
``engine`` writes ``engine.json`` (the reference engine's greedy choices on the
random-init Qwen2.5-3B-architecture decoder, ``engine_model.py``).
"""

from __future__ import annotations

import json
import math
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _ref():
    src = os.environ.get("KVBOOST_REF_SRC")
    if not src or not os.path.isdir(src):
        raise SystemExit("set KVBOOST_REF_SRC to the reference's src/ directory")
    sys.path.insert(0, src)
    import kvboost.flash_attn_ext as fae            # noqa: E402
    import kvboost.kv_quantize as kq                 # noqa: E402
    import kvboost.models as models                  # noqa: E402
    import kvboost.chunk_registry as cr              # noqa: E402
    from kvboost.cpu_paged import block_allocator, chunk_to_blocks, paged_attn_cpu  # noqa: E402
    return fae, kq, models, cr, block_allocator, chunk_to_blocks, paged_attn_cpu


def _store(t: torch.Tensor) -> np.ndarray:
    """float32 as is; 16-bit floats as their raw uint16 bit patterns (exact, half the size)."""
    if t.dtype == torch.float32:
        return t.numpy()
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def attention_cases(fae):
    """Each case: inputs (float32 exact values), dtype, and the reference output."""
    cases = [
        # name, B, Hq, Hkv, Sq, Skv, D, dtype, causal
        ("square_causal_f32", 1, 2, 2, 100, 100, 64, torch.float32, True),
        ("square_noncausal_f32", 2, 2, 2, 16, 16, 64, torch.float32, False),
        ("seq1_f32", 1, 4, 4, 1, 1, 64, torch.float32, True),
        ("cross_noncausal_f32", 1, 4, 4, 8, 128, 64, torch.float32, False),
        ("reuse_gqa4_f32", 1, 8, 2, 24, 88, 128, torch.float32, True),
        ("reuse_gqa4_bf16", 1, 8, 2, 40, 168, 128, torch.bfloat16, True),
        ("reuse_mha_d96_f16", 1, 2, 2, 33, 97, 96, torch.float16, True),
        ("square_d64_bf16", 2, 4, 4, 64, 64, 64, torch.bfloat16, True),
        ("suffix_longer_than_prefix_bf16", 1, 4, 1, 130, 200, 64, torch.bfloat16, True),
    ]
    out = {}
    for i, (name, B, Hq, Hkv, Sq, Skv, D, dt, causal) in enumerate(cases):
        g = torch.Generator().manual_seed(1000 + i)
        q = torch.randn(B, Hq, Sq, D, generator=g).to(dt)
        k = torch.randn(B, Hkv, Skv, D, generator=g).to(dt)
        v = torch.randn(B, Hkv, Skv, D, generator=g).to(dt)
        scale = 1.0 / math.sqrt(D)
        rep = Hq // Hkv
        ke = k.repeat_interleave(rep, dim=1)
        ve = v.repeat_interleave(rep, dim=1)
        if causal and Sq != Skv:
            mask = torch.ones(Sq, Skv, dtype=torch.bool).tril(Skv - Sq)
            o = fae._kvboost_flash_attn(q, ke, ve, scale, True, attn_mask=mask)
        else:
            o = fae._kvboost_flash_attn(q, ke, ve, scale, causal)
        out[name + "/q"] = _store(q)
        out[name + "/k"] = _store(k)
        out[name + "/v"] = _store(v)
        out[name + "/o"] = _store(o)
        out[name + "/meta"] = np.array([B, Hq, Hkv, Sq, Skv, D, int(causal),
                                        {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}[dt]],
                                       dtype=np.int64)
    return out


def quant_cases(kq):
    out = {}
    g = torch.Generator().manual_seed(7)
    for i, (H, S, D) in enumerate([(2, 128, 64), (2, 128, 128), (1, 100, 96)]):
        key = torch.randn(1, H, S, D, generator=g).to(torch.float16)
        val = (torch.randn(1, H, S, D, generator=g) * 3).to(torch.float16)
        if i == 1:
            key[0, 0, 5] = 0  # an all-zero row exercises the clamp(min=1e-8)
        qkv = kq.quantize_kv(((key, val),), bits=8)
        layer = qkv.layers[0]
        deq = kq.dequantize_kv(qkv)[0]
        p = f"q{i}/"
        out[p + "key"] = key.numpy()
        out[p + "val"] = val.numpy()
        out[p + "key_q"] = layer.key_q.numpy()
        out[p + "key_scale"] = layer.key_scale.numpy()
        out[p + "val_q"] = layer.val_q.numpy()
        out[p + "val_scale"] = layer.val_scale.numpy()
        out[p + "key_deq"] = deq[0].numpy()
        out[p + "val_deq"] = deq[1].numpy()
    return out


def quant_bf16_cases(kq):
    """``quantize_kv`` on the dtypes a model hands it: bfloat16 (the arithmetic then
    runs in bfloat16 and only the scales are cast to float16) and float16, with
    all-zero K rows / V columns and magnitudes whose float16 scales are subnormal."""
    out = {}
    g = torch.Generator().manual_seed(8)
    cases = [(torch.bfloat16, 2, 128, 128, 1.0), (torch.bfloat16, 1, 100, 96, 1e-3),
             (torch.bfloat16, 2, 128, 64, 300.0), (torch.float16, 2, 128, 128, 1e-3),
             (torch.bfloat16, 1, 16, 128, 1.0)]
    for i, (dt, H, S, D, mag) in enumerate(cases):
        key = (torch.randn(1, H, S, D, generator=g) * mag).to(dt)
        val = (torch.randn(1, H, S, D, generator=g) * mag * 2).to(dt)
        key[0, 0, 3] = 0
        val[0, H - 1, :, 5] = 0
        qkv = kq.quantize_kv(((key, val),), bits=8)
        layer = qkv.layers[0]
        deq = kq.dequantize_kv(qkv)[0]
        p = f"b{i}/"
        out[p + "dtype"] = np.array(1 if dt == torch.bfloat16 else 2)
        out[p + "key"] = _store(key)
        out[p + "val"] = _store(val)
        out[p + "key_q"] = layer.key_q.numpy()
        out[p + "key_scale"] = _store(layer.key_scale)
        out[p + "val_q"] = layer.val_q.numpy()
        out[p + "val_scale"] = _store(layer.val_scale)
        out[p + "key_deq"] = _store(deq[0])
        out[p + "val_deq"] = _store(deq[1])
    return out


class _PresetModel:
    """Stands in for the model in ``CacheBlendRecompute._deviation_recompute``: its
    forward returns a preset full-context K/V (the legacy tuple form)."""

    def __init__(self, fresh):
        self.fresh = fresh
        self._p = torch.zeros(1)

    def parameters(self):
        return iter([self._p])

    def __call__(self, input_ids=None, position_ids=None, use_cache=True, **kw):
        from types import SimpleNamespace
        assert input_ids.shape[1] == self.fresh[0][0].shape[2]
        return SimpleNamespace(past_key_values=self.fresh)


def cacheblend_cases():
    """``CacheBlendRecompute._deviation_recompute`` (``cacheblend.py:103-197``) with the
    full-context forward replaced by a preset K/V, so the deviation / top-k / patch
    steps run exactly as shipped.  Per-token perturbation magnitudes are spread so
    the selected set does not hinge on rounding."""
    from kvboost.cacheblend import CacheBlendRecompute
    out = {}
    # name: (dtype, layers, heads, S, D, ratio, min_dev, kind)
    cases = [("spread_f32", torch.float32, 3, 2, 40, 64, 0.15, 0.01, "spread"),
             ("none_above_f32", torch.float32, 2, 2, 24, 64, 0.15, 0.01, "tiny"),
             ("few_above_f32", torch.float32, 2, 1, 50, 128, 0.3, 0.05, "few"),
             ("gapped_bf16", torch.bfloat16, 3, 2, 64, 128, 0.15, 0.01, "gapped"),
             ("zero_row_f32", torch.float32, 2, 2, 20, 96, 0.2, 0.01, "zero")]
    for ci, (name, dt, L, H, S, D, ratio, min_dev, kind) in enumerate(cases):
        g = torch.Generator().manual_seed(500 + ci)
        perm = torch.randperm(S, generator=g)
        if kind == "spread":
            mag = 0.05 + 0.9 * perm.float() / S
        elif kind == "tiny":
            mag = torch.full((S,), 1e-4)
        elif kind == "few":
            mag = torch.full((S,), 0.05)
            mag[perm[:5]] = 1.0 + perm[:5].float() / S
        elif kind == "gapped":
            mag = 0.05 + 0.45 * perm.float() / S
            k = max(1, int(S * ratio))
            mag[perm[:k]] = 2.0 + 0.5 * torch.arange(k).float()
        else:
            mag = 0.05 + 0.9 * perm.float() / S
        cached, fresh = [], []
        for l in range(L):
            ck = torch.randn(1, H, S, D, generator=g)
            cv = torch.randn(1, H, S, D, generator=g)
            fk = ck + mag.view(1, 1, S, 1) * torch.randn(1, H, S, D, generator=g)
            fv = cv + torch.randn(1, H, S, D, generator=g)
            if kind == "zero" and l == 1:
                ck[:, :, 4] = 0
            cached.append((ck.to(dt), cv.to(dt)))
            fresh.append((fk.to(dt), fv.to(dt)))
        blend = CacheBlendRecompute(recompute_ratio=ratio, min_deviation=min_dev, device="cpu")
        patched = blend._deviation_recompute(list(range(S)), tuple(cached), S,
                                             _PresetModel(tuple(fresh)))
        # The reference's output, reduced to what it decided: the patched positions
        # (every other position, and every V, is checked to be an exact copy).
        pk = torch.stack([k for k, _ in patched])
        pv = torch.stack([v for _, v in patched])
        ck = torch.stack([k for k, _ in cached])
        cv = torch.stack([v for _, v in cached])
        fk = torch.stack([k for k, _ in fresh])
        fv = torch.stack([v for _, v in fresh])
        pos = (pk != ck).flatten(0, 2).any(dim=0).any(dim=-1).nonzero().flatten()
        keep = torch.ones(S, dtype=torch.bool)
        keep[pos] = False
        assert torch.equal(pk[:, :, :, pos], fk[:, :, :, pos])
        assert torch.equal(pv[:, :, :, pos], fv[:, :, :, pos])
        assert torch.equal(pk[:, :, :, keep], ck[:, :, :, keep])
        assert torch.equal(pv[:, :, :, keep], cv[:, :, :, keep])
        p = f"{name}/"
        out[p + "meta"] = np.array([L, H, S, D, 1 if dt == torch.bfloat16 else 0])
        out[p + "ratio"] = np.array(ratio)
        out[p + "min_dev"] = np.array(min_dev)
        out[p + "cached_k"] = np.stack([_store(k[0]) for k, _ in cached])
        out[p + "fresh_k"] = np.stack([_store(k[0]) for k, _ in fresh])
        out[p + "patched_positions"] = pos.numpy().astype(np.int32)
    return out


def paged_cases(block_allocator, chunk_to_blocks, paged_attn_cpu, models):
    """Scripted allocator/mapper history plus gathers and paged attention."""
    BA = block_allocator.BlockAllocator
    CBM = chunk_to_blocks.ChunkBlockMapper
    tables = {}
    a = BA(num_layers=1, num_heads=2, head_dim=8, num_blocks=40, block_size=16, dtype=torch.float32)
    m = CBM(a)

    def chunk(cid, length, seed):
        g = torch.Generator().manual_seed(seed)
        kv = ((torch.randn(1, 2, length, 8, generator=g), torch.randn(1, 2, length, 8, generator=g)),)
        return models.CachedChunk(chunk_id=cid, text="", token_ids=list(range(length)),
                                  past_key_values=kv, position_start=0, position_end=length,
                                  prefix_hash=cid, content_hash=cid + "c")

    c1, c2, c3 = chunk("c1", 128, 1), chunk("c2", 100, 2), chunk("c3", 40, 3)
    tables["load_c1"] = m.load_chunk(c1)
    tables["load_c2"] = m.load_chunk(c2)
    tables["reload_c1"] = m.load_chunk(c1)
    asm = models.AssembledPrompt(full_token_ids=[], cached_past_kv=None, cached_length=268,
                                 live_token_ids=[], live_position_ids=[], chunk_boundaries=[],
                                 cache_hit_ratio=0.0)
    tbl, clen = m.build_block_table(asm, [c1, c2, c3])
    tables["build_c1_c2_c3"] = tbl
    tables["build_cached_len"] = clen
    m.on_evict("c2")
    tables["after_evict_alloc3"] = a.allocate(3)
    shared = a.fork(tables["load_c1"][:2])
    tables["cow_first"] = a.ensure_writable(shared[0])
    new_tbl, new_off = paged_attn_cpu.append_kv_to_blocks(
        a, 0, list(tables["load_c1"]), 128, torch.randn(2, 20, 8), torch.randn(2, 20, 8))
    tables["append_20_after_128"] = new_tbl
    tables["append_new_offset"] = new_off
    tables["free_blocks_end"] = a.free_blocks
    tables["free_list_end"] = list(a._free)

    arrays = {}
    # read_kv over a permuted table of a random pool
    b2 = BA(num_layers=1, num_heads=3, head_dim=16, num_blocks=24, block_size=16, dtype=torch.float32)
    g = torch.Generator().manual_seed(11)
    b2.pools[0].copy_(torch.randn(b2.pools[0].shape, generator=g))
    table = torch.randperm(24, generator=g)[:7].tolist()
    k, v = b2.read_kv(0, table, 100)
    arrays["read/pool"] = b2.pools[0].numpy()
    arrays["read/table"] = np.array(table, dtype=np.int64)
    arrays["read/k"] = k.numpy()
    arrays["read/v"] = v.numpy()
    # paged_attention_fwd: GQA 6 q heads over 3 kv heads, batch of 2 + an empty history
    q = torch.randn(3, 6, 5, 16, generator=g)
    out = paged_attn_cpu.paged_attention_fwd(q, b2, [table, table[:3], []], [100, 37, 0], 0,
                                             causal=True)
    arrays["pattn/q"] = q.numpy()
    arrays["pattn/o"] = out.numpy()
    arrays["pattn/seq_lens"] = np.array([100, 37, 0], dtype=np.int64)
    arrays["pattn/table_b1_len"] = np.array([3], dtype=np.int64)
    return tables, arrays


def hash_cases(models, cr):
    rng = np.random.default_rng(5)
    out = {"content": [], "chained": [], "splits": []}
    for n in (0, 1, 5, 128, 300):
        ids = rng.integers(0, 151936, size=n).tolist()
        out["content"].append({"ids": ids, "hash": models.content_hash_from_tokens(ids)})
    parent = None
    ids = rng.integers(0, 151936, size=4096).tolist()
    reg = cr.ChunkRegistry(chunk_size=128)
    for s, e, sl in reg.split(ids):
        h = models.chained_hash(sl, parent)
        out["chained"].append({"start": s, "end": e, "parent": parent, "hash": h})
        parent = h
    out["chained_ids"] = ids
    for n in (31, 32, 100, 159, 160, 161, 300, 4096):
        out["splits"].append({"n": n, "spans": [(s, e) for s, e, _ in reg.split(list(range(n)))]})
    return out


def main():
    fae, kq, models, cr, ba, c2b, pac = _ref()
    np.savez_compressed(os.path.join(HERE, "attention.npz"), **attention_cases(fae))
    np.savez_compressed(os.path.join(HERE, "kv_quant.npz"), **quant_cases(kq))
    tables, arrays = paged_cases(ba, c2b, pac, models)
    np.savez_compressed(os.path.join(HERE, "paged.npz"), **arrays)
    with open(os.path.join(HERE, "paged_tables.json"), "w") as f:
        json.dump(tables, f, indent=1)
    with open(os.path.join(HERE, "hashes.json"), "w") as f:
        json.dump(hash_cases(models, cr), f)
    print("golden fixtures written to", HERE)




def assembly_cases(models, cr):
    """Reference KVCacheManager + PromptAssembler on toy chunks: what gets reused."""
    import kvboost.cache_manager as cm
    import kvboost.prompt_assembler as pa
    cache = cm.KVCacheManager(max_cache_bytes=1 << 30, device="cpu")
    reg = cr.ChunkRegistry(chunk_size=128)
    asm = pa.PromptAssembler(cache_manager=cache, chunk_registry=reg, mode=pa.AssemblyMode.CHUNK_REUSE)
    rng = np.random.default_rng(21)
    base = rng.integers(0, 50000, size=1000).tolist()

    def put(ids):
        parent, pos = None, 0
        for s, e, sl in reg.split(ids):
            h = models.chained_hash(sl, parent)
            kv = ((torch.zeros(1, 1, len(sl), 4), torch.zeros(1, 1, len(sl), 4)),)
            cache.store(models.CachedChunk(chunk_id=h, text="", token_ids=sl, past_key_values=kv,
                                           position_start=s, position_end=e, prefix_hash=h,
                                           content_hash=models.content_hash_from_tokens(sl)))
            parent = h

    put(base[:640])                     # 5 chunks cached
    other = rng.integers(0, 50000, size=300).tolist()
    put(other)                          # an unrelated document (2 chunks + a 44-token tail)
    prompts = {
        "full_prefix_plus_tail": base[:640] + rng.integers(0, 50000, size=77).tolist(),
        "partial_prefix": base[:300] + rng.integers(0, 50000, size=200).tolist(),
        "diverges_in_chunk_3": base[:256] + [7] + base[257:700],
        "no_match": rng.integers(0, 50000, size=400).tolist(),
        "other_doc_tail": other[:300] + [1, 2, 3],
        "short": base[:20],
    }
    out = {}
    for name, ids in prompts.items():
        a = asm.assemble(ids, chunk_splits=reg.split(ids))
        out[name] = {"ids": ids, "cached_length": a.cached_length,
                     "boundaries": [list(b) for b in a.chunk_boundaries],
                     "live": len(a.live_token_ids)}
    import kvboost.batch as kb
    groups = [[base[:512] + [1] * 40, base[:512] + [2] * 40], [base[:300], base[:200] + [5] * 100],
              [base[:128] * 2, base[:256]]]
    out["common_prefix"] = [{"ids": g, "common": kb.find_common_chunk_prefix(g, 128)} for g in groups]
    # group_by_prefix (batch.py:86-104): prompts keyed by their first three chunks
    tail = lambda n: rng.integers(0, 50000, size=n).tolist()
    many = [base[:400] + tail(30), other[:200], base[:384] + tail(5), base[:383] + tail(90),
            [], base[:500], other[:200] + [9], tail(100)]
    out["group_by_prefix"] = {"ids": many, "groups": list(
        kb.group_by_prefix([""] * len(many), many, 128).values())}
    out["stored"] = {"base": base[:640], "other": other}
    return out


def main_assembly():
    fae, kq, models, cr, ba, c2b, pac = _ref()
    with open(os.path.join(HERE, "assembly.json"), "w") as f:
        json.dump(assembly_cases(models, cr), f)
    print("assembly fixture written")


class _TopK:
    """Records the top candidates of every greedy choice the reference engine makes
    (``InferenceEngine._sample``, ``engine.py:982-988``), in call order."""

    K = 8

    def __init__(self, engine_cls):
        self.cls = engine_cls
        self.orig = engine_cls.__dict__["_sample"].__func__
        self.calls = []

    def __enter__(self):
        orig, calls, k = self.orig, self.calls, self.K

        def recording(logits, temperature, do_sample):
            top = logits.float().reshape(-1).topk(k)
            chosen = orig(logits, temperature, do_sample)
            calls.append((top.indices.tolist(), top.values.tolist(), int(chosen)))
            return chosen
        self.cls._sample = staticmethod(recording)
        return self

    def __exit__(self, *exc):
        self.cls._sample = staticmethod(self.orig)

    def take(self):
        out, self.calls[:] = list(self.calls), []
        return out


def engine_cases():
    """The reference's ``InferenceEngine`` in CHUNK_KV_REUSE mode on the CPU
    (``engine.py:207-365``, ``:415-507``, ``:592-753``) on the random-init
    Qwen2.5-3B-architecture decoder of ``engine_model.py``, one engine, one
    scripted sequence of calls:

    1. ``warm`` of a 3072-token prefix (24 chunks of 128);
    2. ``generate`` of prefix + 1024 new tokens, ``recompute_strategy`` "none",
       32 new tokens;
    3. ``generate`` of another 1024-token suffix with "selective" (23 seams),
       32 new tokens;
    4. ``generate_batch`` of 8 prompts of 3072 + 1024 tokens (the TTFT workload's
       shape), 16 new tokens;
    5. ``generate_batch`` of 3 prompts with ragged suffixes (1024 / 700 / 333
       tokens; the reference right-pads them and passes no mask), 16 new tokens.

    Stored per call: the generated ids, ``cached_tokens``, ``prompt_tokens``,
    ``kv_reuse_ratio``, the top-8 candidates (ids and logits) of every greedy
    choice; at the end the prefix-chained keys of every cached chunk."""
    sys.path.insert(0, HERE)
    import engine_model as em
    from kvboost.engine import InferenceEngine, RecomputeStrategy
    model = em.build_model(0)
    tok = em.IntTokenizer()
    eng = InferenceEngine(model, tok, max_cache_bytes=64 << 30,
                          recompute_strategy=RecomputeStrategy.NONE, device="cpu")
    prefix, singles, batch, ragged = em.prompts()
    out = {"weights": em.weight_checksum(model), "calls": []}
    with _TopK(InferenceEngine) as rec:
        w = eng.warm(em.text(prefix))
        out["warm"] = {"chunks_stored": w.chunks_stored, "token_count": w.token_count,
                       "aligned": w.chunk_boundary_aligned}

        def one(kind, strategy, prompts, new):
            eng.recompute_strategy = RecomputeStrategy(strategy)
            if kind == "generate":
                rs = [eng.generate(em.text(prompts[0]), max_new_tokens=new)]
            else:
                rs = eng.generate_batch([em.text(p) for p in prompts], max_new_tokens=new)
            calls = rec.take()
            B = len(rs)
            gen = [[int(t) for t in r.output_text.split()] for r in rs]
            assert all(len(g) == new for g in gen), "an end-of-sequence id was generated"
            # call order: single prompt = steps; batch = step-major over the prompts
            tops = [[calls[s * B + b] for s in range(new)] for b in range(B)]
            for b in range(B):    # (the top-k order of tied logits is arbitrary)
                assert [t[2] for t in tops[b]] == gen[b]
            out["calls"].append({
                "kind": kind, "strategy": strategy, "new_tokens": new,
                "prompts": [list(p) for p in prompts],
                "generated": gen,
                "cached_tokens": [r.cached_tokens for r in rs],
                "prompt_tokens": [r.prompt_tokens for r in rs],
                "kv_reuse_ratio": [r.kv_reuse_ratio for r in rs],
                "top_ids": [[t[0] for t in tb] for tb in tops],
                "top_logits": [[t[1] for t in tb] for tb in tops]})
            print(kind, strategy, "done", [g[:4] for g in gen], flush=True)

        one("generate", "none", singles[:1], 32)
        one("generate", "selective", singles[1:], 32)
        one("batch", "none", batch, 16)
        one("batch", "none", ragged, 16)
    out["chunk_keys"] = sorted(eng.cache_manager._hot.keys())
    return out


def main_engine():
    _ref()
    with open(os.path.join(HERE, "engine.json"), "w") as f:
        json.dump(engine_cases(), f)
    print("engine fixture written")


def main_blocks():
    """The quantise-on-store and CacheBlend fixtures."""
    fae, kq, models, cr, ba, c2b, pac = _ref()
    np.savez_compressed(os.path.join(HERE, "kv_quant_model_dtypes.npz"), **quant_bf16_cases(kq))
    np.savez_compressed(os.path.join(HERE, "cacheblend.npz"), **cacheblend_cases())
    print("quantise-on-store and CacheBlend fixtures written")


if __name__ == "__main__":
    # with arguments, only the named groups: core, assembly, blocks, engine
    # (engine runs a 3B-parameter model on the CPU: about ten minutes)
    groups = sys.argv[1:] or ["core", "assembly", "blocks", "engine"]
    if "core" in groups:
        main()
    if "assembly" in groups:
        main_assembly()
    if "blocks" in groups:
        main_blocks()
    if "engine" in groups:
        main_engine()
