"""KVBoost engine with a device-resident chunk store (chunk KV reuse on B200).

Mirrors the CHUNK_KV_REUSE path of KVBoost's ``InferenceEngine``
(``src/kvboost/engine.py``) with the same public calls -- ``warm``,
``generate``, ``generate_batch``, ``reset_cache``, ``GenerationResult``,
``WarmResult`` -- and the same host logic:

* prompts split into fixed 128-token chunks, tails shorter than 32 tokens
  dropped (``chunk_registry.py:98-110``);
* chunks keyed by the prefix-chained SHA-256 hash (``models.py:137-148``);
* each chunk encoded on its own at its absolute positions, with no
  preceding context (``engine.py:829-850``);
* reuse = the longest run of cached chunks from position 0, found by chained
  lookups (``cache_manager.py:358-393``, ``prompt_assembler.py:99-176``);
* seam repair with ``recompute_strategy="selective"``: the last
  ``recompute_overlap`` tokens before each seam re-encoded over the prefix
  (``selective_recompute.py:99-184``);
* suffix prefill with the cached K/V as ``past_key_values`` at positions
  ``cached_len..`` then greedy / sampled decode (``engine.py:634-753``);
  batched prompts share a common chunk prefix broadcast over the batch
  (``engine.py:235-365``, ``batch.py``).

What changes is where things live and run: chunk K/V stay in GPU memory
(no per-request host->device copy of the reused prefix, which dominates the
reference's TTFT), and every attention call of every forward -- chunk
encoding, seam recompute, suffix prefill, decode -- runs on the sm_100a
prefill kernels through ``install_flash_attention``.
"""

from __future__ import annotations

import enum
import hashlib
import logging
import struct
import time
from collections import OrderedDict
from dataclasses import dataclass
from typing import Dict, List, Optional, Sequence, Tuple, Union

import torch

from .flash_attn_ext import install_flash_attention

log = logging.getLogger(__name__)

TokenIds = List[int]


class GenerationMode(str, enum.Enum):
    BASELINE = "baseline"
    PREFIX_CACHE = "prefix_cache"
    CHUNK_KV_REUSE = "chunk_kv_reuse"


class RecomputeStrategy(str, enum.Enum):
    SELECTIVE = "selective"
    CACHEBLEND = "cacheblend"
    NONE = "none"


@dataclass
class GenerationResult:
    """Same fields as ``engine.py:61-73``."""
    mode: str
    prompt: str
    output_text: str
    generated_tokens: int
    ttft_ms: float
    total_ms: float
    tokens_per_sec: float
    kv_reuse_ratio: float
    prompt_tokens: int
    cached_tokens: int
    first_token_logits: Optional[object] = None
    generated_ids: Optional[List[int]] = None


@dataclass
class WarmResult:
    """Same fields as ``models.py:115-126``."""
    chunks_stored: int
    token_count: int
    chunk_size: int
    chunk_boundary_aligned: bool
    partial_tail_tokens: int
    alignment_warning: Optional[str] = None


# ── chunk keys and split (bit-identical to the reference) ─────────────────────

def _token_bytes(ids: Sequence[int]) -> bytes:
    return struct.pack("<%dI" % len(ids), *[int(t) & 0xFFFFFFFF for t in ids])


def chained_hash(token_ids: Sequence[int], parent_hash: Optional[str] = None) -> str:
    """``models.py:137-148``: SHA-256 of (parent or "root") + little-endian int32 tokens."""
    return hashlib.sha256((parent_hash or "root").encode("utf-8") + _token_bytes(token_ids)).hexdigest()


def content_hash_from_tokens(token_ids: Sequence[int]) -> str:
    """``models.py:131-134``."""
    return hashlib.sha256(_token_bytes(token_ids)).hexdigest()


def fixed_split(token_ids: Sequence[int], chunk_size: int = 128,
                min_chunk_tokens: int = 32) -> List[Tuple[int, int, List[int]]]:
    """``ChunkRegistry._fixed_split`` (``chunk_registry.py:98-110``)."""
    out, pos, n = [], 0, len(token_ids)
    while pos < n:
        end = min(pos + chunk_size, n)
        if end - pos >= min_chunk_tokens:
            out.append((pos, end, list(token_ids[pos:end])))
        pos = end
    return out


def find_common_chunk_prefix(all_token_ids: List[TokenIds], chunk_size: int) -> int:
    """Tokens shared by every prompt, in whole chunks (same result as ``batch.py:31-54``):
    the longest common prefix of all prompts rounded down to a multiple of
    ``chunk_size``; a lone prompt shares all of itself."""
    if len(all_token_ids) < 2:
        return len(all_token_ids[0]) if all_token_ids else 0
    first = all_token_ids[0]
    agree = min(len(ids) for ids in all_token_ids)
    for ids in all_token_ids[1:]:
        agree = next((i for i, (a, b) in enumerate(zip(first[:agree], ids)) if a != b), agree)
    return agree - agree % chunk_size


def group_by_prefix(token_ids_list: List[TokenIds], chunk_size: int,
                    n_prefix_chunks: int = 3) -> Dict[str, List[int]]:
    """Prompt indices grouped by the content hash of their first ``n_prefix_chunks``
    chunks, groups in order of first appearance (``batch.py:86-104``)."""
    groups: Dict[str, List[int]] = {}
    for i, ids in enumerate(token_ids_list):
        head = ids[:n_prefix_chunks * chunk_size]
        groups.setdefault(content_hash_from_tokens(head) if head else "empty", []).append(i)
    return groups


# ── device-resident chunk store ───────────────────────────────────────────────

@dataclass
class DeviceChunk:
    chunk_id: str
    token_ids: List[int]
    position_start: int
    position_end: int
    keys: Optional[torch.Tensor]     # [layers, kv_heads, len, head_dim] on the GPU
    values: Optional[torch.Tensor]   # (None for a chunk held in the int8 block pool)
    hits: int = 0
    block_ids: Optional[List[int]] = None   # its blocks in the engine's int8 pool
    pool_bytes: int = 0

    @property
    def length(self) -> int:
        return self.position_end - self.position_start

    def nbytes(self) -> int:
        if self.block_ids is not None:
            return self.pool_bytes
        return self.keys.numel() * self.keys.element_size() * 2


class DeviceChunkStore:
    """Byte-budgeted LRU store of chunk K/V in GPU memory, keyed by prefix hash.

    Plays the role of ``KVCacheManager``'s hot tier (``cache_manager.py:141-292``)
    without the CPU round trip: ``get`` / ``store`` / ``lookup`` chained by parent
    hash, LRU eviction when the byte budget is exceeded, hit/miss stats.
    """

    def __init__(self, max_bytes: int, on_evict=None):
        self.max_bytes = int(max_bytes)
        self._chunks: "OrderedDict[str, DeviceChunk]" = OrderedDict()
        self.bytes = 0
        self.hits = self.misses = self.evictions = 0
        self.on_evict = on_evict

    def get(self, chunk_id: str) -> Optional[DeviceChunk]:
        c = self._chunks.get(chunk_id)
        if c is not None:
            self._chunks.move_to_end(chunk_id)
        return c

    def lookup(self, token_ids: Sequence[int], parent_hash: Optional[str]) -> Optional[DeviceChunk]:
        c = self.get(chained_hash(token_ids, parent_hash))
        if c is None:
            self.misses += 1
        else:
            self.hits += 1
            c.hits += 1
        return c

    def make_room(self, size: int) -> bool:
        """Evict least-recently-used chunks until ``size`` more bytes fit."""
        if size > self.max_bytes:
            return False
        while self.bytes + size > self.max_bytes and self._chunks:
            _, old = self._chunks.popitem(last=False)
            self.bytes -= old.nbytes()
            self.evictions += 1
            if self.on_evict is not None:
                self.on_evict(old)
        return True

    def store(self, chunk: DeviceChunk) -> bool:
        size = chunk.nbytes()
        if not self.make_room(size):
            return False
        self._chunks[chunk.chunk_id] = chunk
        self.bytes += size
        return True

    def clear(self) -> None:
        if self.on_evict is not None:
            for c in self._chunks.values():
                self.on_evict(c)
        self._chunks.clear()
        self.bytes = 0
        self.hits = self.misses = self.evictions = 0

    def __len__(self) -> int:
        return len(self._chunks)

    def stats(self) -> Dict[str, float]:
        total = self.hits + self.misses
        return {"chunks": len(self._chunks), "bytes": self.bytes, "max_bytes": self.max_bytes,
                "hits": self.hits, "misses": self.misses, "evictions": self.evictions,
                "hit_rate": self.hits / total if total else 0.0}


def plan_reuse(token_ids: Sequence[int], store: DeviceChunkStore, chunk_size: int = 128,
               min_chunk_tokens: int = 32):
    """Longest contiguous run of cached chunks from position 0.

    Chained lookups as ``find_matching_chunks`` (``cache_manager.py:358-393``),
    then the contiguous-from-0 stitching of ``_chunk_reuse``
    (``prompt_assembler.py:99-176``).  Returns ``(chunks, cached_len,
    boundaries)``.
    """
    matches = []
    parent = None
    for start, end, ids in fixed_split(token_ids, chunk_size, min_chunk_tokens):
        c = store.lookup(ids, parent)
        if c is not None:
            matches.append((start, c))
            parent = chained_hash(ids, parent)
        else:
            parent = None
    chunks, boundaries, covered = [], [], 0
    for start, c in sorted(matches, key=lambda x: x[0]):
        if start != covered:
            break
        chunks.append(c)
        boundaries.append((start, start + c.length))
        covered = start + c.length
    return chunks, covered, boundaries


# ── engine ────────────────────────────────────────────────────────────────────

class KVBoost:
    """Chunk-level KV reuse over a HuggingFace causal LM, on the sm_100a kernels."""

    def __init__(self, model, tokenizer=None, *, max_cache_bytes: int = 16 << 30,
                 chunk_size: int = 128, min_chunk_tokens: int = 32,
                 recompute_overlap: int = 16,
                 recompute_strategy: Union[str, RecomputeStrategy] = RecomputeStrategy.SELECTIVE,
                 recompute_ratio: float = 0.15, kv_cache_bits: int = 16,
                 int8_pool_blocks: Optional[int] = None, device: str = "cuda"):
        """``kv_cache_bits=8`` keeps cached chunks KIVI-int8 in a device block pool,
        quantised on store by one kernel per chunk (the reference's
        ``kv_cache_bits=8`` store, ``cache_manager.py:164-175``), dequantised on
        assembly by the paged gather kernel; the pool has ``int8_pool_blocks``
        16-token blocks (default: what ``max_cache_bytes`` buys, at most 8192)."""
        if kv_cache_bits not in (8, 16):
            raise ValueError("kv_cache_bits must be 16 or 8")
        self.device = torch.device(device)
        self.model = model.to(self.device).eval()
        self.tokenizer = tokenizer
        self.chunk_size = chunk_size
        self.min_chunk_tokens = min_chunk_tokens
        self.recompute_overlap = recompute_overlap
        self.recompute_strategy = RecomputeStrategy(recompute_strategy)
        self.kv_cache_bits = kv_cache_bits
        self.pool = None
        if kv_cache_bits == 8:
            from .paged import DeviceBlockAllocator
            cfg = self.model.config
            L = cfg.num_hidden_layers
            H = getattr(cfg, "num_key_value_heads", None) or cfg.num_attention_heads
            D = getattr(cfg, "head_dim", None) or cfg.hidden_size // cfg.num_attention_heads
            self._block_bytes = L * (2 * H * 16 * D + H * 16 * 6 + H * D * 6)
            nblk = int8_pool_blocks or max(1, min(int(max_cache_bytes) // self._block_bytes, 8192))
            self.pool = DeviceBlockAllocator(L, H, D, nblk, device=self.device)
            max_cache_bytes = min(int(max_cache_bytes), nblk * self._block_bytes)
        self.store = DeviceChunkStore(max_cache_bytes, on_evict=self._release_chunk)
        from .cacheblend import CacheBlendRecompute
        self.cacheblend_recompute = CacheBlendRecompute(recompute_ratio=recompute_ratio)
        self._flash_attn_patched = install_flash_attention(self.model)

    def _release_chunk(self, chunk: "DeviceChunk") -> None:
        if chunk.block_ids is not None and self.pool is not None:
            self.pool.free(chunk.block_ids)

    @classmethod
    def from_pretrained(cls, model_name: str, dtype=torch.bfloat16, **kwargs) -> "KVBoost":
        from transformers import AutoModelForCausalLM, AutoTokenizer
        tok = AutoTokenizer.from_pretrained(model_name)
        if tok.pad_token is None:
            tok.pad_token = tok.eos_token
        model = AutoModelForCausalLM.from_pretrained(model_name, dtype=dtype,
                                                     attn_implementation="sdpa")
        return cls(model, tok, **kwargs)

    # ── helpers ───────────────────────────────────────────────────────────────
    def _encode(self, prompt: Union[str, Sequence[int]]) -> TokenIds:
        if isinstance(prompt, str):
            if self.tokenizer is None:
                raise ValueError("a tokenizer is needed for text prompts")
            return self.tokenizer.encode(prompt, add_special_tokens=True)
        return [int(t) for t in prompt]

    def _decode_text(self, ids: List[int]) -> str:
        if self.tokenizer is None:
            return " ".join(str(i) for i in ids)
        return self.tokenizer.decode(ids, skip_special_tokens=True)

    def _sync(self) -> None:
        if self.device.type == "cuda":
            torch.cuda.synchronize(self.device)

    @property
    def _eos(self) -> Optional[int]:
        return getattr(self.tokenizer, "eos_token_id", None) if self.tokenizer else None

    @staticmethod
    def _layers(cache) -> List[Tuple[torch.Tensor, torch.Tensor]]:
        if hasattr(cache, "layers"):
            return [(l.keys, l.values) for l in cache.layers]
        return [(k, v) for k, v in zip(cache.key_cache, cache.value_cache)]

    @staticmethod
    def _cache_from(keys: torch.Tensor, values: torch.Tensor, batch: int = 1):
        """DynamicCache from stacked [layers, kv_heads, len, D] K/V, broadcast over batch."""
        from transformers import DynamicCache
        cache = DynamicCache()
        for l in range(keys.shape[0]):
            k = keys[l].unsqueeze(0).expand(batch, -1, -1, -1)
            v = values[l].unsqueeze(0).expand(batch, -1, -1, -1)
            cache.update(k, v, l)
        return cache

    def _forward(self, ids: torch.Tensor, pos: torch.Tensor, cache=None, keep=None):
        """Model forward with the cache; logits only at the last position, or at the
        sequence positions in the index tensor ``keep``."""
        with torch.no_grad():
            return self.model(input_ids=ids, position_ids=pos, past_key_values=cache,
                              use_cache=True, logits_to_keep=1 if keep is None else keep)

    def _encode_layers(self, ids: List[int], position_offset: int):
        """Per-layer ``[1, H, S, D]`` K/V of one chunk encoded on its own at its
        absolute positions (``engine.py:829-850``), as the model's cache holds them."""
        x = torch.tensor([ids], dtype=torch.long, device=self.device)
        pos = torch.arange(position_offset, position_offset + len(ids), device=self.device)[None]
        from transformers import DynamicCache
        out = self._forward(x, pos, DynamicCache())
        return self._layers(out.past_key_values)

    def _encode_to_kv(self, ids: List[int], position_offset: int):
        layers = self._encode_layers(ids, position_offset)
        return (torch.stack([k[0] for k, _ in layers]), torch.stack([v[0] for _, v in layers]))

    _STORE_BATCH = 32   # encoded chunks held back for one quantise-on-store launch

    def _store_chunk(self, key: str, ids: List[int], pos: int, pending=None) -> bool:
        """Encode one chunk and cache it.  int8 store: the model cache's tensors are
        queued in ``pending`` and written by one quantise-on-store launch per batch
        (``_flush_pending``); the chunk is registered at once (later kernels on the
        stream see its blocks written)."""
        if self.pool is None:
            k, v = self._encode_to_kv(ids, pos)
            return self.store.store(DeviceChunk(key, ids, pos, pos + len(ids), k, v))
        layers = self._encode_layers(ids, pos)
        nblk = (len(ids) + 15) // 16
        size = nblk * self._block_bytes
        if self.store.bytes + size > self.store.max_bytes:
            self._flush_pending(pending)      # eviction may hand queued blocks back out
        if not self.store.make_room(size):
            return False
        blocks = self.pool.allocate(nblk)
        item = (blocks, [k for k, _ in layers], [v for _, v in layers])
        if pending is None:
            self.pool.store_chunk_int8(*item)
        else:
            pending.append(item)
            if len(pending) >= self._STORE_BATCH:
                self._flush_pending(pending)
        return self.store.store(DeviceChunk(key, ids, pos, pos + len(ids), None, None,
                                            block_ids=blocks, pool_bytes=size))

    def _flush_pending(self, pending) -> None:
        if pending:
            self.pool.store_chunks_int8(pending)
            pending.clear()

    def _chunk_kv(self, chunks: List["DeviceChunk"]):
        """Stacked ``[L, H, P, D]`` K/V of a run of cached chunks in the model's dtype."""
        if chunks[0].block_ids is None:
            return (torch.cat([c.keys for c in chunks], dim=2),
                    torch.cat([c.values for c in chunks], dim=2))
        from .paged import block_table_tensor, paged_materialize
        dt = next(self.model.parameters()).dtype
        P = sum(c.length for c in chunks)
        # each chunk starts on a block boundary: gather through a per-token-exact
        # table (chunks shorter than their blocks leave no gaps in the sequence)
        if any(c.length % 16 for c in chunks[:-1]):
            raise RuntimeError("only the last cached chunk may end inside a 16-token block")
        table = block_table_tensor([[b for c in chunks for b in c.block_ids]], self.device)
        L, H, D = self.pool.num_layers, self.pool.num_heads, self.pool.head_dim
        kv_pad = (P + 127) // 128 * 128
        ws = torch.empty(L, 2, 1, H, kv_pad, D, dtype=dt, device=self.device)
        empty = torch.empty(1, H, 0, D, dtype=dt, device=self.device)
        for layer in range(L):
            paged_materialize(self.pool, layer, table, P, empty, empty, workspace=ws[layer])
        return ws[:, 0, 0, :, :P], ws[:, 1, 0, :, :P]

    def _sample(self, logits: torch.Tensor, temperature: float, do_sample: bool) -> torch.Tensor:
        if do_sample:
            probs = torch.softmax(logits.float() / max(temperature, 1e-5), dim=-1)
            return torch.multinomial(probs, 1)[..., 0]
        return logits.argmax(dim=-1)

    # ── cache population ─────────────────────────────────────────────────────
    def warm(self, text: Union[str, Sequence[int]], position_offset: int = 0) -> WarmResult:
        """Encode and cache every fixed-size chunk of ``text`` (``engine.py:415-507``)."""
        token_ids = self._encode(text)
        added = self._store_chunks(token_ids, position_offset)
        n = len(token_ids)
        tail = n % self.chunk_size
        aligned = tail == 0 or tail < self.min_chunk_tokens
        warning = None if aligned else (
            f"Prompt length {n} tokens is not a multiple of chunk_size {self.chunk_size}. "
            f"The last {tail} tokens will not be cached and must be recomputed on every "
            f"generate() call.")
        return WarmResult(added, n, self.chunk_size, aligned, tail, warning)

    warm_chunks = warm

    def _store_chunks(self, token_ids: TokenIds, position_offset: int = 0,
                      cacheable_prefix_len: Optional[int] = None) -> int:
        """Encode and store the not-yet-cached chunks of ``token_ids``; with
        ``cacheable_prefix_len`` only chunks that end within that many tokens
        (``engine.py:919-979``).  Returns how many were stored."""
        added, pos, parent = 0, position_offset, None
        pending: list = []
        for _, _, ids in fixed_split(token_ids, self.chunk_size, self.min_chunk_tokens):
            key = chained_hash(ids, parent)
            within = cacheable_prefix_len is None or pos + len(ids) <= cacheable_prefix_len
            if within and self.store.get(key) is None:
                if self._store_chunk(key, ids, pos, pending):
                    added += 1
            parent = key
            pos += len(ids)
        self._flush_pending(pending)
        return added

    def _store_prompt_chunks(self, token_ids: TokenIds,
                             cacheable_prefix_len: Optional[int] = None) -> None:
        """Cache the prompt's not-yet-cached chunks (``engine.py:919-979``)."""
        self._store_chunks(token_ids, 0, cacheable_prefix_len)

    def reset_cache(self) -> None:
        self.store.clear()

    # ── assembly and seam repair ─────────────────────────────────────────────
    def _assemble(self, token_ids: TokenIds, repair_seams: bool = True):
        """Stacked ``[L, H, P, D]`` K/V of the reused run (seams repaired per the
        strategy), its length and its chunk boundaries."""
        return self._assemble_run(token_ids, repair_seams)[:4]

    def _assemble_run(self, token_ids: TokenIds, repair_seams: bool = True):
        """``_assemble`` plus the list of reused chunks."""
        chunks, cached_len, boundaries = plan_reuse(token_ids, self.store, self.chunk_size,
                                                    self.min_chunk_tokens)
        if not chunks:
            return None, None, 0, boundaries, chunks
        keys, values = self._chunk_kv(chunks)
        if repair_seams and len(boundaries) > 1:
            if self.recompute_strategy == RecomputeStrategy.SELECTIVE:
                keys, values = self._recompute_seams(token_ids, keys, values, boundaries[:-1])
            elif self.recompute_strategy == RecomputeStrategy.CACHEBLEND:
                keys, values = self._cacheblend(token_ids, keys.contiguous(), values.contiguous(),
                                                cached_len)
        return keys, values, cached_len, boundaries, chunks

    def _cacheblend(self, token_ids, keys, values, cached_len):
        """``cacheblend.py:103-197``: a full-context forward over the cached tokens,
        then the deviation / top-k / patch on the device (``kvb_cacheblend_fwd``)."""
        from transformers import DynamicCache
        x = torch.tensor([token_ids[:cached_len]], dtype=torch.long, device=self.device)
        pos = torch.arange(0, cached_len, device=self.device)[None]
        out = self._forward(x, pos, DynamicCache())
        layers = self._layers(out.past_key_values)
        self.cacheblend_recompute.repair(keys, values, [k for k, _ in layers],
                                         [v for _, v in layers])
        return keys, values

    def _recompute_seams(self, token_ids, keys, values, seams):
        """``selective_recompute.py:99-184``: re-encode the last ``recompute_overlap``
        tokens before each seam with the (already repaired) prefix as context."""
        for _, end in seams:
            start = max(0, end - self.recompute_overlap)
            if start >= end:
                continue
            cache = self._cache_from(keys[:, :, :start].contiguous(),
                                     values[:, :, :start].contiguous())
            x = torch.tensor([token_ids[start:end]], dtype=torch.long, device=self.device)
            pos = torch.arange(start, end, device=self.device)[None]
            out = self._forward(x, pos, cache)
            layers = self._layers(out.past_key_values)
            fresh_k = torch.stack([k[0, :, start:end] for k, _ in layers])
            fresh_v = torch.stack([v[0, :, start:end] for _, v in layers])
            keys = torch.cat([keys[:, :, :start], fresh_k, keys[:, :, end:]], dim=2)
            values = torch.cat([values[:, :, :start], fresh_v, values[:, :, end:]], dim=2)
        return keys, values

    # ── generation ────────────────────────────────────────────────────────────
    def generate(self, prompt: Union[str, Sequence[int]], max_new_tokens: int = 64,
                 mode: Union[str, GenerationMode] = GenerationMode.CHUNK_KV_REUSE,
                 temperature: float = 1.0, do_sample: bool = False,
                 cacheable_prefix_len: Optional[int] = None) -> GenerationResult:
        """One prompt (``engine.py:207-233``).  ``CHUNK_KV_REUSE`` stitches the cached
        chunks (seam repair by ``recompute_strategy``) and then caches the prompt's
        new chunks -- with ``cacheable_prefix_len`` only those ending within that
        many tokens, so a per-query tail never enters the cache; ``PREFIX_CACHE``
        reuses the cached run from position 0 without repair (and stores the same
        way); ``BASELINE`` runs the whole prompt and stores nothing."""
        self._sync()
        t_start = time.perf_counter()
        token_ids = self._encode(prompt)
        mode = GenerationMode(mode)
        if mode == GenerationMode.BASELINE:
            keys = values = None
            cached_len = 0
        else:
            keys, values, cached_len, _ = self._assemble(
                token_ids, repair_seams=mode == GenerationMode.CHUNK_KV_REUSE)
        res = self._decode_batch([token_ids], keys, values, cached_len, max_new_tokens,
                                 temperature, do_sample, mode.value,
                                 prompts=[prompt if isinstance(prompt, str) else ""],
                                 t_start=t_start)[0]
        if mode == GenerationMode.BASELINE:
            res.kv_reuse_ratio = 0.0
        if mode != GenerationMode.BASELINE:     # both reuse modes store (engine.py:733)
            self._store_prompt_chunks(token_ids, cacheable_prefix_len=cacheable_prefix_len)
        return res

    def generate_batch(self, prompts: List[Union[str, Sequence[int]]], max_new_tokens: int = 64,
                       temperature: float = 1.0, do_sample: bool = False) -> List[GenerationResult]:
        """Prompts sharing a chunk-aligned prefix (``engine.py:235-365``): the shared
        K/V is assembled once (no seam repair, as in the reference) and broadcast
        over the batch; the suffixes are right-padded with the pad id to the longest
        and prefilled as one batch with no padding mask, each prompt's first token
        taken at its own last real position; decode then runs from the padded
        length for every prompt (``batch.py:69-83``, ``:107-175``), so a shorter
        prompt's context holds its pad tokens exactly as in the reference."""
        if len(prompts) == 1:
            return [self.generate(prompts[0], max_new_tokens, temperature=temperature,
                                  do_sample=do_sample)]
        self._sync()
        t_start = time.perf_counter()
        all_ids = [self._encode(p) for p in prompts]
        common = find_common_chunk_prefix(all_ids, self.chunk_size)
        keys = values = None
        cached_len = 0
        if common > 0:
            keys, values, cached_len, _ = self._assemble(all_ids[0][:common + 1],
                                                         repair_seams=False)
        texts = [p if isinstance(p, str) else "" for p in prompts]
        res = self._decode_batch(all_ids, keys, values, cached_len, max_new_tokens,
                                 temperature, do_sample, "chunk_kv_reuse_batch",
                                 prompts=texts, t_start=t_start)
        ratio = cached_len / max(max(len(ids) for ids in all_ids), 1)
        for r in res:
            r.kv_reuse_ratio = ratio
        for ids in all_ids:
            self._store_prompt_chunks(ids)
        return res

    def generate_many(self, prompts: List[Union[str, Sequence[int]]], max_new_tokens: int = 64,
                      temperature: float = 1.0, do_sample: bool = False) -> List[GenerationResult]:
        """Prompts grouped by their first three chunks (``engine.py:367-407``): a group
        of one runs through ``generate``, larger groups through ``generate_batch``;
        results in the order of ``prompts``."""
        all_ids = [self._encode(p) for p in prompts]
        results: List[Optional[GenerationResult]] = [None] * len(prompts)
        for idx in group_by_prefix(all_ids, self.chunk_size).values():
            group = [prompts[i] for i in idx]
            if len(group) == 1:
                out = [self.generate(group[0], max_new_tokens, temperature=temperature,
                                     do_sample=do_sample)]
            else:
                out = self.generate_batch(group, max_new_tokens, temperature=temperature,
                                          do_sample=do_sample)
            for i, r in zip(idx, out):
                results[i] = r
        return results

    @property
    def _pad(self) -> int:
        """``pad_token_id or eos_token_id`` as ``engine.py:283`` picks it (0 without a
        tokenizer)."""
        tok = self.tokenizer
        pad = getattr(tok, "pad_token_id", None) if tok is not None else None
        return int(pad or (self._eos or 0))

    def _decode_batch(self, all_ids: List[TokenIds], keys, values, cached_len: int,
                      max_new_tokens: int, temperature: float, do_sample: bool, mode_name: str,
                      prompts: List[str], t_start: float) -> List[GenerationResult]:
        """Suffix prefill over the reused prefix, then decode (``engine.py:634-753``;
        several prompts: ``engine.py:266-330`` and ``batch.py:107-175``).

        ``ttft_ms`` runs from the start of the ``generate`` call (so it includes
        prefix assembly and seam repair, which the reference's clock at
        ``engine.py:648`` leaves out) to the first sampled token on the host."""
        B = len(all_ids)
        suffixes = [ids[cached_len:] for ids in all_ids]
        lens = [len(s) for s in suffixes]
        width = max(lens)
        t0 = t_start
        from transformers import DynamicCache
        if width:
            cache = self._cache_from(keys, values, B) if keys is not None else DynamicCache()
            x = torch.tensor([s + [self._pad] * (width - len(s)) for s in suffixes],
                             dtype=torch.long, device=self.device)
            pos = torch.arange(cached_len, cached_len + width, device=self.device)
            pos = pos[None].expand(B, -1)
            keep = sorted({n - 1 for n in lens})
            out = self._forward(x, pos, cache,
                                keep=torch.tensor(keep, device=self.device) if len(keep) > 1
                                else None)
            col = torch.tensor([keep.index(n - 1) if len(keep) > 1 else 0 for n in lens],
                               device=self.device)
            last = out.logits[torch.arange(B, device=self.device), col]
            step_pos = cached_len + width
        else:  # everything cached: re-feed the last token (engine.py:688-712)
            cache = self._cache_from(keys[:, :, :cached_len - 1].contiguous(),
                                     values[:, :, :cached_len - 1].contiguous(), B)
            x = torch.tensor([[ids[-1]] for ids in all_ids], dtype=torch.long, device=self.device)
            pos = torch.full((B, 1), cached_len - 1, dtype=torch.long, device=self.device)
            out = self._forward(x, pos, cache)
            last = out.logits[:, -1, :]
            step_pos = cached_len
        nxt = self._sample(last, temperature, do_sample)
        first_logits = last.float()
        generated = [[int(t)] for t in nxt.tolist()]          # .tolist() synchronises
        t_first = time.perf_counter()
        cache = out.past_key_values
        eos = self._eos
        # one prompt stops after an end-of-sequence token, first one included
        # (engine.py:715-717); a batch marks a prompt done only from its second
        # token on and feeds done prompts the end id (batch.py:144-170)
        done = [B == 1 and g[-1] == eos for g in generated]
        while len(generated[0]) < max_new_tokens and not all(done):
            x = nxt[:, None]
            pos = torch.full((B, 1), step_pos, dtype=torch.long, device=self.device)
            out = self._forward(x, pos, cache)
            cache = out.past_key_values
            nxt = self._sample(out.logits[:, -1, :], temperature, do_sample)
            feed = []
            for b, t in enumerate(nxt.tolist()):
                if done[b]:
                    feed.append(eos if eos is not None else int(t))
                else:
                    generated[b].append(int(t))
                    done[b] = int(t) == eos
                    feed.append(int(t))
            if B > 1:
                nxt = torch.tensor(feed, dtype=torch.long, device=self.device)
            step_pos += 1
        t1 = time.perf_counter()
        results = []
        for b in range(B):
            n = len(all_ids[b])
            results.append(GenerationResult(
                mode=mode_name, prompt=prompts[b], output_text=self._decode_text(generated[b]),
                generated_tokens=len(generated[b]), ttft_ms=(t_first - t0) * 1e3,
                total_ms=(t1 - t0) * 1e3,
                tokens_per_sec=len(generated[b]) / max(t1 - t0, 1e-9),
                kv_reuse_ratio=cached_len / max(n, 1), prompt_tokens=n,
                cached_tokens=cached_len, first_token_logits=first_logits[b].cpu().numpy(),
                generated_ids=generated[b]))
        return results

    def cache_stats(self) -> Dict[str, float]:
        return self.store.stats()

    def verify_correctness(self, prompt: Union[str, Sequence[int]],
                           max_new_tokens: int = 32) -> bool:
        """Warm the prompt's first ``chunk_size`` multiple and compare greedy
        ``BASELINE`` with ``CHUNK_KV_REUSE`` output (``engine.py:993-1040``; the
        prompt is an argument here because the engine may run without a
        tokenizer)."""
        ids = self._encode(prompt)
        self.warm(ids[:len(ids) - len(ids) % self.chunk_size])
        base = self.generate(ids, max_new_tokens, mode=GenerationMode.BASELINE)
        cached = self.generate(ids, max_new_tokens, mode=GenerationMode.CHUNK_KV_REUSE)
        return base.generated_ids == cached.generated_ids

    def stats(self) -> Dict[str, float]:
        return self.store.stats()
