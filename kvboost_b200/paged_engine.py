"""Paged-pool generation engine: the drop-in for KVBoost's ``CPUPagedEngine``.

Mirrors ``src/kvboost/cpu_paged/cpu_engine.py:72-516``: the chunk-reuse engine
(``KVBoost``) whose single-prompt generation keeps the sequence's K/V in a
16-token block pool instead of a growing cache tensor:

1. the reused chunks are loaded into the pool through the chunk mapper (a
   chunk already in the pool is forked, so its blocks are shared), giving the
   sequence's block table (``cpu_engine.py:187-206``);
2. the prompt's new tokens run as one model forward over the assembled
   (seam-repaired) prefix, and their K/V are appended to the pool after the
   prefix -- every layer at the same slots, new blocks taken from the free list
   by the first layer (``:208-248``, ``:440-475``); a fully cached prompt
   re-feeds its last token and appends it after the prefix (``:250-282``);
3. each decode step runs the model with no cache: the paged interceptor
   (``flash_attn_ext.install_paged_attention``) appends the step's K/V at the
   next slot and attends over the pool (``:284-310``, ``:344-408``);
4. the sequence's own blocks (past the reused prefix) go back to the free list,
   then the prompt's new chunks are stored (``:312-319``, ``:499-512``).

The block bookkeeping (free-list order, forks, copy-on-write, which blocks are
freed) follows the reference step for step, so block tables are identical.
What differs is where it runs: the pool lives in GPU memory in the model's
dtype (the reference's pool is float16 because its ``from_pretrained`` loads
the model in float16), the appends are device scatters, the prefill runs on the
sm_100a prefill kernel and the decode steps on the paged attention path.  The
reference class raises under transformers 5.x (it indexes the returned
``DynamicCache`` as a tuple, ``cpu_engine.py:451``); this one reads the cache's
layers.  ``generate_batch`` / ``generate_many`` are ``KVBoost``'s (the
reference's paged engine inherits them unchanged), and ``BASELINE`` mode runs
the whole prompt as in ``KVBoost``.
"""

from __future__ import annotations

import time
from typing import List, Optional, Sequence, Tuple, Union

import torch

from .engine import GenerationMode, GenerationResult, KVBoost, TokenIds
from .flash_attn_ext import install_paged_attention, uninstall_paged_attention
from .paged import BLOCK_SIZE, DeviceBlockAllocator, DeviceChunkMapper


def _model_dims(model) -> Tuple[int, int, int]:
    """(layers, KV heads, head dim) as ``_infer_model_dims`` (``cpu_engine.py:56-69``)
    reads them, with the config's explicit ``head_dim`` where it has one."""
    cfg = model.config
    heads = cfg.num_attention_heads
    kv = getattr(cfg, "num_key_value_heads", None) or heads
    d = getattr(cfg, "head_dim", None) or cfg.hidden_size // heads
    return cfg.num_hidden_layers, kv, d


class PagedEngine(KVBoost):
    """``KVBoost`` with the paged decode loop of ``CPUPagedEngine``.

    ``block_size`` (16, the paged kernels' block) and ``num_blocks`` (pool size)
    as in the reference; ``pool_dtype`` defaults to the model's dtype.
    """

    def __init__(self, model, tokenizer=None, *, max_cache_bytes: int = 16 << 30,
                 block_size: int = BLOCK_SIZE, num_blocks: int = 4096,
                 pool_dtype: Optional[torch.dtype] = None, **kwargs) -> None:
        super().__init__(model, tokenizer, max_cache_bytes=max_cache_bytes, **kwargs)
        L, H, D = _model_dims(self.model)
        dt = pool_dtype or next(self.model.parameters()).dtype
        self.allocator = DeviceBlockAllocator(L, H, D, num_blocks, block_size,
                                              device=self.device, dtype=dt)
        self.chunk_mapper = DeviceChunkMapper(self.allocator)
        self._num_layers, self._block_size = L, block_size
        store_evict = self.store.on_evict

        def on_evict(chunk):      # chunk blocks leave the pool with the chunk (:124-126)
            store_evict(chunk)
            self.chunk_mapper.on_evict(chunk.chunk_id)
        self.store.on_evict = on_evict

    # ── generation ────────────────────────────────────────────────────────────
    def generate(self, prompt: Union[str, Sequence[int]], max_new_tokens: int = 64,
                 mode: Union[str, GenerationMode] = GenerationMode.CHUNK_KV_REUSE,
                 temperature: float = 1.0, do_sample: bool = False,
                 cacheable_prefix_len: Optional[int] = None) -> GenerationResult:
        mode = GenerationMode(mode)
        if mode == GenerationMode.BASELINE:
            return super().generate(prompt, max_new_tokens, mode, temperature, do_sample)
        self._sync()
        t0 = time.perf_counter()
        token_ids = self._encode(prompt)
        reuse = mode == GenerationMode.CHUNK_KV_REUSE
        keys, values, cached_len, _, chunks = self._assemble_run(token_ids, repair_seams=reuse)
        res = self._paged_decode(prompt, token_ids, chunks, keys, values, cached_len,
                                 max_new_tokens, temperature, do_sample, mode.value, t0,
                                 # the reference passes its hit ratio only in reuse mode
                                 cached_len / max(len(token_ids), 1) if reuse else 0.0)
        self._store_prompt_chunks(token_ids, cacheable_prefix_len=cacheable_prefix_len)
        return res

    def _append_layers(self, layers, table: List[int], slot: int,
                       skip: int) -> Tuple[List[int], int]:
        """The tokens from ``skip`` on of each layer's cache appended at ``slot``
        (``_append_new_kv_to_pool``, ``cpu_engine.py:440-475``)."""
        n_new = layers[0][0].shape[2] - skip
        if n_new <= 0:
            return table, slot
        for layer, (k, v) in enumerate(layers):
            table, _ = self.allocator.append_kv(layer, table, slot, k[0, :, skip:],
                                                v[0, :, skip:])
        return table, slot + n_new

    def _paged_decode(self, prompt, token_ids: TokenIds, chunks, keys, values, cached_len: int,
                      max_new_tokens: int, temperature: float, do_sample: bool, mode_name: str,
                      t0: float, hit_ratio: float) -> GenerationResult:
        from transformers import DynamicCache
        table: List[int] = []
        in_pool = 0
        if keys is not None and cached_len > 0:
            for c in chunks:      # the chunks as cached (before any seam repair)
                k, v = self._chunk_kv([c])
                table.extend(self.chunk_mapper.load_chunk(
                    c.chunk_id, [(k[l][None], v[l][None]) for l in range(k.shape[0])]))
            in_pool = cached_len
        live = token_ids[cached_len:]
        if live:
            cache = self._cache_from(keys, values) if keys is not None else DynamicCache()
            x = torch.tensor([live], dtype=torch.long, device=self.device)
            pos = torch.arange(cached_len, cached_len + len(live), device=self.device)[None]
            skip = cached_len
        else:     # fully cached: re-feed the last token at its position
            cache = (self._cache_from(keys[:, :, :cached_len - 1].contiguous(),
                                      values[:, :, :cached_len - 1].contiguous())
                     if cached_len > 1 else DynamicCache())
            x = torch.tensor([[token_ids[-1]]], dtype=torch.long, device=self.device)
            pos = torch.tensor([[cached_len - 1]], dtype=torch.long, device=self.device)
            skip = cached_len - 1
        out = self._forward(x, pos, cache)
        first_logits = out.logits[0, -1, :].float()
        generated = [int(self._sample(out.logits[:, -1, :], temperature, do_sample)[0])]
        t_first = time.perf_counter()
        table, in_pool = self._append_layers(self._layers(out.past_key_values), table, in_pool,
                                             skip)
        del out, cache
        cur = cached_len + len(live)
        state = {"allocator": self.allocator, "block_table": table, "_write_slot": in_pool}
        eos = self._eos
        install_paged_attention(self.model, state)
        try:
            while len(generated) < max_new_tokens and generated[-1] != eos:
                x = torch.tensor([[generated[-1]]], dtype=torch.long, device=self.device)
                p = torch.tensor([[cur]], dtype=torch.long, device=self.device)
                with torch.no_grad():
                    logits = self.model(input_ids=x, position_ids=p, use_cache=False,
                                        logits_to_keep=1).logits
                state["_write_slot"] += 1
                generated.append(int(self._sample(logits[:, -1, :], temperature, do_sample)[0]))
                cur += 1
        finally:
            uninstall_paged_attention(self.model)
        table = state["block_table"]
        t1 = time.perf_counter()
        # the sequence's own blocks (past the reused prefix's) return to the free list
        cached_blocks = (cached_len + self._block_size - 1) // self._block_size
        if table[cached_blocks:]:
            self.allocator.free(table[cached_blocks:])
        self.last_block_table = table
        return GenerationResult(
            mode=mode_name, prompt=prompt if isinstance(prompt, str) else "",
            output_text=self._decode_text(generated), generated_tokens=len(generated),
            ttft_ms=(t_first - t0) * 1e3, total_ms=(t1 - t0) * 1e3,
            tokens_per_sec=len(generated) / max(t1 - t0, 1e-9), kv_reuse_ratio=hit_ratio,
            prompt_tokens=len(token_ids), cached_tokens=cached_len,
            first_token_logits=first_logits.cpu().numpy(), generated_ids=generated)

    def paged_stats(self) -> dict:
        """``paged_stats`` (``cpu_engine.py:514-522``)."""
        return {"block_utilization": self.allocator.utilization(),
                "free_blocks": self.allocator.free_blocks,
                "used_blocks": self.allocator.used_blocks,
                "num_blocks": self.allocator.num_blocks,
                "loaded_chunks": self.chunk_mapper.loaded_chunks(),
                "blocks_used_by_chunks": self.chunk_mapper.blocks_used_by_chunks()}


# the reference's name for it
CPUPagedEngine = PagedEngine
