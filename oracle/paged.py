"""Oracle: paged KV block bookkeeping and the block-table gather.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

* ``AllocatorModel`` restates the id bookkeeping of ``BlockAllocator``
  (``src/kvboost/cpu_paged/block_allocator.py``): the free list starts as
  ``[0 .. num_blocks-1]`` and ``allocate`` pops from its END (``:76``, ``:93``),
  so the first allocation returns ``num_blocks-1, num_blocks-2, ...``;
  ``free`` decrements ref counts and appends at rc<=1 (``:98-107``); ``fork``
  increments (``:109-119``); ``ensure_writable`` pops a fresh id when rc>1
  (``:121-141``).
* ``MapperModel`` restates ``ChunkBlockMapper.load_chunk`` /
  ``build_block_table`` / ``on_evict`` (``chunk_to_blocks.py:57-139``):
  ``ceil(len/bs)`` fresh blocks per new chunk, a fork of the same ids on a
  repeat load, and concatenation in chunk order.
* ``append_slots`` restates the block bookkeeping of ``append_kv_to_blocks``
  (``cpu_paged/paged_attn_cpu.py:111-163``).
* ``gather`` restates ``BlockAllocator.read_kv`` (``block_allocator.py:178-206``):
  logical token ``t`` lives at ``(table[t // bs], t % bs)``.
"""

from __future__ import annotations

from typing import Dict, List

import numpy as np


class AllocatorModel:
    def __init__(self, num_blocks: int):
        self.num_blocks = num_blocks
        self.free_list: List[int] = list(range(num_blocks))
        self.ref: Dict[int, int] = {}

    def allocate(self, n: int) -> List[int]:
        if len(self.free_list) < n:
            raise RuntimeError(
                f"BlockAllocator OOM: requested {n} blocks but only "
                f"{len(self.free_list)} free (pool size {self.num_blocks}).")
        ids = [self.free_list.pop() for _ in range(n)]
        for b in ids:
            self.ref[b] = 1
        return ids

    def free(self, ids: List[int]) -> None:
        for b in ids:
            rc = self.ref.get(b, 0)
            if rc <= 1:
                self.ref.pop(b, None)
                self.free_list.append(b)
            else:
                self.ref[b] = rc - 1

    def fork(self, ids: List[int]) -> List[int]:
        for b in ids:
            self.ref[b] = self.ref.get(b, 1) + 1
        return list(ids)

    def ensure_writable(self, b: int) -> int:
        rc = self.ref.get(b, 1)
        if rc <= 1:
            return b
        if not self.free_list:
            raise RuntimeError("BlockAllocator OOM during copy-on-write.")
        nb = self.free_list.pop()
        self.ref[nb] = 1
        self.ref[b] = rc - 1
        return nb


class MapperModel:
    def __init__(self, alloc: AllocatorModel, block_size: int):
        self.alloc = alloc
        self.bs = block_size
        self.chunk_blocks: Dict[str, List[int]] = {}

    def load_chunk(self, chunk_id: str, length: int) -> List[int]:
        if chunk_id in self.chunk_blocks:
            return self.alloc.fork(self.chunk_blocks[chunk_id])
        ids = self.alloc.allocate((length + self.bs - 1) // self.bs)
        self.chunk_blocks[chunk_id] = ids
        return list(ids)

    def build_block_table(self, chunks) -> List[int]:
        table: List[int] = []
        for cid, length in chunks:
            table.extend(self.load_chunk(cid, length))
        return table

    def on_evict(self, chunk_id: str) -> None:
        ids = self.chunk_blocks.pop(chunk_id, None)
        if ids is not None:
            self.alloc.free(ids)


def append_slots(alloc: AllocatorModel, table: List[int], slot_offset: int, n: int,
                 block_size: int):
    """Block bookkeeping of ``append_kv_to_blocks`` (``cpu_paged/paged_attn_cpu.py:111-163``)
    for ``n`` tokens from logical slot ``slot_offset``: a block is allocated when the
    table runs out, and every touched block is made writable (copy-on-write) in
    token order.  Returns ``(table, slot_offset + n)``."""
    table = list(table)
    for t in range(n):
        bi = (slot_offset + t) // block_size
        if bi >= len(table):
            table.extend(alloc.allocate(1))
        table[bi] = alloc.ensure_writable(table[bi])
    return table, slot_offset + n


def gather(pool_kv: np.ndarray, table: List[int], seq_len: int):
    """pool_kv: ``[num_blocks, 2, H, bs, D]`` -> (K, V) each ``[H, seq_len, D]``."""
    nb = len(table)
    g = pool_kv[np.asarray(table, dtype=np.int64)]            # [nb, 2, H, bs, D]
    H, bs, D = g.shape[2], g.shape[3], g.shape[4]
    k = g[:, 0].transpose(1, 0, 2, 3).reshape(H, nb * bs, D)[:, :seq_len]
    v = g[:, 1].transpose(1, 0, 2, 3).reshape(H, nb * bs, D)[:, :seq_len]
    return k, v


def gather_scales(scale_per_block: np.ndarray, table: List[int], seq_len: int,
                  block_size: int, per_token: bool):
    """Per-token view of block scales.

    per_token=True : ``scale_per_block`` is ``[num_blocks, H, bs]`` -> ``[H, seq_len]``.
    per_token=False: ``scale_per_block`` is ``[num_blocks, H, D]`` (one row per block,
    copied from the owning chunk) -> ``[H, seq_len, D]``.
    """
    g = np.asarray(scale_per_block)[np.asarray(table, dtype=np.int64)]
    if per_token:                                               # [nb, H, bs]
        H = g.shape[1]
        return g.transpose(1, 0, 2).reshape(H, -1)[:, :seq_len]
    tok_block = np.arange(seq_len) // block_size                # [nb, H, D]
    return g[tok_block].transpose(1, 0, 2)


def dequant_gather(pool_q: np.ndarray, k_scale: np.ndarray, v_scale: np.ndarray,
                   table: List[int], seq_len: int, block_size: int):
    """int8 paged pool -> float16 K/V ``[H, seq_len, D]`` exactly as the reference.

    ``pool_q``: int8 ``[num_blocks, 2, H, bs, D]``; ``k_scale``: float16
    ``[num_blocks, H, bs]`` (per token); ``v_scale``: float16 ``[num_blocks, H, D]``
    (per channel of the owning chunk).  Each value is ``float16(q * s)``
    (``kv_quantize.py:102-109``).
    """
    from .kv_quant import dequantize_int8
    kq, vq = gather(pool_q, table, seq_len)                     # [H, S, D] int8
    ks = gather_scales(k_scale, table, seq_len, block_size, per_token=True)   # [H, S]
    vs = gather_scales(v_scale, table, seq_len, block_size, per_token=False)  # [H, S, D]
    k = dequantize_int8(kq, ks[..., None])
    v = dequantize_int8(vq, vs)
    return k, v
