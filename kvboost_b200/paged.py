"""Device-resident int8 paged KV pool and the paged reuse-prefill op.

The bookkeeping mirrors KVBoost's CPU pool so block tables are identical:

* ``DeviceBlockAllocator`` -- ``BlockAllocator`` (``cpu_paged/block_allocator.py``):
  free list ``[0 .. num_blocks-1]`` popped from the end (``:76``, ``:93``), ref
  counts, ``fork`` (``:109-119``), copy-on-write ``ensure_writable``
  (``:121-141``), ``free`` (``:98-107``), ``free_blocks`` / ``used_blocks`` /
  ``utilization``.  The storage is on the GPU and int8: per layer
  ``[num_blocks, 2, num_kv_heads, 16, head_dim]`` (the reference pool's
  layout, ``:67-73``) plus per-block scales.
* ``DeviceChunkMapper`` -- ``ChunkBlockMapper`` (``cpu_paged/chunk_to_blocks.py:57-139``):
  ``ceil(len/16)`` fresh blocks per new chunk, a fork of the same ids for a
  chunk already loaded, tables concatenated in chunk order, ``on_evict``.

Chunks are stored KIVI int8 exactly as ``quantize_kv(bits=8)`` produces them
(``kv_quantize.py:73-100``): K with one float16 scale per token, V with one
float16 scale per channel of the chunk.  ``quantize_chunk_int8`` reproduces
that arithmetic on the GPU bit for bit (torch float16 ops round each result
like the reference's CPU ops).  The kernel reads the scales as float32
copies of those float16 values.

``paged_prefill_attention`` runs the suffix prefill over the pool with the
block-table gather and the int8 dequantisation fused into the kernel's K/V
load stage (``kvb_paged_prefill_fwd``).
"""

from __future__ import annotations

import ctypes
import math
import threading
from typing import Dict, List, Optional, Sequence, Tuple

import torch

from . import _lib
from .ops import _DTYPES, _check_tensor, _stream_handle, status_word

BLOCK_SIZE = 16


def quantize_chunk_int8(key: torch.Tensor, val: torch.Tensor):
    """KIVI int8 of one chunk, same arithmetic as ``_quantize_int8`` (``kv_quantize.py:73-100``).

    key/val: ``[..., S, D]`` float16.  Returns ``(key_q int8, key_scale fp16 [...,S,1],
    val_q int8, val_scale fp16 [...,1,D])``.
    """
    key = key.to(torch.float16)
    val = val.to(torch.float16)
    key_amax = key.abs().amax(dim=-1, keepdim=True).clamp(min=1e-8)
    key_scale = key_amax / 127.0
    key_q = (key / key_scale).round().clamp(-128, 127).to(torch.int8)
    val_amax = val.abs().amax(dim=-2, keepdim=True).clamp(min=1e-8)
    val_scale = val_amax / 127.0
    val_q = (val / val_scale).round().clamp(-128, 127).to(torch.int8)
    return key_q, key_scale.to(torch.float16), val_q, val_scale.to(torch.float16)


def _layer_list(x) -> List[torch.Tensor]:
    """Per-layer ``[H, S, D]`` views of a stacked ``[L, H, S, D]`` tensor or of a
    sequence of ``[H, S, D]`` / ``[1, H, S, D]`` tensors."""
    if isinstance(x, torch.Tensor):
        if x.dim() != 4:
            raise ValueError("stacked K/V must be [layers, heads, tokens, head_dim]")
        return list(x.unbind(0))
    out = []
    for t in x:
        if t.dim() == 4:
            if t.shape[0] != 1:
                raise ValueError("per-layer K/V must be [H, S, D] or [1, H, S, D]")
            t = t[0]
        if t.dim() != 3:
            raise ValueError("per-layer K/V must be [H, S, D] or [1, H, S, D]")
        out.append(t)
    return out


class DeviceBlockAllocator:
    """Block allocator over a GPU int8 KV pool (``BlockAllocator`` semantics)."""

    def __init__(self, num_layers: int, num_heads: int, head_dim: int, num_blocks: int = 4096,
                 block_size: int = BLOCK_SIZE, device="cuda", dtype=torch.int8) -> None:
        """``dtype``: ``torch.int8`` for KIVI-quantised chunks (per-block scales), or
        ``torch.float16`` / ``torch.bfloat16`` for a pool holding K/V as is (the
        reference's paged engine pool, which tokens are appended to one by one)."""
        if block_size != BLOCK_SIZE:
            raise ValueError("the paged kernels use 16-token blocks")
        if dtype not in (torch.int8, torch.float16, torch.bfloat16):
            raise ValueError("pool dtype must be int8, float16 or bfloat16")
        self.num_layers = num_layers
        self.num_heads = num_heads
        self.head_dim = head_dim
        self.num_blocks = num_blocks
        self.block_size = block_size
        self.dtype = dtype
        self.device = torch.device(device)
        self.pools: List[torch.Tensor] = [
            torch.zeros(num_blocks, 2, num_heads, block_size, head_dim, dtype=dtype,
                        device=self.device) for _ in range(num_layers)]
        # float16 scales as the reference stores them, and the float32 copies the kernel reads
        self.k_scale16 = [torch.zeros(num_blocks, num_heads, block_size, dtype=torch.float16,
                                      device=self.device) for _ in range(num_layers)]
        self.v_scale16 = [torch.zeros(num_blocks, num_heads, head_dim, dtype=torch.float16,
                                      device=self.device) for _ in range(num_layers)]
        self.k_scale = [torch.zeros(num_blocks, num_heads, block_size, dtype=torch.float32,
                                    device=self.device) for _ in range(num_layers)]
        self.v_scale = [torch.zeros(num_blocks, num_heads, head_dim, dtype=torch.float32,
                                    device=self.device) for _ in range(num_layers)]
        self._free: List[int] = list(range(num_blocks))
        self._ref_count: Dict[int, int] = {}
        self._lock = threading.Lock()

    # ── allocation (block_allocator.py:85-141) ─────────────────────────────────
    def allocate(self, n: int) -> List[int]:
        with self._lock:
            if len(self._free) < n:
                raise RuntimeError(
                    f"BlockAllocator OOM: requested {n} blocks but only "
                    f"{len(self._free)} free (pool size {self.num_blocks}).")
            ids = [self._free.pop() for _ in range(n)]
            for b in ids:
                self._ref_count[b] = 1
            return ids

    def free(self, block_ids: List[int]) -> None:
        with self._lock:
            for b in block_ids:
                rc = self._ref_count.get(b, 0)
                if rc <= 1:
                    self._ref_count.pop(b, None)
                    self._free.append(b)
                else:
                    self._ref_count[b] = rc - 1

    def fork(self, block_ids: List[int]) -> List[int]:
        with self._lock:
            for b in block_ids:
                self._ref_count[b] = self._ref_count.get(b, 1) + 1
        return list(block_ids)

    def ensure_writable(self, block_id: int) -> int:
        with self._lock:
            rc = self._ref_count.get(block_id, 1)
            if rc <= 1:
                return block_id
            if not self._free:
                raise RuntimeError("BlockAllocator OOM during copy-on-write.")
            new_id = self._free.pop()
            self._ref_count[new_id] = 1
            self._ref_count[block_id] = rc - 1
        for t in (*self.pools, *self.k_scale16, *self.v_scale16, *self.k_scale, *self.v_scale):
            t[new_id].copy_(t[block_id])
        return new_id

    @property
    def free_blocks(self) -> int:
        return len(self._free)

    @property
    def used_blocks(self) -> int:
        return self.num_blocks - len(self._free)

    def utilization(self) -> float:
        return self.used_blocks / self.num_blocks

    # ── storage ────────────────────────────────────────────────────────────────
    def write_chunk_int8(self, layer: int, block_ids: List[int], key_q: torch.Tensor,
                         key_scale: torch.Tensor, val_q: torch.Tensor,
                         val_scale: torch.Tensor) -> None:
        """Store one quantised chunk (``[1 or H.., S, D]`` as ``quantize_kv`` returns it).

        Token t of the chunk goes to ``block_ids[t // 16]``, slot ``t % 16``; every
        block of the chunk gets the chunk's per-channel V scale.
        """
        H, D, bs = self.num_heads, self.head_dim, self.block_size
        kq = key_q.reshape(H, -1, D)
        S = kq.shape[1]
        n = len(block_ids)
        if n * bs < S:
            raise ValueError(f"{n} blocks cannot hold {S} tokens")
        idx = torch.as_tensor(block_ids, dtype=torch.long, device=self.device)

        def blocked(t, last):  # [H, S, last] -> [n, H, bs, last], zero padded
            pad = torch.zeros(H, n * bs, last, dtype=t.dtype, device=self.device)
            pad[:, :S] = t.to(self.device)
            return pad.view(H, n, bs, last).permute(1, 0, 2, 3)

        pool = self.pools[layer]
        pool[idx, 0] = blocked(kq, D)
        pool[idx, 1] = blocked(val_q.reshape(H, -1, D), D)
        ks = blocked(key_scale.reshape(H, -1, 1).to(torch.float16), 1)[..., 0]   # [n, H, bs]
        self.k_scale16[layer][idx] = ks
        self.k_scale[layer][idx] = ks.float()
        vs = val_scale.reshape(H, D).to(torch.float16).to(self.device)
        self.v_scale16[layer][idx] = vs.unsqueeze(0).expand(n, H, D)
        self.v_scale[layer][idx] = vs.float().unsqueeze(0).expand(n, H, D)

    def store_chunk_int8(self, block_ids: List[int], keys, values) -> None:
        """Quantise one freshly encoded chunk on the device and store it in its blocks,
        every layer in one launch (``kvb_quantize_store``).

        ``keys`` / ``values``: per layer, the chunk's K/V as ``[H, S, D]`` or
        ``[1, H, S, D]`` tensors (the model cache's own per-layer tensors, any
        strides with a contiguous last dimension), or one stacked ``[L, H, S, D]``
        tensor, in bfloat16 or float16.  Same bytes in the pool and the same scales
        as quantising with the reference's arithmetic in that dtype
        (``kv_quantize.py:73-100``) and then ``write_chunk_int8``: token t in
        ``block_ids[t // 16]``, slot ``t % 16``, zero-padded last block, the chunk's
        per-channel V scales in every block of the chunk.
        """
        if self.dtype != torch.int8:
            raise RuntimeError("store_chunk_int8 needs an int8 pool")
        ks, vs = _layer_list(keys), _layer_list(values)
        L = len(ks)
        if L != len(vs) or not 1 <= L <= min(self.num_layers, _lib.KVB_MAX_LAYERS):
            raise ValueError(f"need K and V for 1..{self.num_layers} layers, got {len(ks)} / {len(vs)}")
        ref = ks[0]
        if ref.dtype not in _DTYPES:
            raise TypeError("chunk K/V must be bfloat16 or float16")
        H, S, D = ref.shape
        if H != self.num_heads or D != self.head_dim:
            raise ValueError(f"chunk K/V {tuple(ref.shape)} do not match the pool's heads / head_dim")
        n = len(block_ids)
        if n * self.block_size < S or n > _lib.KVB_MAX_CHUNK_BLOCKS:
            raise ValueError(f"{n} blocks cannot hold {S} tokens (at most "
                             f"{_lib.KVB_MAX_CHUNK_BLOCKS} blocks per chunk)")
        pool_dev = self.pools[0].device
        for t in ks + vs:
            if t.shape != ref.shape or t.dtype != ref.dtype or t.device != pool_dev:
                raise ValueError("every layer's K and V must share shape, dtype and the pool's device")
        if any(t.stride() != ref.stride() or t.stride(2) != 1 or t.stride(0) % 8 or t.stride(1) % 8
               or t.data_ptr() % 16 for t in ks + vs):
            ks = [t.contiguous() for t in ks]
            vs = [t.contiguous() for t in vs]
            ref = ks[0]
        p = _lib.KvbQuantizeStoreParams()
        p.dtype, p.head_dim, p.num_layers, p.num_kv_heads = _DTYPES[ref.dtype], D, L, H
        p.num_tokens, p.num_chunk_blocks = S, n
        for i, b in enumerate(block_ids):
            p.block_ids[i] = int(b)
        p.num_pool_blocks = self.num_blocks
        arrays = [_lib.pointer_array([t.data_ptr() for t in group]) for group in (
            ks, vs, self.pools[:L], self.k_scale16[:L], self.v_scale16[:L],
            self.k_scale[:L], self.v_scale[:L])]
        (p.src_k, p.src_v, p.pool, p.k_scale16, p.v_scale16, p.k_scale, p.v_scale) = [
            ctypes.cast(a, _lib._pp) for a in arrays]
        p.src_head_stride, p.src_row_stride = ref.stride(0), ref.stride(1)
        with torch.cuda.device(pool_dev):
            _lib.check(_lib.load().kvb_quantize_store(ctypes.byref(p), _stream_handle(pool_dev)),
                       "kvb_quantize_store")

    def store_chunks_int8(self, chunks) -> None:
        """``store_chunk_int8`` for several chunks in one launch
        (``kvb_quantize_store_batch``): ``chunks`` is a sequence of
        ``(block_ids, keys, values)`` as ``store_chunk_int8`` takes them, with
        disjoint blocks.  The pointer tables, token counts and block ids travel to
        the device in one copy on the current stream."""
        if chunks:
            self.launch_prepared(self.prepare_chunks_int8(chunks))

    def launch_prepared(self, prepared) -> None:
        """Launch a batch built by ``prepare_chunks_int8`` (capturable in a CUDA
        graph: no host memory is read at launch)."""
        p, _, _ = prepared
        dev = self.pools[0].device
        with torch.cuda.device(dev):
            _lib.check(_lib.load().kvb_quantize_store_batch(ctypes.byref(p), _stream_handle(dev)),
                       "kvb_quantize_store_batch")

    def prepare_chunks_int8(self, chunks):
        """Device tables for ``launch_prepared``: returns ``(params, device tables,
        sources)``; keep it alive while launches that use it may run."""
        if self.dtype != torch.int8:
            raise RuntimeError("store_chunks_int8 needs an int8 pool")
        if not chunks:
            raise ValueError("no chunks")
        items = [(list(b), _layer_list(k), _layer_list(v)) for b, k, v in chunks]
        L = len(items[0][1])
        ref = items[0][1][0]
        if ref.dtype not in _DTYPES:
            raise TypeError("chunk K/V must be bfloat16 or float16")
        H, _, D = ref.shape
        if H != self.num_heads or D != self.head_dim or not 1 <= L <= min(self.num_layers,
                                                                          _lib.KVB_MAX_LAYERS):
            raise ValueError("chunk K/V do not match the pool's layers / heads / head_dim")
        pool_dev = self.pools[0].device
        seen, fixed = set(), []
        for blocks, ks, vs in items:
            if len(ks) != L or len(vs) != L:
                raise ValueError("every chunk needs K and V for the same layers")
            S = ks[0].shape[1]
            if len(blocks) * self.block_size < S or len(blocks) > _lib.KVB_MAX_CHUNK_BLOCKS:
                raise ValueError(f"{len(blocks)} blocks cannot hold {S} tokens")
            if seen.intersection(blocks):
                raise ValueError("the chunks' blocks overlap")
            seen.update(blocks)
            st0 = ks[0].stride()
            for t in ks + vs:
                if t.shape != (H, S, D) or t.dtype != ref.dtype or t.device != pool_dev:
                    raise ValueError("chunk K/V must share heads, head_dim, dtype and the pool's device")
            if any(t.stride() != st0 or st0[2] != 1 or st0[0] % 8 or st0[1] % 8 or t.data_ptr() % 16
                   for t in ks + vs):   # one layout per chunk: contiguous copies
                ks, vs = [t.contiguous() for t in ks], [t.contiguous() for t in vs]
            fixed.append((blocks, ks, vs))
        items = fixed
        n, mb = len(items), max(len(b) for b, _, _ in items)
        src = [p for _, ks, vs in items for k, v in zip(ks, vs) for p in (k.data_ptr(), v.data_ptr())]
        strides = [x for _, ks, _ in items for x in ks[0].stride()[:2]]
        tables = [t.data_ptr() for group in (self.pools, self.k_scale16, self.v_scale16,
                                             self.k_scale, self.v_scale) for t in group[:L]]
        tokens = [ks[0].shape[1] for _, ks, _ in items]
        bids = [x for b, _, _ in items for x in (b + [-1] * (mb - len(b)))]
        n64 = len(src) + len(strides) + len(tables)
        host = torch.empty(n64 * 8 + (len(tokens) + len(bids)) * 4, dtype=torch.uint8).pin_memory()
        host[:n64 * 8].view(torch.int64).copy_(torch.tensor(src + strides + tables, dtype=torch.int64))
        host[n64 * 8:].view(torch.int32).copy_(torch.tensor(tokens + bids, dtype=torch.int32))
        dev = host.to(pool_dev, non_blocking=True)
        base = dev.data_ptr()
        p = _lib.KvbQuantizeStoreBatch()
        p.dtype, p.head_dim, p.num_layers, p.num_kv_heads = _DTYPES[ref.dtype], D, L, H
        p.num_chunks, p.max_chunk_blocks, p.num_pool_blocks = n, mb, self.num_blocks
        p.src = base
        p.src_strides = base + len(src) * 8
        p.tables = base + (len(src) + len(strides)) * 8
        p.num_tokens = base + n64 * 8
        p.block_ids = base + n64 * 8 + len(tokens) * 4
        p.status = status_word(pool_dev).data_ptr()
        return p, dev, items

    def write_chunk(self, layer: int, block_ids: List[int], key: torch.Tensor,
                    val: torch.Tensor) -> None:
        """Store one chunk's K/V (``[1 or H.., S, D]``) as is in a 16-bit pool: token t
        goes to ``block_ids[t // 16]``, slot ``t % 16`` (``chunk_to_blocks.py:57-101``)."""
        if self.dtype == torch.int8:
            raise RuntimeError("int8 pools store KIVI chunks (write_chunk_int8)")
        H, D, bs = self.num_heads, self.head_dim, self.block_size
        k = key.reshape(H, -1, D)
        S = k.shape[1]
        n = len(block_ids)
        if n * bs < S:
            raise ValueError(f"{n} blocks cannot hold {S} tokens")
        idx = torch.as_tensor(block_ids, dtype=torch.long, device=self.device)
        for kv, t in ((0, k), (1, val.reshape(H, -1, D))):
            pad = torch.zeros(H, n * bs, D, dtype=self.dtype, device=self.device)
            pad[:, :S] = t.to(self.device, self.dtype)
            self.pools[layer][idx, kv] = pad.view(H, n, bs, D).permute(1, 0, 2, 3)

    @property
    def pool_format(self) -> int:
        return _lib.KVB_POOL_INT8_KIVI if self.dtype == torch.int8 else _lib.KVB_POOL_COMPUTE

    def append_kv(self, layer: int, block_table: List[int], slot_offset: int,
                  k: torch.Tensor, v: torch.Tensor) -> Tuple[List[int], int]:
        """``append_kv_to_blocks`` (``cpu_paged/paged_attn_cpu.py:111-163``) for a 16-bit
        pool: token t of ``k``/``v`` (``[H, n, D]``) goes to logical slot
        ``slot_offset + t``; blocks are allocated from the free list when the table
        runs out and shared blocks are copied on write, in the reference's order.  The
        block bookkeeping stays on the host; the n tokens are written by one device
        scatter instead of a Python loop of per-token copies.  Returns the updated
        table and the next slot."""
        if self.dtype == torch.int8:
            raise RuntimeError("int8 pools hold whole KIVI chunks (write_chunk_int8)")
        table = list(block_table)
        bs = self.block_size
        n = k.shape[1]
        blocks, slots = [], []
        for t in range(n):
            pos = slot_offset + t
            bi = pos // bs
            if bi >= len(table):
                table.extend(self.allocate(1))
            bid = self.ensure_writable(table[bi])
            table[bi] = bid
            blocks.append(bid)
            slots.append(pos % bs)
        if n:
            bidx = torch.as_tensor(blocks, dtype=torch.long, device=self.device)
            sidx = torch.as_tensor(slots, dtype=torch.long, device=self.device)
            pool = self.pools[layer]
            pool[bidx, 0, :, sidx] = k.permute(1, 0, 2).to(self.device, self.dtype)
            pool[bidx, 1, :, sidx] = v.permute(1, 0, 2).to(self.device, self.dtype)
        return table, slot_offset + n

    def read_kv(self, layer: int, block_ids: List[int], seq_len: int):
        """K/V ``[H, seq_len, D]`` of a 16-bit pool gathered through the table
        (``block_allocator.py:178-206``); int8 pools: see ``read_dequant``."""
        if self.dtype == torch.int8:
            return self.read_dequant(layer, block_ids, seq_len)
        idx = torch.as_tensor(block_ids, dtype=torch.long, device=self.device)
        g = self.pools[layer][idx]
        n, H, bs, D = g.shape[0], self.num_heads, self.block_size, self.head_dim
        k = g[:, 0].permute(1, 0, 2, 3).reshape(H, n * bs, D)[:, :seq_len]
        v = g[:, 1].permute(1, 0, 2, 3).reshape(H, n * bs, D)[:, :seq_len]
        return k, v

    def read_dequant(self, layer: int, block_ids: List[int], seq_len: int):
        """float16 K/V ``[H, seq_len, D]`` exactly as the reference's dequantise+gather."""
        idx = torch.as_tensor(block_ids, dtype=torch.long, device=self.device)
        g = self.pools[layer][idx]                                 # [n, 2, H, bs, D]
        n, H, bs, D = g.shape[0], self.num_heads, self.block_size, self.head_dim
        kq = g[:, 0].permute(1, 0, 2, 3).reshape(H, n * bs, D)[:, :seq_len]
        vq = g[:, 1].permute(1, 0, 2, 3).reshape(H, n * bs, D)[:, :seq_len]
        ks = self.k_scale16[layer][idx].permute(1, 0, 2).reshape(H, n * bs)[:, :seq_len]
        vs = self.v_scale16[layer][idx][torch.arange(seq_len, device=self.device) // bs]
        k = kq.to(torch.float16) * ks.unsqueeze(-1)
        v = vq.to(torch.float16) * vs.permute(1, 0, 2)
        return k, v


class DeviceChunkMapper:
    """``ChunkBlockMapper`` over a ``DeviceBlockAllocator``."""

    def __init__(self, allocator: DeviceBlockAllocator) -> None:
        self.allocator = allocator
        self._chunk_blocks: Dict[str, List[int]] = {}
        self._lock = threading.Lock()

    def load_chunk(self, chunk_id: str, layers_kv: Sequence[Tuple[torch.Tensor, torch.Tensor]],
                   quantized: Optional[Sequence[tuple]] = None) -> List[int]:
        """Store a chunk (per layer (K, V) ``[1, H, S, D]``, or already-quantised
        layers ``(key_q, key_scale, val_q, val_scale)``) and return its blocks."""
        with self._lock:
            if chunk_id in self._chunk_blocks:
                return self.allocator.fork(self._chunk_blocks[chunk_id])
        bs = self.allocator.block_size
        if self.allocator.dtype != torch.int8:   # 16-bit pool: the chunk as is
            S = layers_kv[0][0].shape[-2]
            block_ids = self.allocator.allocate((S + bs - 1) // bs)
            for layer, (k, v) in enumerate(layers_kv):
                self.allocator.write_chunk(layer, block_ids, k, v)
            with self._lock:
                self._chunk_blocks[chunk_id] = block_ids
            return list(block_ids)
        if quantized is None:
            quantized = [quantize_chunk_int8(k, v) for k, v in layers_kv]
        S = quantized[0][0].shape[-2]
        block_ids = self.allocator.allocate((S + bs - 1) // bs)
        for layer, (kq, ks, vq, vs) in enumerate(quantized):
            self.allocator.write_chunk_int8(layer, block_ids, kq, ks, vq, vs)
        with self._lock:
            self._chunk_blocks[chunk_id] = block_ids
        return list(block_ids)

    def build_block_table(self, chunks) -> List[int]:
        """Concatenate the chunks' block lists in order (``chunk_to_blocks.py:105-125``)."""
        table: List[int] = []
        for chunk_id, layers_kv in chunks:
            table.extend(self.load_chunk(chunk_id, layers_kv))
        return table

    def on_evict(self, chunk_id: str) -> None:
        with self._lock:
            ids = self._chunk_blocks.pop(chunk_id, None)
        if ids is not None:
            self.allocator.free(ids)

    def loaded_chunks(self) -> int:
        return len(self._chunk_blocks)

    def blocks_used_by_chunks(self) -> int:
        with self._lock:
            return sum(len(v) for v in self._chunk_blocks.values())


def _workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    """Scratch for the materialised-prefix strategy, taken from torch's caching
    allocator on the current stream for this call only: its reuse is ordered on
    that stream, so calls on concurrent streams never share a workspace."""
    return torch.empty(nbytes, dtype=torch.uint8, device=device)


def block_table_tensor(tables: Sequence[Sequence[int]], device) -> torch.Tensor:
    """Pad per-sequence tables into a device int32 ``[B, max_blocks]`` array."""
    mb = max(1, max(len(t) for t in tables))
    out = torch.zeros(len(tables), mb, dtype=torch.int32)
    for i, t in enumerate(tables):
        if t:
            out[i, :len(t)] = torch.as_tensor(t, dtype=torch.int32)
    return out.to(device)


def paged_prefill_attention(q: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor,
                            allocator: DeviceBlockAllocator, layer: int,
                            block_tables: torch.Tensor, prefix_len: int,
                            prefix_lens: Optional[torch.Tensor] = None,
                            softmax_scale: Optional[float] = None, causal: bool = True,
                            out: Optional[torch.Tensor] = None, return_lse: bool = True,
                            fused_only: bool = False):
    """Suffix prefill over an int8 paged prefix (``kvb_paged_prefill_fwd``).

    When each KV tile would be dequantised by many CTAs (long suffixes under
    GQA) the library asks for a workspace and dequantises the prefix once
    into it; ``fused_only=True`` forces the fused gather+dequant path.

    q: ``[B, Hq, q_len, D]``; k_new/v_new: the suffix's own ``[B, Hkv, q_len, D]``;
    block_tables: device int32 ``[B, max_blocks]``; ``prefix_len``: cached tokens
    (``prefix_lens`` device int32 ``[B]`` for per-sequence lengths, with
    ``prefix_len`` their maximum).  Sequence b attends to its prefix followed by
    its suffix, bottom-right causal.  Returns ``(o, lse)``.
    """
    _check_tensor("q", q, 4)
    _check_tensor("k_new", k_new, 4)
    _check_tensor("v_new", v_new, 4)
    B, Hq, Sq, D = q.shape
    if k_new.shape != v_new.shape or k_new.shape[0] != B or k_new.shape[2] != Sq or k_new.shape[3] != D:
        raise RuntimeError("k_new/v_new must be [B, Hkv, q_len, D] matching q")
    Hkv = k_new.shape[1]
    if Hkv != allocator.num_heads or D != allocator.head_dim:
        raise RuntimeError("pool heads / head_dim do not match the query")
    if block_tables.dtype != torch.int32 or not block_tables.is_cuda or block_tables.dim() != 2 \
            or not block_tables.is_contiguous():
        raise RuntimeError("block_tables must be a contiguous 2-D int32 CUDA tensor")
    if softmax_scale is None:
        softmax_scale = 1.0 / math.sqrt(D)
    if out is None:
        out = torch.empty_like(q)
    lse = torch.empty(B, Hq, Sq, dtype=torch.float32, device=q.device) if return_lse else None
    p = _lib.KvbPagedPrefillParams()
    p.dtype = _DTYPES[q.dtype]
    p.head_dim, p.batch, p.num_q_heads, p.num_kv_heads = D, B, Hq, Hkv
    p.q_len, p.causal, p.softmax_scale = Sq, 1 if causal else 0, float(softmax_scale)
    p.q, p.o = q.data_ptr(), out.data_ptr()
    p.lse = lse.data_ptr() if lse is not None else None
    p.q_batch_stride, p.q_head_stride, p.q_row_stride = q.stride(0), q.stride(1), q.stride(2)
    p.o_batch_stride, p.o_head_stride, p.o_row_stride = out.stride(0), out.stride(1), out.stride(2)
    if lse is not None:
        p.lse_batch_stride, p.lse_head_stride = lse.stride(0), lse.stride(1)
    p.k_new, p.v_new = k_new.data_ptr(), v_new.data_ptr()
    p.k_new_batch_stride, p.k_new_head_stride, p.k_new_row_stride = k_new.stride()[:3]
    p.v_new_batch_stride, p.v_new_head_stride, p.v_new_row_stride = v_new.stride()[:3]
    p.kv_pool = allocator.pools[layer].data_ptr()
    p.pool_format = allocator.pool_format
    if allocator.dtype == torch.int8:
        p.k_scale = allocator.k_scale[layer].data_ptr()
        p.v_scale = allocator.v_scale[layer].data_ptr()
    elif allocator.dtype != k_new.dtype:
        raise RuntimeError("a 16-bit pool must hold the compute dtype")
    p.num_blocks, p.block_size = allocator.num_blocks, allocator.block_size
    p.block_tables, p.max_blocks_per_seq = block_tables.data_ptr(), block_tables.shape[1]
    p.prefix_len = int(prefix_len)
    p.prefix_lens = prefix_lens.data_ptr() if prefix_lens is not None else None
    p.status = status_word(q.device).data_ptr()
    lib = _lib.load()
    need = int(lib.kvb_paged_prefill_workspace_bytes(p)) if fused_only is False else 0
    if need > 0:
        ws = _workspace(q.device, need)
        p.workspace, p.workspace_bytes = ws.data_ptr(), ws.numel()
    with torch.cuda.device(q.device):
        rc = lib.kvb_paged_prefill_fwd(p, _stream_handle(q.device))
    _lib.check(rc, "kvb_paged_prefill_fwd")
    return out, lse


def paged_prefill_attention_noalloc(q: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor,
                                    allocator: DeviceBlockAllocator, layer: int,
                                    block_tables: torch.Tensor, prefix_len: int,
                                    out: torch.Tensor, lse: Optional[torch.Tensor] = None,
                                    prefix_lens: Optional[torch.Tensor] = None,
                                    softmax_scale: Optional[float] = None, causal: bool = True,
                                    status: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``paged_prefill_attention`` through ``kvb_paged_prefill_fwd_noalloc``.

    For callers that must not allocate device memory while a request runs
    (memory planned up front, or a caching-allocator pool that must not grow):
    nothing is allocated here or in the library.  ``out`` (and ``lse``
    ``[B, Hq, q_len]`` float32, if wanted) are the caller's; ``status`` is an
    optional preallocated int32 word the kernels OR wait-timeout bits into.
    The prefix is always dequantised into the library's static 32 MiB
    per-device scratch, so ``2 * B * Hkv * round_up(prefix_len + q_len, 128) *
    D * 2`` bytes must fit in it.  Calls that overlap in time share that
    scratch and race; the first call on a device must precede any stream
    capture.  Returns ``out``.
    """
    _check_tensor("q", q, 4)
    _check_tensor("k_new", k_new, 4)
    _check_tensor("v_new", v_new, 4)
    _check_tensor("out", out, 4)
    B, Hq, Sq, D = q.shape
    if k_new.shape != v_new.shape or k_new.shape[0] != B or k_new.shape[2] != Sq or k_new.shape[3] != D:
        raise RuntimeError("k_new/v_new must be [B, Hkv, q_len, D] matching q")
    if out.shape != q.shape or out.dtype != q.dtype:
        raise RuntimeError("out must match q in shape and dtype")
    Hkv = k_new.shape[1]
    if Hkv != allocator.num_heads or D != allocator.head_dim:
        raise RuntimeError("pool heads / head_dim do not match the query")
    if block_tables.dtype != torch.int32 or not block_tables.is_cuda or block_tables.dim() != 2 \
            or not block_tables.is_contiguous():
        raise RuntimeError("block_tables must be a contiguous 2-D int32 CUDA tensor")
    if lse is not None and (lse.dtype != torch.float32 or tuple(lse.shape) != (B, Hq, Sq)
                            or lse.stride(2) != 1):
        raise RuntimeError("lse must be float32 [B, Hq, q_len] with contiguous rows")
    if softmax_scale is None:
        softmax_scale = 1.0 / math.sqrt(D)
    p = _lib.KvbPagedPrefillParams()
    p.dtype = _DTYPES[q.dtype]
    p.head_dim, p.batch, p.num_q_heads, p.num_kv_heads = D, B, Hq, Hkv
    p.q_len, p.causal, p.softmax_scale = Sq, 1 if causal else 0, float(softmax_scale)
    p.q, p.o = q.data_ptr(), out.data_ptr()
    p.lse = lse.data_ptr() if lse is not None else None
    p.q_batch_stride, p.q_head_stride, p.q_row_stride = q.stride(0), q.stride(1), q.stride(2)
    p.o_batch_stride, p.o_head_stride, p.o_row_stride = out.stride(0), out.stride(1), out.stride(2)
    if lse is not None:
        p.lse_batch_stride, p.lse_head_stride = lse.stride(0), lse.stride(1)
    p.k_new, p.v_new = k_new.data_ptr(), v_new.data_ptr()
    p.k_new_batch_stride, p.k_new_head_stride, p.k_new_row_stride = k_new.stride()[:3]
    p.v_new_batch_stride, p.v_new_head_stride, p.v_new_row_stride = v_new.stride()[:3]
    p.kv_pool = allocator.pools[layer].data_ptr()
    p.pool_format = allocator.pool_format
    if allocator.dtype == torch.int8:
        p.k_scale = allocator.k_scale[layer].data_ptr()
        p.v_scale = allocator.v_scale[layer].data_ptr()
    elif allocator.dtype != k_new.dtype:
        raise RuntimeError("a 16-bit pool must hold the compute dtype")
    p.num_blocks, p.block_size = allocator.num_blocks, allocator.block_size
    p.block_tables, p.max_blocks_per_seq = block_tables.data_ptr(), block_tables.shape[1]
    p.prefix_len = int(prefix_len)
    p.prefix_lens = prefix_lens.data_ptr() if prefix_lens is not None else None
    p.status = status.data_ptr() if status is not None else None
    with torch.cuda.device(q.device):
        rc = _lib.load().kvb_paged_prefill_fwd_noalloc(p, _stream_handle(q.device))
    _lib.check(rc, "kvb_paged_prefill_fwd_noalloc")
    return out


def paged_materialize(allocator: DeviceBlockAllocator, layer: int, block_tables: torch.Tensor,
                      prefix_len: int, k_new: torch.Tensor, v_new: torch.Tensor,
                      prefix_lens: Optional[torch.Tensor] = None,
                      workspace: Optional[torch.Tensor] = None):
    """Dense K/V of each sequence: its paged int8 prefix dequantised, then its fresh
    suffix (``kvb_paged_materialize``).

    ``k_new``/``v_new``: ``[B, Hkv, q_len, D]`` in the compute dtype (q_len may be 0
    with ``[B, Hkv, 0, D]`` tensors).  Returns ``(K, V)``, each ``[B, Hkv, kv_pad, D]``
    with ``kv_pad = round_up(prefix_len + q_len, 128)``; sequence b's keys are rows
    ``[0, prefix_len_b + q_len)``, zeros up to the next multiple of 128.  The device
    form of the reference's ``read_kv`` + dequantise + concatenate.
    """
    _check_tensor("k_new", k_new, 4)
    _check_tensor("v_new", v_new, 4)
    if k_new.shape != v_new.shape:
        raise RuntimeError("k_new and v_new must have the same shape")
    B, Hkv, Sq, D = k_new.shape
    if Hkv != allocator.num_heads or D != allocator.head_dim:
        raise RuntimeError("pool heads / head_dim do not match k_new")
    if block_tables.dtype != torch.int32 or not block_tables.is_cuda or block_tables.dim() != 2 \
            or not block_tables.is_contiguous() or block_tables.shape[0] != B:
        raise RuntimeError("block_tables must be a contiguous [B, max_blocks] int32 CUDA tensor")
    kv_pad = (int(prefix_len) + Sq + 127) // 128 * 128
    need = 2 * B * Hkv * kv_pad * D
    if workspace is None:
        workspace = torch.empty(need, dtype=k_new.dtype, device=k_new.device)
    if workspace.dtype != k_new.dtype or workspace.numel() < need or not workspace.is_contiguous():
        raise RuntimeError(f"workspace must be a contiguous {k_new.dtype} tensor of >= {need} elements")
    p = _lib.KvbPagedPrefillParams()
    p.dtype = _DTYPES[k_new.dtype]
    p.head_dim, p.batch, p.num_q_heads, p.num_kv_heads = D, B, Hkv, Hkv
    p.q_len = Sq
    if Sq > 0:
        p.k_new, p.v_new = k_new.data_ptr(), v_new.data_ptr()
        p.k_new_batch_stride, p.k_new_head_stride, p.k_new_row_stride = k_new.stride()[:3]
        p.v_new_batch_stride, p.v_new_head_stride, p.v_new_row_stride = v_new.stride()[:3]
    p.kv_pool = allocator.pools[layer].data_ptr()
    p.pool_format = allocator.pool_format
    if allocator.dtype == torch.int8:
        p.k_scale = allocator.k_scale[layer].data_ptr()
        p.v_scale = allocator.v_scale[layer].data_ptr()
    elif allocator.dtype != k_new.dtype:
        raise RuntimeError("a 16-bit pool must hold the compute dtype")
    p.num_blocks, p.block_size = allocator.num_blocks, allocator.block_size
    p.block_tables, p.max_blocks_per_seq = block_tables.data_ptr(), block_tables.shape[1]
    p.prefix_len = int(prefix_len)
    p.prefix_lens = prefix_lens.data_ptr() if prefix_lens is not None else None
    p.status = status_word(k_new.device).data_ptr()
    p.workspace, p.workspace_bytes = workspace.data_ptr(), workspace.numel() * workspace.element_size()
    with torch.cuda.device(k_new.device):
        rc = _lib.load().kvb_paged_materialize(p, _stream_handle(k_new.device))
    _lib.check(rc, "kvb_paged_materialize")
    kv = workspace[:need].view(2, B, Hkv, kv_pad, D)
    return kv[0], kv[1]


def paged_attention_fwd(query: torch.Tensor, allocator: DeviceBlockAllocator,
                        block_tables: Sequence[Sequence[int]], seq_lens: Sequence[int],
                        layer: int, causal: bool = True, scale: Optional[float] = None,
                        top_left: bool = False) -> torch.Tensor:
    """Paged attention over K/V held entirely in the pool (``paged_attention_fwd``,
    ``cpu_paged/paged_attn_cpu.py:33-108``).

    query ``[B, Hq, Sq, D]``; sequence b attends to the first ``seq_lens[b]`` tokens
    of its block table (GQA over the pool's heads); an empty history gives zeros.
    Masking for ``Sq > 1`` with ``causal``: bottom-right (query i sees keys up to
    ``seq_len - Sq + i``, the queries being the last Sq tokens) by default;
    ``top_left=True`` reproduces the reference's ``is_causal`` SDPA call
    (``:100-104``), which aligns the mask to the first key.  One gather pass
    (dequantising int8 pools) into dense K/V, then the prefill kernel per sequence.
    Returns ``[B, Hq, Sq, D]`` in the query's dtype.
    """
    _check_tensor("query", query, 4)
    B, Hq, Sq, D = query.shape
    if len(block_tables) != B or len(seq_lens) != B:
        raise ValueError("one block table and one seq_len per batch element")
    if Hq % allocator.num_heads or D != allocator.head_dim:
        raise RuntimeError("query heads / head_dim do not match the pool")
    out = torch.zeros_like(query)
    L = [int(x) for x in seq_lens]
    if B == 0 or Sq == 0 or max(L) == 0:
        return out
    dev = query.device
    bt = block_table_tensor([list(t) for t in block_tables], dev)
    plens = torch.tensor(L, dtype=torch.int32, device=dev)
    empty = torch.empty(B, allocator.num_heads, 0, D, dtype=query.dtype, device=dev)
    K, V = paged_materialize(allocator, layer, bt, max(L), empty, empty, prefix_lens=plens)
    from .ops import decode_attention, prefill_attention
    group = Hq // allocator.num_heads
    for b in range(B):
        if L[b] == 0:
            continue
        kb, vb = K[b:b + 1, :, :L[b]], V[b:b + 1, :, :L[b]]
        if Sq <= 16 and Sq * group <= 256 and Sq <= L[b]:
            decode_attention(query[b:b + 1], kb, vb, scale, causal and Sq > 1, out=out[b:b + 1],
                             return_lse=False, top_left=top_left)
        else:
            prefill_attention(query[b:b + 1], kb, vb, scale, causal and Sq > 1, out=out[b:b + 1],
                              return_lse=False, top_left=top_left)
    return out
