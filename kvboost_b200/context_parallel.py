"""Context-parallel reuse prefill over a chunk-sharded int8 paged pool.

For one very long prompt whose cached 128-token chunks are spread over the GPUs
of a box (chunk c on rank ``c % G``, at local chunk slot ``c // G``), every rank:

1. all-gathers the pool shards (int8 K/V blocks and their fp32 scales) over
   NVLink with NCCL, so each rank holds the whole reused prefix;
2. all-gathers the suffix's own K/V (each rank projected the K/V of its own
   query rows) and puts it back in token order;
3. dequantises + gathers prefix and suffix once into dense K/V
   (``kvb_paged_materialize``);
4. runs the prefill for its causally balanced share of the query rows over all
   heads: the suffix is cut into 2G equal chunks and rank r takes chunks r and
   2G-1-r (zig-zag), each a dense launch whose key range ends at its own last
   row (bottom-right causal over prefix + suffix).

Outputs stay sharded by query rows.  When the pool is sharded by KV head
instead, ``bench.py --workload paged_long`` splits the heads with no
collective at all; this module serves pools placed by chunk.
"""

from __future__ import annotations

import ctypes
from typing import List, Optional, Sequence, Tuple

import torch

from . import _lib
from .ops import _DTYPES, _stream_handle, prefill_attention, status_word
from .paged import DeviceBlockAllocator, block_table_tensor, paged_materialize

CHUNK_TOKENS = 128
BLOCKS_PER_CHUNK = CHUNK_TOKENS // 16


def local_chunk_slots(num_chunks: int, world: int, rank: int) -> List[int]:
    """Global chunk ids this rank stores, in local slot order."""
    return list(range(rank, num_chunks, world))


def shard_chunks(num_chunks: int, world: int) -> int:
    """Chunk slots every rank's shard reserves (the largest rank's count)."""
    return (num_chunks + world - 1) // world


def gathered_block_table(num_chunks: int, world: int) -> List[int]:
    """Block ids of the prefix in the gathered pool, token order.

    Rank r's shard occupies gathered blocks ``[r * n, (r + 1) * n)`` with
    ``n = shard_chunks * 8``; chunk c sits at local slot ``c // world``.
    """
    nlb = shard_chunks(num_chunks, world) * BLOCKS_PER_CHUNK
    table = []
    for c in range(num_chunks):
        base = (c % world) * nlb + (c // world) * BLOCKS_PER_CHUNK
        table.extend(range(base, base + BLOCKS_PER_CHUNK))
    return table


def zigzag_chunks(q_len: int, world: int, rank: int) -> List[Tuple[int, int]]:
    """This rank's two query-row ranges: chunks r and 2G-1-r of 2G equal chunks."""
    n = 2 * world
    if q_len % n:
        raise ValueError(f"q_len {q_len} must split into {n} equal chunks")
    c = q_len // n
    return [(rank * c, (rank + 1) * c), ((n - 1 - rank) * c, (n - rank) * c)]


def zigzag_token_index(q_len: int, world: int) -> torch.Tensor:
    """Row index that puts all-gathered zig-zag rows (rank-major, two chunks per
    rank) back in token order."""
    n = 2 * world
    c = q_len // n
    src = torch.empty(q_len, dtype=torch.long)
    for r in range(world):
        for j, (s, e) in enumerate(zigzag_chunks(q_len, world, r)):
            src[s:e] = torch.arange((2 * r + j) * c, (2 * r + j + 1) * c)
    return src


def make_shard_allocator(num_chunks: int, world: int, num_heads: int, head_dim: int,
                         device) -> DeviceBlockAllocator:
    """An empty one-layer pool sized for this rank's shard of ``num_chunks`` chunks."""
    return DeviceBlockAllocator(1, num_heads, head_dim,
                                shard_chunks(num_chunks, world) * BLOCKS_PER_CHUNK, device=device)


def gather_pool(local: DeviceBlockAllocator, full: DeviceBlockAllocator, layer: int = 0,
                group=None) -> None:
    """All-gather every rank's shard of ``layer`` into ``full`` (layer 0), NCCL.

    ``full`` must have ``world * local.num_blocks`` blocks.  The int8 blocks and
    the fp32 scales the kernels read are gathered; the fp16 scale copies are not.
    """
    import torch.distributed as dist
    world = dist.get_world_size(group)
    if full.num_blocks != world * local.num_blocks:
        raise ValueError("full pool must hold world * local blocks")
    _all_gather(full.pools[0], local.pools[layer], group)
    _all_gather(full.k_scale[0], local.k_scale[layer], group)
    _all_gather(full.v_scale[0], local.v_scale[layer], group)


def _all_gather(out: torch.Tensor, inp: torch.Tensor, group=None) -> None:
    """Concatenate every rank's ``inp`` along dim 0 into ``out`` (NCCL: one
    all_gather_into_tensor; other backends: all_gather of a list)."""
    import torch.distributed as dist
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(out, inp, group=group)
    else:
        dist.all_gather(list(out.chunk(dist.get_world_size(group))), inp, group=group)


def gather_suffix_kv(k_local: torch.Tensor, v_local: torch.Tensor, q_len: int,
                     group=None, index: Optional[torch.Tensor] = None):
    """All-gather the suffix K/V rows of every rank's zig-zag chunks and return them
    in token order, ``[1, Hkv, q_len, D]`` each."""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    _, Hkv, rows, D = k_local.shape
    kv = torch.stack([k_local[0], v_local[0]]).permute(2, 0, 1, 3).contiguous()  # [rows, 2, Hkv, D]
    buf = torch.empty(world * rows, 2, Hkv, D, dtype=k_local.dtype, device=k_local.device)
    _all_gather(buf, kv, group)
    if index is None:
        index = zigzag_token_index(q_len, world).to(k_local.device)
    full = buf.index_select(0, index)                        # token order
    full = full.permute(1, 2, 0, 3)                          # [2, Hkv, q_len, D]
    return full[0].unsqueeze(0), full[1].unsqueeze(0)


def cp_rank_prefill(q_local: torch.Tensor, full_pool: DeviceBlockAllocator,
                    k_full: torch.Tensor, v_full: torch.Tensor, prefix_len: int, q_len: int,
                    world: int, rank: int, softmax_scale: Optional[float] = None,
                    out: Optional[torch.Tensor] = None, workspace: Optional[torch.Tensor] = None,
                    table: Optional[torch.Tensor] = None) -> torch.Tensor:
    """The compute of one rank once the pool and the suffix K/V are gathered:
    dequantise prefix + suffix once, then one bottom-right-causal launch per
    zig-zag query chunk, each over the keys up to its own last row."""
    if prefix_len % CHUNK_TOKENS:
        raise ValueError("the reused prefix is whole 128-token chunks")
    if table is None:
        table = block_table_tensor([gathered_block_table(prefix_len // CHUNK_TOKENS, world)],
                                   q_local.device)
    K, V = paged_materialize(full_pool, 0, table, prefix_len, k_full, v_full,
                             workspace=workspace)
    return zigzag_prefill(q_local, K, V, prefix_len, q_len, world, rank, softmax_scale, out)


def zigzag_prefill(q_local: torch.Tensor, K: torch.Tensor, V: torch.Tensor, prefix_len: int,
                   q_len: int, world: int, rank: int, softmax_scale: Optional[float] = None,
                   out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """One bottom-right-causal launch per zig-zag query chunk of this rank, each over
    the dense keys up to its own last row."""
    if out is None:
        out = torch.empty_like(q_local)
    c = q_len // (2 * world)
    for j, (s, e) in enumerate(zigzag_chunks(q_len, world, rank)):
        kv_len = prefix_len + e
        prefill_attention(q_local[:, :, j * c:(j + 1) * c], K[:, :, :kv_len], V[:, :, :kv_len],
                          softmax_scale, True, out=out[:, :, j * c:(j + 1) * c],
                          return_lse=False)
    return out


BARRIER_TIMEOUT_NS = 2_000_000_000


def peer_barrier(signal_slots: Sequence[int], rank: int, epoch: int, device,
                 timeout_ns: int = BARRIER_TIMEOUT_NS,
                 status: Optional[torch.Tensor] = None) -> None:
    """``kvb_peer_barrier`` on the current stream of ``device``: ``signal_slots[r]`` is
    rank r's signal array (``world`` int32 words) as mapped here.  A wait that runs
    out ORs ``KVB_STATUS_PEER_WAIT`` into the status word (read it with
    ``ops.read_status``); the call itself never blocks the host."""
    sig = _lib.KvbPeerSignals()
    for r, ptr in enumerate(signal_slots):
        sig.slot[r] = ptr
    sig.world, sig.rank = len(signal_slots), rank
    st = status if status is not None else status_word(torch.device(device))
    with torch.cuda.device(device):
        rc = _lib.load().kvb_peer_barrier(sig, epoch, timeout_ns, st.data_ptr(),
                                          _stream_handle(torch.device(device)))
    _lib.check(rc, "kvb_peer_barrier")


class PeerShardBuffer:
    """This rank's shard of a context-parallel prompt, in memory the other ranks
    read directly over NVLink.

    One buffer (``kvb_peer_shard_layout``) holds the rank's prefix chunks as an
    int8 pool (``.alloc``, a one-layer ``DeviceBlockAllocator`` whose pool and
    fp32 scales are views of the buffer) and the suffix K/V of its zig-zag query
    rows (``.suffix_k`` / ``.suffix_v``, ``[Hkv, 2c, D]``).  With ``symmetric``
    the buffer comes from torch's symmetric memory and is mapped into every rank
    (``.bases`` = every rank's buffer address in this process); otherwise it is
    plain device memory and the caller supplies the bases (one process holding
    several ranks' shards).
    """

    def __init__(self, num_chunks: int, world: int, num_kv_heads: int, head_dim: int,
                 q_len: int, dtype=torch.bfloat16, device="cuda", group=None,
                 symmetric: bool = True):
        self.world = world
        self.num_chunks = num_chunks
        self.shard_blocks = shard_chunks(num_chunks, world) * BLOCKS_PER_CHUNK
        if q_len % (2 * world):
            raise ValueError(f"q_len {q_len} must split into {2 * world} equal chunks")
        self.zz_rows = q_len // (2 * world)
        self.q_len, self.dtype = q_len, dtype
        off = (ctypes.c_int64 * 5)()
        total = _lib.load().kvb_peer_shard_layout(num_kv_heads, head_dim, self.shard_blocks,
                                                  self.zz_rows, off)
        if total < 0:
            raise ValueError("unsupported shard geometry")
        self.offsets = list(off)
        self.handle = None
        self.epoch = 0
        if symmetric:
            import torch.distributed as dist
            import torch.distributed._symmetric_memory as symm_mem
            self.buf = symm_mem.empty(total, dtype=torch.uint8, device=device)
            grp = group if group is not None else dist.group.WORLD
            self.handle = symm_mem.rendezvous(self.buf, grp)
            self.bases = [int(p) for p in self.handle.buffer_ptrs]
            # the barrier's signal words: one int32 per rank, zero before the first use
            self.sig = symm_mem.empty(8, dtype=torch.int32, device=device)
            self.sig.zero_()
            self.sig_handle = symm_mem.rendezvous(self.sig, grp)
            self.sig_slots = [int(p) for p in self.sig_handle.buffer_ptrs]
            self.rank = dist.get_rank(grp)
            torch.cuda.synchronize(device)
            dist.barrier(group=grp)
        else:
            self.buf = torch.zeros(total, dtype=torch.uint8, device=device)
            self.bases = [self.buf.data_ptr()]
        H, D, sb, r2 = num_kv_heads, head_dim, self.shard_blocks, 2 * self.zz_rows
        b = self.buf
        self.alloc = DeviceBlockAllocator(1, H, D, sb, device=device)
        self.alloc.pools[0] = b[off[0]:off[1]].view(torch.int8).view(sb, 2, H, 16, D)
        self.alloc.k_scale[0] = b[off[1]:off[2]].view(torch.float32).view(sb, H, 16)
        self.alloc.v_scale[0] = b[off[2]:off[3]].view(torch.float32).view(sb, H, D)
        self.suffix_k = b[off[3]:off[4]].view(dtype).view(H, r2, D)
        self.suffix_v = b[off[4]:total].view(dtype).view(H, r2, D)

    def barrier(self, timeout_ms: int = 2000) -> None:
        """Every rank's writes to its shard buffer are visible to the others after this:
        ``kvb_peer_barrier`` over the ranks' signal words, enqueued on the current
        stream.  A rank that does not arrive within the timeout makes the others'
        barrier kernels give up and set ``KVB_STATUS_PEER_WAIT`` in their status
        words instead of hanging."""
        if self.handle is not None:
            self.epoch += 1
            peer_barrier(self.sig_slots, self.rank, self.epoch, self.buf.device,
                         timeout_ns=int(timeout_ms) * 1_000_000)


def materialize_from_peers(bases: Sequence[int], shard_blocks: int, zz_rows: int,
                           num_kv_heads: int, head_dim: int, dtype, table: torch.Tensor,
                           prefix_len: int, q_len: int, num_blocks: int,
                           workspace: Optional[torch.Tensor] = None):
    """Dense K/V of the whole prompt read from every rank's shard buffer in place
    (``kvb_paged_materialize_peers``); returns ``(K, V)`` ``[1, Hkv, kv_pad, D]``."""
    world = len(bases)
    kv_pad = (int(prefix_len) + q_len + 127) // 128 * 128
    need = 2 * num_kv_heads * kv_pad * head_dim
    dev = table.device
    if workspace is None:
        workspace = torch.empty(need, dtype=dtype, device=dev)
    if workspace.dtype != dtype or workspace.numel() < need:
        raise RuntimeError(f"workspace must be a {dtype} tensor of >= {need} elements")
    p = _lib.KvbPagedPrefillParams()
    p.dtype = _DTYPES[dtype]
    p.head_dim, p.batch, p.num_q_heads, p.num_kv_heads = head_dim, 1, num_kv_heads, num_kv_heads
    p.q_len, p.prefix_len = q_len, int(prefix_len)
    p.num_blocks, p.block_size = num_blocks, 16
    p.block_tables, p.max_blocks_per_seq = table.data_ptr(), table.shape[1]
    p.status = status_word(dev).data_ptr()
    p.workspace, p.workspace_bytes = workspace.data_ptr(), workspace.numel() * workspace.element_size()
    sh = _lib.KvbPeerShards()
    for r, ptr in enumerate(bases):
        sh.base[r] = ptr
    sh.world, sh.shard_blocks, sh.zigzag_rows = world, shard_blocks, zz_rows
    with torch.cuda.device(dev):
        rc = _lib.load().kvb_paged_materialize_peers(p, sh, _stream_handle(dev))
    _lib.check(rc, "kvb_paged_materialize_peers")
    kv = workspace[:need].view(2, 1, num_kv_heads, kv_pad, head_dim)
    return kv[0], kv[1]


def cp_reuse_prefill_peers(q_local: torch.Tensor, shards: PeerShardBuffer, prefix_len: int,
                           rank: int, softmax_scale: Optional[float] = None,
                           out: Optional[torch.Tensor] = None,
                           workspace: Optional[torch.Tensor] = None,
                           table: Optional[torch.Tensor] = None) -> torch.Tensor:
    """This rank's share of a context-parallel reuse prefill with the gather fused
    into the dequantise pass: a cross-GPU barrier, one kernel that reads every
    block and suffix row from its owner's buffer over NVLink into dense K/V, then
    the zig-zag launches.  ``shards.suffix_k/v`` must hold this rank's rows."""
    H, _, D = shards.suffix_k.shape
    if table is None:
        table = block_table_tensor([gathered_block_table(prefix_len // CHUNK_TOKENS, shards.world)],
                                   q_local.device)
    shards.barrier()
    K, V = materialize_from_peers(shards.bases, shards.shard_blocks, shards.zz_rows, H, D,
                                  shards.dtype, table, prefix_len, shards.q_len,
                                  shards.world * shards.shard_blocks, workspace)
    return zigzag_prefill(q_local, K, V, prefix_len, shards.q_len, shards.world, rank,
                          softmax_scale, out)


def cp_reuse_prefill(q_local: torch.Tensor, k_local: torch.Tensor, v_local: torch.Tensor,
                     local_pool: DeviceBlockAllocator, full_pool: DeviceBlockAllocator,
                     prefix_len: int, q_len: int, softmax_scale: Optional[float] = None,
                     group=None, out: Optional[torch.Tensor] = None,
                     workspace: Optional[torch.Tensor] = None,
                     table: Optional[torch.Tensor] = None,
                     index: Optional[torch.Tensor] = None) -> torch.Tensor:
    """This rank's share of a context-parallel reuse prefill.

    q_local: ``[1, Hq, 2c, D]`` the rank's zig-zag query rows (chunk r then chunk
    2G-1-r, c = q_len / 2G); k_local/v_local: ``[1, Hkv, 2c, D]`` the suffix K/V of
    the same rows; ``local_pool``: this rank's shard of the prefix chunks;
    ``full_pool``: receives the gathered pool.  Returns ``[1, Hq, 2c, D]``.
    """
    import torch.distributed as dist
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    gather_pool(local_pool, full_pool, 0, group)
    k_full, v_full = gather_suffix_kv(k_local, v_local, q_len, group, index)
    return cp_rank_prefill(q_local, full_pool, k_full, v_full, prefix_len, q_len, world, rank,
                           softmax_scale, out, workspace, table)
