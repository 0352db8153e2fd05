"""The reference's CPU attention path as torch calls (the timed CPU baseline).

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``): the CPU leg of
``bench.py`` and its ``--impl reference`` arm time these functions, and
``tests/test_oracle_golden.py`` pins them to the reference's own outputs.

On CPU tensors, KVBoost's ``_kvboost_flash_attn`` is one call of
``torch.nn.functional.scaled_dot_product_attention`` with the caller's mask and
``is_causal = causal and mask is None`` (``src/kvboost/flash_attn_ext.py:97-103``);
it takes K/V with the query's head count.  A reuse prefill reaches it from
HuggingFace with K/V expanded by ``repeat_interleave`` and HF's bottom-right
boolean mask ``ones(q, kv).tril(kv - q)``; the paged path gathers the prefix
with ``BlockAllocator.read_kv`` (``src/kvboost/cpu_paged/block_allocator.py:178-206``)
after ``dequantize_kv`` (``src/kvboost/kv_quantize.py:102-109``: int8 to
float16 times the float16 scale).  These functions make exactly those torch
calls, in the inputs' own 16-bit dtype, so timing them times the reference's
CPU arithmetic (torch's SDPA kernels on all host threads), not a
restatement of it in another library.
"""

from __future__ import annotations

import math
from typing import Optional, Sequence

import torch
import torch.nn.functional as F


def kvboost_flash_attn_cpu(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float,
                           causal: bool = True,
                           attn_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``_kvboost_flash_attn`` on CPU tensors (``flash_attn_ext.py:97-103``)."""
    return F.scaled_dot_product_attention(q, k, v, attn_mask=attn_mask, scale=scale,
                                          is_causal=(causal and attn_mask is None))


def reuse_prefill(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float) -> torch.Tensor:
    """One reuse prefill as HF hands it to the dispatcher: ``[B, Hq, Sq, D]`` queries over
    ``[B, Hkv, Skv, D]`` keys, GQA expanded, bottom-right mask when ``Sq != Skv``."""
    rep = q.shape[1] // k.shape[1]
    if rep > 1:
        k = k.repeat_interleave(rep, dim=1)
        v = v.repeat_interleave(rep, dim=1)
    sq, skv = q.shape[2], k.shape[2]
    if sq == skv:
        return kvboost_flash_attn_cpu(q, k, v, scale, True)
    mask = torch.ones(sq, skv, dtype=torch.bool).tril(skv - sq)
    return kvboost_flash_attn_cpu(q, k, v, scale, True, attn_mask=mask)


def dequantize_int8(q: torch.Tensor, scale_f16: torch.Tensor) -> torch.Tensor:
    """``_dequantize_int8`` (``kv_quantize.py:102-109``): float16 product."""
    return q.to(torch.float16) * scale_f16


def read_kv(pool: torch.Tensor, block_ids: Sequence[int], seq_len: int):
    """``BlockAllocator.read_kv`` (``block_allocator.py:178-206``) on one layer's pool
    ``[num_blocks, 2, H, block, D]``: K, V ``[H, seq_len, D]``."""
    blocks = pool[list(block_ids)]                       # [n, 2, H, bs, D]
    n, _, h, bs, d = blocks.shape
    k = blocks[:, 0].permute(1, 0, 2, 3).reshape(h, n * bs, d)[:, :seq_len]
    v = blocks[:, 1].permute(1, 0, 2, 3).reshape(h, n * bs, d)[:, :seq_len]
    return k, v


def default_scale(d: int) -> float:
    return 1.0 / math.sqrt(d)
