"""Oracle: softmax attention with offset-causal masking, GQA, varlen, paged.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

Semantics restated from the reference:

* The reference's CPU path is ``_kvboost_flash_attn`` falling through to
  ``torch.nn.functional.scaled_dot_product_attention``
  (``src/kvboost/flash_attn_ext.py:68-103``; torch 2.11.0 installed, the
  reference pins only ``torch>=2.1.0`` in ``pyproject.toml:24``).  SDPA is the
  published softmax(Q K^T * scale) V.
* Reuse prefill hands SDPA HuggingFace's explicit boolean mask, which is
  bottom-right aligned: key ``j`` is visible to query ``i`` iff
  ``j <= i + (kv_len - q_len)`` (``torch.ones(q, kv).tril(kv - q)``).  For
  ``q_len == kv_len`` this is the reference kernel's ``kv_row > q_row`` mask
  (``src/kvboost/csrc/flash_attn_kernel.cu:148,193``).
* GQA follows ``paged_attn_cpu.py:87-88``: KV head ``h // (Hq // Hkv)`` serves
  query head ``h`` (``repeat_interleave``).
* LSE follows the reference kernel: ``L = log(l) + m`` over the *scaled*
  scores, natural log (``flash_attn_kernel.cu:236-245``).  Rows with no
  visible key produce ``O = 0`` and ``L = -inf``, as the reference kernel's
  ``inv_l = 0`` branch does (``flash_attn_kernel.cu:238``).
"""

from __future__ import annotations

import math
from typing import List, Optional, Sequence, Tuple

import numpy as np


def _as_f(x, dtype):
    x = np.asarray(x)
    return x.astype(dtype, copy=False)


def visible_mask(q_len: int, kv_len: int, causal: bool, top_left: bool = False) -> np.ndarray:
    """Boolean ``[q_len, kv_len]`` mask; True = key visible.

    Bottom-right causal by default; ``top_left=True`` is SDPA's ``is_causal``.
    """
    if not causal:
        return np.ones((q_len, kv_len), dtype=bool)
    off = 0 if top_left else kv_len - q_len
    qi = np.arange(q_len)[:, None]
    kj = np.arange(kv_len)[None, :]
    return kj <= qi + off


def _attend_head(q, k, v, scale, mask):
    """One head: q [Sq,D], k/v [Skv,D] -> (o [Sq,D], lse [Sq])."""
    s = (q @ k.T) * scale
    s = np.where(mask, s, -np.inf)
    m = s.max(axis=1, keepdims=True) if s.shape[1] else np.full((s.shape[0], 1), -np.inf)
    m_safe = np.where(np.isfinite(m), m, 0.0)
    p = np.exp(s - m_safe)
    l = p.sum(axis=1, keepdims=True)
    with np.errstate(divide="ignore", invalid="ignore"):
        o = np.where(l > 0, (p @ v) / np.where(l > 0, l, 1.0), 0.0)
        lse = np.where(l[:, 0] > 0, np.log(np.where(l[:, 0] > 0, l[:, 0], 1.0)) + m_safe[:, 0], -np.inf)
    return o, lse


def attention(q, k, v, scale: Optional[float] = None, causal: bool = True,
              compute_dtype=np.float64, q_chunk: int = 1024,
              top_left: bool = False) -> Tuple[np.ndarray, np.ndarray]:
    """Dense attention oracle.

    q: [B, Hq, Sq, D]; k, v: [B, Hkv, Skv, D] (any float dtype, values taken
    exactly).  Returns ``(o [B,Hq,Sq,D] float32, lse [B,Hq,Sq] float32)``.
    """
    q = _as_f(q, compute_dtype)
    k = _as_f(k, compute_dtype)
    v = _as_f(v, compute_dtype)
    B, Hq, Sq, D = q.shape
    Hkv, Skv = k.shape[1], k.shape[2]
    if Hq % Hkv:
        raise ValueError(f"num_q_heads ({Hq}) must be divisible by num_kv_heads ({Hkv})")
    g = Hq // Hkv
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    mask = visible_mask(Sq, Skv, causal, top_left)
    o = np.zeros((B, Hq, Sq, D), dtype=np.float32)
    lse = np.full((B, Hq, Sq), -np.inf, dtype=np.float32)
    for b in range(B):
        for h in range(Hq):
            kh, vh = k[b, h // g], v[b, h // g]
            for r0 in range(0, Sq, q_chunk):
                r1 = min(Sq, r0 + q_chunk)
                oh, lh = _attend_head(q[b, h, r0:r1], kh, vh, scale, mask[r0:r1])
                o[b, h, r0:r1] = oh
                lse[b, h, r0:r1] = lh
    return o, lse


def attention_varlen(q, k, v, cu_seqlens_q: Sequence[int], cu_seqlens_k: Sequence[int],
                     scale: Optional[float] = None, causal: bool = True,
                     compute_dtype=np.float64) -> Tuple[np.ndarray, np.ndarray]:
    """Packed varlen oracle.

    q: [Tq, Hq, D], k/v: [Tk, Hkv, D]; request ``i`` owns rows
    ``cu_seqlens_q[i]:cu_seqlens_q[i+1]`` of q and the matching rows of k/v.
    Each request is masked with its own bottom-right offset, as the
    reference does per request.  Returns ``(o [Tq,Hq,D], lse [Hq,Tq])``.
    """
    q = _as_f(q, compute_dtype)
    k = _as_f(k, compute_dtype)
    v = _as_f(v, compute_dtype)
    Tq, Hq, D = q.shape
    Hkv = k.shape[1]
    g = Hq // Hkv
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    o = np.zeros((Tq, Hq, D), dtype=np.float32)
    lse = np.full((Hq, Tq), -np.inf, dtype=np.float32)
    for i in range(len(cu_seqlens_q) - 1):
        q0, q1 = int(cu_seqlens_q[i]), int(cu_seqlens_q[i + 1])
        k0, k1 = int(cu_seqlens_k[i]), int(cu_seqlens_k[i + 1])
        if q1 == q0:
            continue
        mask = visible_mask(q1 - q0, k1 - k0, causal)
        for h in range(Hq):
            oh, lh = _attend_head(q[q0:q1, h], k[k0:k1, h // g], v[k0:k1, h // g], scale, mask)
            o[q0:q1, h] = oh
            lse[h, q0:q1] = lh
    return o, lse


def paged_attention_topleft(query, k_hist: List[np.ndarray], v_hist: List[np.ndarray],
                            scale: Optional[float] = None, causal: bool = True,
                            compute_dtype=np.float64) -> np.ndarray:
    """Restates ``paged_attention_fwd`` (``cpu_paged/paged_attn_cpu.py:33-108``).

    ``k_hist[b]``/``v_hist[b]`` are the gathered ``[Hkv, kv_len, D]`` histories.
    Causality here is SDPA's ``is_causal`` (top-left aligned) and applies only
    when ``Sq > 1`` (``paged_attn_cpu.py:103``); empty history gives zeros
    (``paged_attn_cpu.py:74-76``).
    """
    query = _as_f(query, compute_dtype)
    B, Hq, Sq, D = query.shape
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    out = np.zeros((B, Hq, Sq, D), dtype=np.float32)
    for b in range(B):
        kb = _as_f(k_hist[b], compute_dtype)
        vb = _as_f(v_hist[b], compute_dtype)
        Hkv, kv_len = kb.shape[0], kb.shape[1]
        if kv_len == 0:
            continue
        g = Hq // Hkv
        if causal and Sq > 1:
            mask = np.arange(kv_len)[None, :] <= np.arange(Sq)[:, None]
        else:
            mask = np.ones((Sq, kv_len), dtype=bool)
        for h in range(Hq):
            oh, _ = _attend_head(query[b, h], kb[h // g], vb[h // g], scale, mask)
            out[b, h] = oh
    return out


def causal_pairs(q_len: int, kv_len: int, causal: bool = True) -> int:
    """Number of visible (query, key) pairs under bottom-right causality."""
    if not causal:
        return q_len * kv_len
    off = kv_len - q_len
    total = 0
    # rows i with i + off + 1 keys visible, clipped to [0, kv_len]
    for i in range(q_len):
        total += max(0, min(kv_len, i + off + 1))
    return total


def attention_flops(q_lens, kv_lens, num_q_heads: int, head_dim: int, causal: bool = True) -> int:
    """Algorithmic FLOPs: 4 * D * Hq * sum(visible pairs) (QK^T and PV, 2 FLOP/MAC)."""
    pairs = sum(causal_pairs(int(a), int(b), causal) for a, b in zip(q_lens, kv_lens))
    return 4 * head_dim * num_q_heads * pairs
