"""Torch-facing prefill-attention ops over the sm_100a C ABI.

These are thin: they check tensors, allocate outputs with torch, pass data
pointers + element strides + the current CUDA stream to
``kvb_prefill_fwd`` and return.  No host synchronisation, no copies of the
inputs (any row/head/batch strides are accepted as long as the innermost
dimension is contiguous), and no fallback: an input the kernels cannot take
raises.

Layouts
-------
* ``prefill_attention``        q ``[B, Hq, Sq, D]``, k/v ``[B, Hkv, Skv, D]`` as
  views of any layout (HF hands transposed ``[B, S, H, D]`` views).
* ``prefill_attention_varlen`` packed q ``[Tq, Hq, D]``, k/v ``[Tk, Hkv, D]`` with
  int32 ``cu_seqlens`` on the device.
"""

from __future__ import annotations

import math
from typing import Optional, Tuple

import torch

from . import _lib

_DTYPES = {torch.bfloat16: _lib.KVB_DTYPE_BF16, torch.float16: _lib.KVB_DTYPE_FP16}
_status_words = {}


def status_word(device: torch.device) -> torch.Tensor:
    """Per-device int32 word the kernels OR error codes into (bounded waits)."""
    idx = torch.device(device).index
    if idx is None:
        idx = torch.cuda.current_device()
    w = _status_words.get(idx)
    if w is None:
        w = torch.zeros(1, dtype=torch.int32, device=f"cuda:{idx}")
        _status_words[idx] = w
    return w


def read_status(device=None, reset: bool = True) -> int:
    """Synchronise and return the device status word (0 = no wait ever gave up)."""
    w = status_word(device if device is not None else torch.device("cuda"))
    v = int(w.item())
    if reset and v:
        w.zero_()
    return v


def _check_tensor(name, t, ndim):
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if t.dim() != ndim:
        raise RuntimeError(f"{name} must be {ndim}-D, got {t.dim()}")
    if not t.is_cuda:
        raise RuntimeError(f"{name} must be on CUDA (kvboost_b200 has no CPU path)")
    if t.dtype not in _DTYPES:
        raise RuntimeError(f"{name} must be float16 or bfloat16, got {t.dtype}")
    if t.stride(-1) != 1:
        raise RuntimeError(f"{name} must have a contiguous last (head_dim) dimension")


def _stream_handle(device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def prefill_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                      softmax_scale: Optional[float] = None, causal: bool = True,
                      out: Optional[torch.Tensor] = None, return_lse: bool = True,
                      out_layout: str = "bhsd", top_left: bool = False,
                      kernel: str = "auto",
                      ) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
    """Bottom-right causal (or full) attention with GQA.

    ``top_left=True`` selects torch SDPA's ``is_causal`` alignment (key j
    visible to query i iff j <= i) instead of the bottom-right reuse mask.

    q: ``[B, Hq, Sq, D]``; k, v: ``[B, Hkv, Skv, D]``; ``Hq % Hkv == 0``.
    Returns ``(o, lse)``: o in q's dtype, ``[B, Hq, Sq, D]`` (``out_layout="bhsd"``)
    or ``[B, Sq, Hq, D]`` (``"bshd"``, what HF attention functions return);
    lse float32 ``[B, Hq, Sq]`` (natural log) or None.
    ``kernel``: "auto" (``split_key_plan`` decides), "prefill" or "split" to force one.
    """
    _check_tensor("q", q, 4)
    _check_tensor("k", k, 4)
    _check_tensor("v", v, 4)
    if not (q.dtype == k.dtype == v.dtype):
        raise RuntimeError("q, k, v must have the same dtype")
    if not (q.device == k.device == v.device):
        raise RuntimeError("q, k, v must be on the same device")
    B, Hq, Sq, D = q.shape
    Bk, Hkv, Skv, Dk = k.shape
    if v.shape != k.shape:
        raise RuntimeError(f"k/v shape mismatch: {tuple(k.shape)} vs {tuple(v.shape)}")
    if Bk != B or Dk != D:
        raise RuntimeError("batch / head_dim mismatch between q and k")
    if Hq % Hkv:
        raise RuntimeError(f"num_q_heads ({Hq}) must be divisible by num_kv_heads ({Hkv})")
    if D not in (64, 96, 128):
        raise RuntimeError(f"head_dim must be one of 64, 96, 128, got {D}")
    if softmax_scale is None:
        softmax_scale = 1.0 / math.sqrt(D)
    if out is None:
        if out_layout == "bshd":
            out = torch.empty(B, Sq, Hq, D, dtype=q.dtype, device=q.device).transpose(1, 2)
        else:
            out = torch.empty(B, Hq, Sq, D, dtype=q.dtype, device=q.device)
    lse = torch.empty(B, Hq, Sq, dtype=torch.float32, device=q.device) if return_lse else None
    if B == 0 or Sq == 0:
        return (out.transpose(1, 2) if out_layout == "bshd" else out), lse
    if kernel not in ("auto", "prefill", "split"):
        raise RuntimeError(f"kernel must be 'auto', 'prefill' or 'split', got {kernel!r}")
    use_split, splits = split_key_plan(B, Hq, Hkv, Sq, Skv)
    if kernel != "auto":
        use_split = kernel == "split"
        splits = decode_splits(B, Hkv, Skv, packed_rows=(Hq // Hkv) * Sq)
    if use_split:
        # few query tiles over many keys: GQA heads packed per key tile, keys
        # split over CTAs (same results; see split_key_plan)
        o, l = decode_attention(q, k, v, softmax_scale, causal, out=out, return_lse=return_lse,
                                num_splits=splits, top_left=top_left)
        return (o.transpose(1, 2) if out_layout == "bshd" else o), l

    p = _lib.KvbPrefillParams()
    p.dtype = _DTYPES[q.dtype]
    p.head_dim, p.batch, p.num_q_heads, p.num_kv_heads = D, B, Hq, Hkv
    p.q_len, p.kv_len, p.causal = Sq, Skv, (2 if top_left else 1) if causal else 0
    p.softmax_scale = float(softmax_scale)
    p.q, p.k, p.v, p.o = q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr()
    p.lse = lse.data_ptr() if lse is not None else None
    p.q_batch_stride, p.q_head_stride, p.q_row_stride = q.stride(0), q.stride(1), q.stride(2)
    p.k_batch_stride, p.k_head_stride, p.k_row_stride = k.stride(0), k.stride(1), k.stride(2)
    p.v_batch_stride, p.v_head_stride, p.v_row_stride = v.stride(0), v.stride(1), v.stride(2)
    p.o_batch_stride, p.o_head_stride, p.o_row_stride = out.stride(0), out.stride(1), out.stride(2)
    if lse is not None:
        p.lse_batch_stride, p.lse_head_stride = lse.stride(0), lse.stride(1)
    p.status = status_word(q.device).data_ptr()
    with torch.cuda.device(q.device):
        rc = _lib.load().kvb_prefill_fwd(p, _stream_handle(q.device))
    _lib.check(rc, "kvb_prefill_fwd")
    if out_layout == "bshd":
        return out.transpose(1, 2), lse
    return out, lse


def prefill_attention_varlen(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                             cu_seqlens_q: torch.Tensor, cu_seqlens_k: torch.Tensor,
                             max_seqlen_q: int, max_seqlen_k: int,
                             softmax_scale: Optional[float] = None, causal: bool = True,
                             out: Optional[torch.Tensor] = None, return_lse: bool = True):
    """Packed variable-length batch; each sequence has its own bottom-right offset.

    q: ``[Tq, Hq, D]``, k/v: ``[Tk, Hkv, D]``, cu_seqlens: int32 ``[B+1]`` on the
    device; ``max_seqlen_q`` must bound every ``cu_seqlens_q[i+1]-cu_seqlens_q[i]``.
    Returns ``(o [Tq, Hq, D], lse [Hq, Tq] float32 or None)``.
    """
    _check_tensor("q", q, 3)
    _check_tensor("k", k, 3)
    _check_tensor("v", v, 3)
    if not (q.dtype == k.dtype == v.dtype):
        raise RuntimeError("q, k, v must have the same dtype")
    for name, cu in (("cu_seqlens_q", cu_seqlens_q), ("cu_seqlens_k", cu_seqlens_k)):
        if cu.dtype != torch.int32 or not cu.is_cuda or cu.dim() != 1 or not cu.is_contiguous():
            raise RuntimeError(f"{name} must be a contiguous 1-D int32 CUDA tensor")
    if cu_seqlens_q.numel() != cu_seqlens_k.numel() or cu_seqlens_q.numel() < 2:
        raise RuntimeError("cu_seqlens_q and cu_seqlens_k must both have batch+1 >= 2 entries")
    Tq, Hq, D = q.shape
    Tk, Hkv, _ = k.shape
    if Hq % Hkv:
        raise RuntimeError(f"num_q_heads ({Hq}) must be divisible by num_kv_heads ({Hkv})")
    if D not in (64, 96, 128):
        raise RuntimeError(f"head_dim must be one of 64, 96, 128, got {D}")
    B = cu_seqlens_q.numel() - 1
    if softmax_scale is None:
        softmax_scale = 1.0 / math.sqrt(D)
    if out is None:
        out = torch.empty_like(q)
    lse = torch.empty(Hq, Tq, dtype=torch.float32, device=q.device) if return_lse else None
    if Tq == 0 or max_seqlen_q == 0:
        return out, lse
    p = _lib.KvbPrefillParams()
    p.dtype = _DTYPES[q.dtype]
    p.head_dim, p.batch, p.num_q_heads, p.num_kv_heads = D, B, Hq, Hkv
    p.q_len, p.kv_len, p.causal = int(max_seqlen_q), int(max_seqlen_k), 1 if causal else 0
    p.softmax_scale = float(softmax_scale)
    p.total_q, p.total_k = Tq, Tk
    p.q, p.k, p.v, p.o = q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr()
    p.lse = lse.data_ptr() if lse is not None else None
    p.q_head_stride, p.q_row_stride = q.stride(1), q.stride(0)
    p.k_head_stride, p.k_row_stride = k.stride(1), k.stride(0)
    p.v_head_stride, p.v_row_stride = v.stride(1), v.stride(0)
    p.o_head_stride, p.o_row_stride = out.stride(1), out.stride(0)
    if lse is not None:
        p.lse_head_stride = lse.stride(0)
    p.cu_seqlens_q, p.cu_seqlens_k = cu_seqlens_q.data_ptr(), cu_seqlens_k.data_ptr()
    p.status = status_word(q.device).data_ptr()
    with torch.cuda.device(q.device):
        rc = _lib.load().kvb_prefill_fwd(p, _stream_handle(q.device))
    _lib.check(rc, "kvb_prefill_fwd(varlen)")
    return out, lse


def decode_splits(batch: int, num_kv_heads: int, kv_len: int, num_sms: int = 148,
                  packed_rows: int = 1) -> int:
    """Key-range splits for one wave of CTAs (one per SM), at least two 128-key tiles
    per split: a CTA's fixed cost (setup, first tile, epilogue) is several tiles'
    worth, so a second wave or one-tile splits cost more than they parallelise
    (measured on B200 for batch 1-32, 2-8 KV heads, 2K-16K keys).  ``packed_rows``
    = query heads per KV head x query rows; each 256 of them take one CTA per split,
    and when they fit one 128-row tile each CTA runs two splits (one per slot)."""
    tiles = (kv_len + 127) // 128
    pairs = (packed_rows + 255) // 256
    per_cta = 2 if packed_rows <= 128 else 1
    return max(1, min(per_cta * max(1, num_sms // max(1, batch * num_kv_heads * pairs)), tiles // 2))


def split_key_plan(B: int, Hq: int, Hkv: int, Sq: int, Skv: int, num_sms: int = 148):
    """Whether the split-key kernel beats the one-CTA-per-query-tile-pair prefill
    kernel for this shape, and with how many key splits.

    Cost model in key-tile periods of the slowest wave: the prefill kernel gives
    each CTA two 128-row query tiles (two heads of a GQA pair, or two tiles of one
    head) and all their key tiles; the split-key kernel packs the GQA heads' rows
    (two 128-row tiles per CTA) and splits the keys so that one wave fills the
    SMs (two key ranges per CTA when the packed rows fit one tile), plus about
    two periods for the partials' merge.  Short suffixes over long
    reused prefixes (decode, seams, short reuse prefills) take the split-key
    kernel; everything with enough query tiles to fill the GPU keeps the prefill
    kernel."""
    if Sq > Skv or Sq < 1:
        return False, 1
    cdiv = lambda a, b: -(-a // b)
    kt = cdiv(Skv, 128)
    group = Hq // Hkv
    if group % 2 == 0:
        dense_ctas = B * (Hq // 2) * cdiv(Sq, 128)
    else:
        dense_ctas = B * Hq * cdiv(cdiv(Sq, 128), 2)
    dense = cdiv(dense_ctas, num_sms) * kt
    per_split = B * Hkv * cdiv(group * Sq, 256)
    splits = decode_splits(B, Hkv, Skv, num_sms, group * Sq)
    ctas = per_split * (cdiv(splits, 2) if group * Sq <= 128 and splits > 1 else splits)
    split = cdiv(ctas, num_sms) * cdiv(kt, splits) + 2
    return split < 0.75 * dense, splits


def decode_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                     softmax_scale: Optional[float] = None, causal: bool = True,
                     out: Optional[torch.Tensor] = None, return_lse: bool = True,
                     num_splits: Optional[int] = None, top_left: bool = False):
    """Split-key attention for few queries per head over many keys (decode, q = 1,
    the selective-recompute seams and short reuse suffixes): ``kvb_decode_fwd``.

    Same contract as ``prefill_attention`` (q ``[B, Hq, Sq, D]``, k/v ``[B, Hkv, Skv, D]``,
    bottom-right causal), restricted to Sq <= Skv.  The query heads of a GQA group
    are packed as rows (two 128-row tiles per CTA) so that each key tile is read
    once per group and tile pair, and the key range is split over CTAs (one
    wave); a second launch merges the partial results by their LSE.
    """
    _check_tensor("q", q, 4)
    _check_tensor("k", k, 4)
    _check_tensor("v", v, 4)
    if not (q.dtype == k.dtype == v.dtype) or k.shape != v.shape:
        raise RuntimeError("q, k, v dtypes / k, v shapes must match")
    B, Hq, Sq, D = q.shape
    _, Hkv, Skv, _ = k.shape
    if Hq % Hkv:
        raise RuntimeError(f"num_q_heads ({Hq}) must be divisible by num_kv_heads ({Hkv})")
    if softmax_scale is None:
        softmax_scale = 1.0 / math.sqrt(D)
    if Sq > 1 and q.stride(1) != Sq * q.stride(2):
        q = q.contiguous()
    if out is None:
        out = torch.empty(B, Hq, Sq, D, dtype=q.dtype, device=q.device)
    lse = torch.empty(B, Hq, Sq, dtype=torch.float32, device=q.device) if return_lse else None
    if num_splits is None:
        num_splits = decode_splits(B, Hkv, Skv, packed_rows=(Hq // Hkv) * Sq)
    p = _lib.KvbPrefillParams()
    p.dtype = _DTYPES[q.dtype]
    p.head_dim, p.batch, p.num_q_heads, p.num_kv_heads = D, B, Hq, Hkv
    p.q_len, p.kv_len, p.causal = Sq, Skv, (2 if top_left else 1) if causal else 0
    p.softmax_scale = float(softmax_scale)
    p.q, p.k, p.v, p.o = q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr()
    p.lse = lse.data_ptr() if lse is not None else None
    p.q_batch_stride, p.q_head_stride, p.q_row_stride = q.stride(0), q.stride(1), q.stride(2)
    p.k_batch_stride, p.k_head_stride, p.k_row_stride = k.stride(0), k.stride(1), k.stride(2)
    p.v_batch_stride, p.v_head_stride, p.v_row_stride = v.stride(0), v.stride(1), v.stride(2)
    p.o_batch_stride, p.o_head_stride, p.o_row_stride = out.stride(0), out.stride(1), out.stride(2)
    if lse is not None:
        p.lse_batch_stride, p.lse_head_stride = lse.stride(0), lse.stride(1)
    p.status = status_word(q.device).data_ptr()
    lib = _lib.load()
    need = int(lib.kvb_decode_workspace_bytes(p, int(num_splits)))
    if need < 0:
        _lib.check(_lib.KVB_ERR_INVALID, "kvb_decode_workspace_bytes: " + (
            lib.kvb_last_error().decode("utf-8", "replace")))
    # The partials' workspace comes from torch's caching allocator for this call:
    # its reuse is ordered on the current stream, so calls on concurrent streams
    # never share one.
    ws = torch.empty(need, dtype=torch.uint8, device=q.device)
    stream = _stream_handle(q.device)
    with torch.cuda.device(q.device):
        rc = lib.kvb_decode_fwd(p, int(num_splits), ws.data_ptr(), ws.numel(), stream)
    _lib.check(rc, "kvb_decode_fwd")
    return out, lse
