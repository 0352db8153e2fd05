"""CacheBlend repair of stitched chunk K/V, on the device.

``CacheBlendRecompute`` keeps the reference's knobs and steps
(``src/kvboost/cacheblend.py:56-197``): one full-context forward over the cached
tokens (on the sm_100a prefill kernel, q = kv causal, through the attention hook),
then per cached position the mean over layers of the cosine deviation between
the cached and the full-context K (all KV heads flattened into one vector), the
``max(1, int(S * recompute_ratio))`` most deviated positions above
``min_deviation``, and the full-context K/V copied over the cached K/V there.
The deviation, the selection and the patch are one call into
``kvb_cacheblend_fwd`` (three kernels, no host round trip: the chosen count stays
on the device).

Differences from the reference, both deliberate: the deviation is computed in
float32 (the reference computes it in the K/V dtype, so bfloat16 rounding can
reorder near-equal deviations), and among equal deviations the lower position
is taken first (torch's ``topk`` leaves that order unspecified).
"""

from __future__ import annotations

import ctypes
from typing import List, Optional, Sequence, Tuple, Union

import torch

from . import _lib
from .ops import _DTYPES, _stream_handle
from .paged import _layer_list

LayerKV = Union[torch.Tensor, Sequence[torch.Tensor]]


def num_select(num_tokens: int, recompute_ratio: float) -> int:
    """``max(1, int(num_tokens * recompute_ratio))`` (``cacheblend.py:163``)."""
    return max(1, int(num_tokens * recompute_ratio))


def _strides(layers: List[torch.Tensor], name: str) -> Tuple[int, int]:
    ref = layers[0]
    for t in layers:
        if t.stride() != ref.stride() or t.stride(2) != 1:
            raise ValueError(f"{name}: every layer needs the same strides and a contiguous last dim")
    return ref.stride(0), ref.stride(1)


def cacheblend_fwd(cached_k: LayerKV, cached_v: Optional[LayerKV], fresh_k: LayerKV,
                   fresh_v: Optional[LayerKV], recompute_ratio: float = 0.15,
                   min_deviation: float = 0.01, patch: bool = True):
    """Deviation, selection and (``patch=True``) the in-place patch of ``cached_k`` /
    ``cached_v`` with ``fresh_k`` / ``fresh_v`` at the chosen positions.

    Each K/V argument is a stacked ``[L, H, S_c, D]`` tensor or a per-layer sequence
    of ``[H, S_c, D]`` / ``[1, H, S_c, D]`` tensors; the fresh ones cover the first
    ``S`` cached positions (``S`` = their length), which are the ones compared.
    Returns device tensors ``(deviation [S] float32, selected [k] int32 ascending,
    -1 after the count, num_selected [1] int32)``.
    """
    ck, fk = _layer_list(cached_k), _layer_list(fresh_k)
    L = len(fk)
    if len(ck) != L or not 1 <= L <= _lib.KVB_MAX_LAYERS:
        raise ValueError(f"cached and fresh K need the same 1..{_lib.KVB_MAX_LAYERS} layers")
    H, S, D = fk[0].shape
    dt, dev = fk[0].dtype, fk[0].device
    if dt not in _DTYPES:
        raise TypeError("K/V must be bfloat16 or float16")
    if patch:
        if cached_v is None or fresh_v is None:
            raise ValueError("patching needs cached_v and fresh_v")
        cv, fv = _layer_list(cached_v), _layer_list(fresh_v)
    else:
        cv = fv = []
    for t in ck + cv:
        if t.shape[0] != H or t.shape[2] != D or t.shape[1] < S or t.dtype != dt or t.device != dev:
            raise ValueError("cached K/V must match the fresh heads, head_dim, dtype, device "
                             "and cover at least its positions")
    for t in fk + fv:
        if t.shape != fk[0].shape or t.dtype != dt or t.device != dev:
            raise ValueError("fresh K/V layers must share shape, dtype and device")
    c_hs, c_rs = _strides(ck + cv, "cached K/V")     # patched in place: must share a layout
    if any(t.stride() != fk[0].stride() or t.stride(2) != 1 for t in fk + fv):
        fk = [t.contiguous() for t in fk]             # read only: bring to one layout
        fv = [t.contiguous() for t in fv]
    f_hs, f_rs = _strides(fk + fv, "fresh K/V")
    k = num_select(S, recompute_ratio)
    deviation = torch.empty(S, dtype=torch.float32, device=dev)
    selected = torch.empty(k, dtype=torch.int32, device=dev)
    count = torch.empty(1, dtype=torch.int32, device=dev)
    p = _lib.KvbCacheBlendParams()
    p.dtype, p.head_dim, p.num_layers, p.num_kv_heads = _DTYPES[dt], D, L, H
    p.num_tokens, p.num_select = S, k
    p.min_deviation, p.patch = float(min_deviation), 1 if patch else 0
    arrays = [_lib.pointer_array([t.data_ptr() for t in g]) for g in (ck, cv, fk, fv)]
    p.cached_k, p.cached_v, p.fresh_k, p.fresh_v = [
        ctypes.cast(a, _lib._pp) if len(g) else None for a, g in zip(arrays, (ck, cv, fk, fv))]
    p.cached_head_stride, p.cached_row_stride = c_hs, c_rs
    p.fresh_head_stride, p.fresh_row_stride = f_hs, f_rs
    p.deviation, p.selected, p.num_selected = deviation.data_ptr(), selected.data_ptr(), count.data_ptr()
    with torch.cuda.device(dev):
        _lib.check(_lib.load().kvb_cacheblend_fwd(ctypes.byref(p), _stream_handle(dev)),
                   "kvb_cacheblend_fwd")
    return deviation, selected, count


class CacheBlendRecompute:
    """Same constructor knobs as ``CacheBlendRecompute`` (``cacheblend.py:56-64``)."""

    def __init__(self, recompute_ratio: float = 0.15, min_deviation: float = 0.01,
                 device: Optional[str] = None):
        self.recompute_ratio = recompute_ratio
        self.min_deviation = min_deviation
        self.device = device
        self.last_num_selected: Optional[torch.Tensor] = None

    def repair(self, cached_k: LayerKV, cached_v: LayerKV, fresh_k: LayerKV,
               fresh_v: LayerKV) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        """Patch ``cached_k`` / ``cached_v`` in place (``cacheblend.py:141-197``);
        returns ``(deviation, selected, num_selected)``."""
        out = cacheblend_fwd(cached_k, cached_v, fresh_k, fresh_v, self.recompute_ratio,
                             self.min_deviation, patch=True)
        self.last_num_selected = out[2]
        return out
