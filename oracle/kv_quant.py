"""Oracle: KIVI int8 KV quantisation with the reference's float16 rounding.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

Restates ``_quantize_int8`` / ``_dequantize_int8``
(``src/kvboost/kv_quantize.py:73-109``) for one layer of one chunk:

* K: ``amax`` over head_dim (one scale per token, shape ``[..., S, 1]``,
  ``kv_quantize.py:84-86``), V: ``amax`` over the sequence axis (one scale per
  channel per chunk, shape ``[..., 1, D]``, ``kv_quantize.py:89-91``).
* ``scale = amax.clamp(min=1e-8) / 127`` and ``q = round(x / scale)`` clamped to
  ``[-128, 127]``.  Torch evaluates float16 arithmetic on the CPU in float32
  and rounds each result to float16; numpy float32 ops followed by a cast to
  float16 (round-to-nearest-even) reproduce that bit for bit, and ``np.round``
  is round-half-to-even like ``torch.round``.
* Dequant is ``q.to(float16) * scale_f16`` (``kv_quantize.py:102-109``): the
  exact product rounded once to float16.  Models running in bfloat16 then
  see ``bfloat16(float16(q * s))``.
"""

from __future__ import annotations

import numpy as np


def _f16(x):
    return np.asarray(x, dtype=np.float32).astype(np.float16)


def quantize_int8(key_f16: np.ndarray, val_f16: np.ndarray):
    """key/val: float16 ``[..., S, D]``.  Returns (key_q, key_scale, val_q, val_scale)."""
    with np.errstate(invalid="ignore", divide="ignore"):
        return _quantize_int8(np.asarray(key_f16, dtype=np.float16),
                              np.asarray(val_f16, dtype=np.float16))


def _quantize_int8(key, val):

    key_amax = np.abs(key).max(axis=-1, keepdims=True)
    key_amax = _f16(np.maximum(key_amax.astype(np.float32), np.float32(1e-8)))
    key_scale = _f16(key_amax.astype(np.float32) / np.float32(127.0))
    kq = _f16(key.astype(np.float32) / key_scale.astype(np.float32))
    key_q = np.clip(np.round(kq.astype(np.float32)), -128, 127).astype(np.int8)

    val_amax = np.abs(val).max(axis=-2, keepdims=True)
    val_amax = _f16(np.maximum(val_amax.astype(np.float32), np.float32(1e-8)))
    val_scale = _f16(val_amax.astype(np.float32) / np.float32(127.0))
    vq = _f16(val.astype(np.float32) / val_scale.astype(np.float32))
    val_q = np.clip(np.round(vq.astype(np.float32)), -128, 127).astype(np.int8)
    return key_q, key_scale, val_q, val_scale


def _round_to(x: np.ndarray, dtype: str) -> np.ndarray:
    """float32 values rounded once to ``dtype`` ("f16" or "bf16"), returned as float32."""
    x = np.asarray(x, dtype=np.float32)
    if dtype == "f16":
        return x.astype(np.float16).astype(np.float32)
    return round_to_bf16(x)


def quantize_int8_model_dtype(key: np.ndarray, val: np.ndarray, dtype: str):
    """``_quantize_int8`` (``kv_quantize.py:73-100``) on K/V held in the model's dtype.

    key/val: float32 arrays holding exact ``dtype`` values (``"bf16"`` or ``"f16"``),
    ``[..., S, D]``.  Torch runs each elementwise step in float32 and rounds the
    result to ``dtype``: ``amax`` (exact), ``clamp(min=1e-8)`` (1e-8 rounds to 0 in
    float16, to 1.0012e-8 in bfloat16), ``/ 127`` (the float32 quotient, rounded;
    for every finite 16-bit value this equals rounding ``amax * (1/127)``),
    ``key / key_scale`` (rounded), ``round`` half-to-even, clamp to [-128, 127].
    ``0 / 0`` (an all-zero row in float16) gives NaN, which the int8 cast turns into
    0 on the reference's CPU.  The scales are returned cast to float16 as the
    reference stores them (``kv_quantize.py:93-97``).
    Returns ``(key_q, key_scale_f16, val_q, val_scale_f16)``.
    """
    key = np.asarray(key, dtype=np.float32)
    val = np.asarray(val, dtype=np.float32)

    def one(x, axis):
        amax = np.abs(x).max(axis=axis, keepdims=True)
        amax = _round_to(np.maximum(amax, np.float32(1e-8)), dtype)
        scale = _round_to(amax / np.float32(127.0), dtype)
        with np.errstate(invalid="ignore", divide="ignore"):
            r = _round_to(x / scale, dtype)
        q = np.clip(np.round(r), -128, 127)
        q = np.where(np.isnan(q), 0, q).astype(np.int8)
        return q, scale.astype(np.float16)

    key_q, key_scale = one(key, -1)
    val_q, val_scale = one(val, -2)
    return key_q, key_scale, val_q, val_scale


def dequantize_int8(q: np.ndarray, scale_f16: np.ndarray) -> np.ndarray:
    """``float16(q * scale)``; ``scale`` broadcasts like the reference's."""
    return _f16(q.astype(np.float32) * np.asarray(scale_f16, dtype=np.float16).astype(np.float32))


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round float32 to bfloat16 (nearest-even) and return the uint16 bit pattern."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    rounded = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    nan = np.isnan(x)
    out = rounded.astype(np.uint16)
    out[nan] = 0x7FC0
    return out


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def round_to_bf16(x: np.ndarray) -> np.ndarray:
    """Values of ``x`` rounded to the nearest bfloat16, returned as float32."""
    return bf16_bits_to_f32(f32_to_bf16_bits(x))
