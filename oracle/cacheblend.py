"""Oracle: CacheBlend deviation-guided patching of stitched chunk K/V.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

Restates ``CacheBlendRecompute._deviation_recompute`` (``src/kvboost/cacheblend.py:103-197``)
after its full-context forward pass, which the caller supplies as ``fresh`` K/V:

* per layer and cached position, the K vectors of all KV heads flattened into one
  vector (``cacheblend.py:146-150``), cosine similarity between the cached and the
  fresh vector, ``x.y / (max(|x|, 1e-8) max(|y|, 1e-8))`` (torch's
  ``cosine_similarity``, ``:153``), deviation ``1 - cos`` (``:154``);
* the mean over layers (``:158-159``);
* ``k = max(1, int(S * ratio))`` (``:163``); positions with deviation above
  ``min_deviation`` are candidates (``:166``); none -> nothing patched (``:167-169``);
  the ``min(k, #candidates)`` largest deviations are chosen and sorted by position
  (``:172-174``);
* fresh K and V copied over the cached ones at the chosen positions, every layer
  (``:183-197``).

Arithmetic here is float64; the reference computes in the K/V dtype.  Among equal
deviations torch's ``topk`` order is unspecified; this restatement takes the lower
position first.
"""

from __future__ import annotations

from typing import List

import numpy as np


def deviation(cached_k: np.ndarray, fresh_k: np.ndarray, eps: float = 1e-8) -> np.ndarray:
    """cached_k / fresh_k: ``[L, H, S, D]`` -> mean over layers of ``1 - cos``, ``[S]``."""
    ck = np.asarray(cached_k, dtype=np.float64)
    fk = np.asarray(fresh_k, dtype=np.float64)
    L, H, S, D = ck.shape
    a = ck.transpose(0, 2, 1, 3).reshape(L, S, H * D)
    b = fk.transpose(0, 2, 1, 3).reshape(L, S, H * D)
    dot = (a * b).sum(-1)
    na = np.maximum(np.sqrt((a * a).sum(-1)), eps)
    nb = np.maximum(np.sqrt((b * b).sum(-1)), eps)
    return (1.0 - dot / (na * nb)).mean(axis=0)


def num_select(num_tokens: int, ratio: float) -> int:
    """``max(1, int(num_tokens * recompute_ratio))`` (``cacheblend.py:163``)."""
    return max(1, int(num_tokens * ratio))


def select(dev: np.ndarray, k: int, min_deviation: float) -> List[int]:
    """Positions to patch, ascending: the ``min(k, #above)`` largest deviations above
    ``min_deviation`` (lower position first among equal values)."""
    dev = np.asarray(dev)
    above = np.nonzero(dev > min_deviation)[0]
    if above.size == 0:
        return []
    n = min(k, above.size)
    order = sorted(above.tolist(), key=lambda i: (-dev[i], i))
    return sorted(order[:n])


def patch(cached_k, cached_v, fresh_k, fresh_v, positions):
    """Copies of cached K/V (``[L, H, S, D]``) with the fresh rows at ``positions``."""
    pk, pv = np.array(cached_k, copy=True), np.array(cached_v, copy=True)
    if len(positions):
        idx = np.asarray(positions)
        pk[:, :, idx] = np.asarray(fresh_k)[:, :, idx]
        pv[:, :, idx] = np.asarray(fresh_v)[:, :, idx]
    return pk, pv
