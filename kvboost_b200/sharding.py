"""Placing independent requests on the GPUs of a box (one process per GPU).

A varlen batch of reuse prefills is a set of independent requests, each with its
own suffix and reused prefix; spreading them over the ranks needs no collective.
``lpt_partition`` assigns them longest-processing-time first: requests in order of
decreasing cost, each to the rank with the least work so far (ties to the lower
rank), which keeps the slowest rank within 4/3 of the optimum.  Every rank computes
the same partition from the same lengths, so no rank sends anything.
"""

from __future__ import annotations

import heapq
from typing import List, Sequence


def request_cost(q_len: int, kv_len: int, num_q_heads: int, num_kv_heads: int, head_dim: int,
                 peak_flops: float = 1.651e15, peak_bytes: float = 6.54e12,
                 elem_bytes: int = 2) -> float:
    """Roofline time of one bottom-right causal request: the larger of its FLOPs over
    the tensor peak and its bytes (Q, O, K, V once) over the HBM bandwidth."""
    pairs = q_len * (kv_len - q_len) + q_len * (q_len + 1) // 2
    flops = 4.0 * head_dim * num_q_heads * pairs
    nbytes = elem_bytes * head_dim * (2 * num_q_heads * q_len + 2 * num_kv_heads * kv_len)
    return max(flops / peak_flops, nbytes / peak_bytes)


def lpt_partition(costs: Sequence[float], world: int) -> List[List[int]]:
    """Request indices per rank, each list in increasing index order."""
    if world < 1:
        raise ValueError("world must be >= 1")
    order = sorted(range(len(costs)), key=lambda i: (-costs[i], i))
    heap = [(0.0, r) for r in range(world)]
    parts: List[List[int]] = [[] for _ in range(world)]
    for i in order:
        load, r = heapq.heappop(heap)
        parts[r].append(i)
        heapq.heappush(heap, (load + costs[i], r))
    return [sorted(p) for p in parts]
