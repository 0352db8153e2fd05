"""kvboost_b200 -- B200 (sm_100a) prefill attention for KVBoost's reuse path.

The hot path -- a suffix of queries attending to reused 128-token chunk K/V
plus its own fresh K/V under bottom-right causality -- runs in hand-written
tcgen05/TMA kernels behind the C ABI in ``include/kvb_attn.h``.  The Python
side mirrors KVBoost's own plugin surface (``flash_attn_ext``) so it drops in.
"""

__version__ = "0.1.0"

from .ops import prefill_attention, prefill_attention_varlen, read_status  # noqa: F401
