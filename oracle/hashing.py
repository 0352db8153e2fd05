"""Oracle: chunk keys and the fixed chunk split.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

* ``content_hash``  restates ``content_hash_from_tokens`` (``src/kvboost/models.py:131-134``):
  SHA-256 over each token id as 4 little-endian bytes, hex digest.
* ``chained_hash``  restates ``chained_hash`` (``src/kvboost/models.py:137-148``):
  SHA-256 over ``(parent or "root")`` as UTF-8 followed by the token bytes.
* ``fixed_split``   restates ``ChunkRegistry._fixed_split``
  (``src/kvboost/chunk_registry.py:98-110``): windows ``[pos, min(pos+cs, n))``,
  dropping windows shorter than ``min_chunk_tokens`` (default 32,
  ``chunk_registry.py:43``).
"""

from __future__ import annotations

import hashlib
import struct
from typing import List, Optional, Tuple


def _token_bytes(token_ids) -> bytes:
    return struct.pack("<%dI" % len(token_ids), *[int(t) & 0xFFFFFFFF for t in token_ids])


def content_hash(token_ids) -> str:
    return hashlib.sha256(_token_bytes(token_ids)).hexdigest()


def chained_hash(token_ids, parent_hash: Optional[str] = None) -> str:
    parent = (parent_hash or "root").encode("utf-8")
    return hashlib.sha256(parent + _token_bytes(token_ids)).hexdigest()


def fixed_split(token_ids, chunk_size: int = 128, min_chunk_tokens: int = 32) -> List[Tuple[int, int, list]]:
    out = []
    n = len(token_ids)
    pos = 0
    while pos < n:
        end = min(pos + chunk_size, n)
        if end - pos >= min_chunk_tokens:
            out.append((pos, end, list(token_ids[pos:end])))
        pos = end
    return out


def prefix_chain(token_ids, chunk_size: int = 128, min_chunk_tokens: int = 32) -> List[str]:
    """Prefix hashes of consecutive chunks, each chained on the previous one."""
    parent = None
    keys = []
    for _, _, ids in fixed_split(token_ids, chunk_size, min_chunk_tokens):
        parent = chained_hash(ids, parent)
        keys.append(parent)
    return keys
