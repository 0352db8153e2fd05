"""Host logic of the engine (CPU): chunk split, keys, reuse planning, store.

``tests/golden/assembly.json`` holds what the reference's own
``KVCacheManager`` + ``PromptAssembler`` (``cache_manager.py:358-393``,
``prompt_assembler.py:99-176``) and ``find_common_chunk_prefix``
(``batch.py:31-54``) decided for a set of prompts; the engine's planner must
make the same decisions.
"""

import json
import os

import pytest
import torch

from kvboost_b200.engine import (DeviceChunk, DeviceChunkStore, chained_hash,
                                 content_hash_from_tokens, find_common_chunk_prefix, fixed_split,
                                 group_by_prefix, plan_reuse)
from oracle import hashing as ohash


@pytest.fixture(scope="module")
def assembly(golden_dir):
    with open(os.path.join(golden_dir, "assembly.json")) as f:
        return json.load(f)


def _store_doc(store, ids, nbytes_per_token=8):
    parent = None
    for s, e, sl in fixed_split(ids):
        h = chained_hash(sl, parent)
        z = torch.zeros(1, 1, e - s, nbytes_per_token // 4)
        store.store(DeviceChunk(h, sl, s, e, z, z.clone()))
        parent = h


def test_hashes_match_oracle():
    ids = list(range(1000, 1300))
    assert chained_hash(ids[:128]) == ohash.chained_hash(ids[:128])
    assert chained_hash(ids[128:256], "abc") == ohash.chained_hash(ids[128:256], "abc")
    assert content_hash_from_tokens(ids) == ohash.content_hash(ids)
    assert fixed_split(ids) == ohash.fixed_split(ids)


@pytest.mark.parametrize("name", ["full_prefix_plus_tail", "partial_prefix", "diverges_in_chunk_3",
                                  "no_match", "other_doc_tail", "short"])
def test_reuse_plan_matches_reference_assembler(assembly, name):
    store = DeviceChunkStore(1 << 30)
    _store_doc(store, assembly["stored"]["base"])
    _store_doc(store, assembly["stored"]["other"])
    case = assembly[name]
    chunks, cached, boundaries = plan_reuse(case["ids"], store)
    assert cached == case["cached_length"]
    assert [list(b) for b in boundaries] == case["boundaries"]
    assert len(case["ids"]) - cached == case["live"]


def test_common_chunk_prefix_matches_reference(assembly):
    for g in assembly["common_prefix"]:
        assert find_common_chunk_prefix(g["ids"], 128) == g["common"]


def test_common_chunk_prefix_chunkwise():
    """The same answer as comparing whole chunks from the start (``batch.py:31-54``)
    on random prompt sets that diverge at random places."""
    import random
    rnd = random.Random(3)

    def chunkwise(all_ids, c):
        if len(all_ids) < 2:
            return len(all_ids[0]) if all_ids else 0
        n, common = min(len(x) for x in all_ids), 0
        for i in range(0, n - c + 1, c):
            if any(x[i:i + c] != all_ids[0][i:i + c] for x in all_ids[1:]):
                break
            common = i + c
        return common

    for _ in range(300):
        base = [rnd.randrange(50) for _ in range(rnd.randrange(0, 700))]
        group = []
        for _ in range(rnd.randrange(1, 5)):
            cut = rnd.randrange(0, len(base) + 1)
            group.append(base[:cut] + [rnd.randrange(50) for _ in range(rnd.randrange(0, 300))])
        for c in (16, 128):
            assert find_common_chunk_prefix(group, c) == chunkwise(group, c)
    assert find_common_chunk_prefix([], 128) == 0


def test_group_by_prefix_matches_reference(assembly):
    case = assembly["group_by_prefix"]
    assert list(group_by_prefix(case["ids"], 128).values()) == case["groups"]


def test_store_lru_eviction_by_bytes():
    store = DeviceChunkStore(3 * 128 * 8 * 2)   # room for three 128-token toy chunks
    docs = [[i] * 128 for i in range(4)]
    for d in docs:
        _store_doc(store, d)
    assert len(store) == 3 and store.evictions == 1
    assert store.get(chained_hash(docs[0])) is None          # oldest went first
    store.get(chained_hash(docs[1]))                         # touch -> most recent
    _store_doc(store, [9] * 128)
    assert store.get(chained_hash(docs[1])) is not None
    assert store.get(chained_hash(docs[2])) is None


def test_oversized_chunk_rejected():
    store = DeviceChunkStore(16)
    z = torch.zeros(1, 1, 128, 2)
    assert store.store(DeviceChunk("x", [0] * 128, 0, 128, z, z)) is False
    assert len(store) == 0


def test_pool_chunks_evicted_release_their_blocks():
    """Chunks held in the int8 block pool count their pool bytes and hand their
    blocks back (through ``on_evict``) when LRU eviction or ``clear`` drops them."""
    freed = []
    store = DeviceChunkStore(3 * 1000, on_evict=lambda c: freed.extend(c.block_ids))
    for i in range(4):
        ids = [i] * 128
        ok = store.make_room(1000)
        assert ok
        assert store.store(DeviceChunk(chained_hash(ids), ids, 0, 128, None, None,
                                       block_ids=[8 * i + j for j in range(8)], pool_bytes=1000))
    assert store.bytes == 3000 and freed == list(range(8))
    assert store.make_room(4000) is False
    store.clear()
    assert sorted(freed) == list(range(32)) and store.bytes == 0
