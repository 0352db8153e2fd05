"""Host logic of the device pool (CPU): block tables replayed against the
reference's own scripted history (``tests/golden/paged_tables.json``), and the
device append (``append_kv_to_blocks`` semantics) into a 16-bit pool."""

import json
import os

import torch

from kvboost_b200.paged import DeviceBlockAllocator, DeviceChunkMapper


def _kv(n, seed):
    g = torch.Generator().manual_seed(seed)
    return [(torch.randn(1, 2, n, 8, generator=g), torch.randn(1, 2, n, 8, generator=g))]


def test_device_allocator_and_mapper_tables_bit_exact(golden_dir):
    with open(os.path.join(golden_dir, "paged_tables.json")) as f:
        t = json.load(f)
    a = DeviceBlockAllocator(1, 2, 8, 40, device="cpu", dtype=torch.float16)
    m = DeviceChunkMapper(a)
    assert m.load_chunk("c1", _kv(128, 1)) == t["load_c1"]
    assert m.load_chunk("c2", _kv(100, 2)) == t["load_c2"]
    assert m.load_chunk("c1", _kv(128, 1)) == t["reload_c1"]
    assert m.build_block_table([("c1", _kv(128, 1)), ("c2", _kv(100, 2)),
                                ("c3", _kv(40, 3))]) == t["build_c1_c2_c3"]
    m.on_evict("c2")
    assert a.allocate(3) == t["after_evict_alloc3"]
    shared = a.fork(t["load_c1"][:2])
    assert a.ensure_writable(shared[0]) == t["cow_first"]
    k, v = torch.randn(2, 20, 8), torch.randn(2, 20, 8)
    table, off = a.append_kv(0, list(t["load_c1"]), 128, k, v)
    assert table == t["append_20_after_128"] and off == t["append_new_offset"]
    assert a.free_blocks == t["free_blocks_end"]
    assert a._free == t["free_list_end"]
    # the appended tokens sit at their blocks and slots
    kk, vv = a.read_kv(0, table, 148)
    assert torch.equal(kk[:, 128:148], k.to(torch.float16))
    assert torch.equal(vv[:, 128:148], v.to(torch.float16))


def test_append_kv_rejects_int8_pool():
    a = DeviceBlockAllocator(1, 2, 8, 4, device="cpu")
    try:
        a.append_kv(0, [], 0, torch.zeros(2, 1, 8), torch.zeros(2, 1, 8))
    except RuntimeError:
        return
    raise AssertionError("int8 pools take whole chunks only")
