"""The C-ABI library loads and exports every symbol ``include/*.h`` declares.

CPU only: nothing here launches a kernel.  Argument validation happens on
the host before any CUDA call, so invalid calls can be checked without a GPU.
"""

import ctypes
import os
import subprocess

import pytest

from kvboost_b200 import _build, _lib


@pytest.fixture(scope="module")
def lib():
    if not os.path.exists(_build.LIB_PATH):
        _build.build(verbose=False)
    return _lib.load()


def test_header_declares_expected_entry_points():
    names = _lib.header_symbols()
    for n in ("kvb_flash_attn_fwd", "kvb_prefill_fwd", "kvb_last_error", "kvb_abi_version"):
        assert n in names


def test_every_declared_symbol_is_exported(lib):
    out = subprocess.run(["nm", "-D", "--defined-only", _build.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if line.strip()}
    for name in _lib.header_symbols():
        assert name in exported, f"{name} declared in include/ but not exported"
        assert hasattr(lib, name)


def test_abi_version(lib):
    assert lib.kvb_abi_version() == 2


def test_ctypes_struct_matches_header_size():
    # 11 x int32/float = 44 -> padded to 48, 5 pointers, 14 int64, 3 pointers
    assert ctypes.sizeof(_lib.KvbPrefillParams) == 48 + 5 * 8 + 14 * 8 + 3 * 8


def _params(**kw):
    p = _lib.KvbPrefillParams()
    p.dtype, p.head_dim, p.batch, p.num_q_heads, p.num_kv_heads = 0, 128, 1, 4, 2
    p.q_len, p.kv_len, p.causal, p.softmax_scale = 16, 32, 1, 0.088
    p.q = p.k = p.v = p.o = 4096
    for s in ("q", "k", "v", "o"):
        setattr(p, f"{s}_row_stride", 128)
        setattr(p, f"{s}_head_stride", 128 * 64)
        setattr(p, f"{s}_batch_stride", 128 * 64 * 8)
    for k_, v_ in kw.items():
        setattr(p, k_, v_)
    return p


@pytest.mark.parametrize("field,value,needle", [
    ("head_dim", 80, "head_dim"),
    ("dtype", 7, "dtype"),
    ("num_kv_heads", 3, "divisible"),
    ("causal", 5, "causal"),
    ("q_len", -1, "non-negative"),
    ("q", 0, "non-null"),
    ("k", 4097, "aligned"),
    ("q_row_stride", 100, "multiples of 8"),
])
def test_host_validation_rejects_before_launch(lib, field, value, needle):
    p = _params(**{field: value})
    rc = lib.kvb_prefill_fwd(ctypes.byref(p), None)
    assert rc == _lib.KVB_ERR_INVALID
    assert needle in lib.kvb_last_error().decode()


def test_query_tile_count_limit(lib):
    # query tiles are the grid's y dimension: at most 65535 tiles of 128 rows
    p = _params(q_len=65535 * 128 + 1, kv_len=65535 * 128 + 1)
    assert lib.kvb_prefill_fwd(ctypes.byref(p), None) == _lib.KVB_ERR_UNSUPPORTED
    assert "q_len must be <=" in lib.kvb_last_error().decode()


def test_null_params_rejected(lib):
    assert lib.kvb_prefill_fwd(None, None) == _lib.KVB_ERR_INVALID


def test_compat_entry_validates_head_dim(lib):
    rc = lib.kvb_flash_attn_fwd(4096, 4096, 4096, 4096, None, 1, 2, 8, 48, 0, 0.1, 1, None)
    assert rc == _lib.KVB_ERR_INVALID
    assert b"head_dim" in lib.kvb_last_error()


def test_ctypes_layouts_match_c_compiler(tmp_path):
    """sizeof/offsetof of both parameter structs as gcc sees the header."""
    from kvboost_b200._build import INCLUDE
    structs = {"KvbPrefillParams": _lib.KvbPrefillParams,
               "KvbPagedPrefillParams": _lib.KvbPagedPrefillParams,
               "KvbPeerShards": _lib.KvbPeerShards,
               "KvbPeerSignals": _lib.KvbPeerSignals,
               "KvbQuantizeStoreParams": _lib.KvbQuantizeStoreParams,
               "KvbQuantizeStoreBatch": _lib.KvbQuantizeStoreBatch,
               "KvbCacheBlendParams": _lib.KvbCacheBlendParams}
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "kvb_attn.h"', 'int main(){']
    for name, cls in structs.items():
        lines.append(f'printf("{name} %zu\\n", sizeof({name}));')
        for f, _ in cls._fields_:
            lines.append(f'printf("{name}.{f} %zu\\n", offsetof({name}, {f}));')
    lines.append('return 0;}')
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-I", INCLUDE, "-o", str(exe), str(src)], check=True)
    got = dict(l.split() for l in subprocess.run([str(exe)], capture_output=True, text=True,
                                                  check=True).stdout.splitlines())
    for name, cls in structs.items():
        assert int(got[name]) == ctypes.sizeof(cls)
        for f, _ in cls._fields_:
            assert int(got[f"{name}.{f}"]) == getattr(cls, f).offset, f"{name}.{f}"


def test_paged_strategy_selection():
    """The workspace strategy is chosen only when many CTAs read each KV tile."""
    from kvboost_b200 import _lib
    lib = _lib.load()
    p = _lib.KvbPagedPrefillParams()
    p.dtype, p.head_dim, p.batch, p.num_q_heads, p.num_kv_heads = 0, 128, 1, 64, 8
    p.q_len, p.causal, p.softmax_scale = 2048, 1, 0.088
    p.q = p.o = p.k_new = p.v_new = p.kv_pool = p.k_scale = p.v_scale = p.block_tables = 4096
    for f in ("q", "o", "k_new", "v_new"):
        setattr(p, f"{f}_head_stride", 128 * 2048)
        setattr(p, f"{f}_row_stride", 128)
    p.num_blocks, p.block_size, p.max_blocks_per_seq, p.prefix_len = 8192, 16, 2048, 32768
    assert lib.kvb_paged_prefill_workspace_bytes(p) == 2 * 8 * (32768 + 2048) * 128 * 2
    p.q_len = 16  # a seam-recompute-sized suffix stays fused (reads int8 once)
    p.num_q_heads = 16
    assert lib.kvb_paged_prefill_workspace_bytes(p) == 0


def test_peer_shard_layout(lib):
    """Region offsets of a context-parallel shard buffer (host-side arithmetic)."""
    off = (ctypes.c_int64 * 5)()
    total = lib.kvb_peer_shard_layout(8, 128, 1024, 512, off)
    pool = 1024 * 2 * 8 * 16 * 128
    ks, vs, sfx = 1024 * 8 * 16 * 4, 1024 * 8 * 128 * 4, 8 * 1024 * 128 * 2
    assert list(off) == [0, pool, pool + ks, pool + ks + vs, pool + ks + vs + sfx]
    assert total == pool + ks + vs + 2 * sfx
    assert all(o % 16 == 0 for o in off)
    assert lib.kvb_peer_shard_layout(8, 80, 1024, 512, off) == -1


def _qstore(**kw):
    import ctypes as C
    p = _lib.KvbQuantizeStoreParams()
    p.dtype, p.head_dim, p.num_layers, p.num_kv_heads = 0, 128, 2, 2
    p.num_tokens, p.num_chunk_blocks, p.num_pool_blocks = 128, 8, 64
    for i in range(8):
        p.block_ids[i] = 63 - i
    ptrs = _lib.pointer_array([4096, 8192])
    for f in ("src_k", "src_v", "pool", "k_scale16", "v_scale16", "k_scale", "v_scale"):
        setattr(p, f, C.cast(ptrs, _lib._pp))
    p.src_head_stride, p.src_row_stride = 128 * 128, 128
    for k_, v_ in kw.items():
        setattr(p, k_, v_)
    return p, ptrs


@pytest.mark.parametrize("field,value,needle", [
    ("head_dim", 80, "head_dim"),
    ("dtype", 3, "dtype"),
    ("num_layers", 0, "num_layers"),
    ("num_layers", 129, "num_layers"),
    ("num_tokens", 0, "num_tokens"),
    ("num_chunk_blocks", 7, "ceil(num_tokens / 16)"),
    ("num_pool_blocks", 60, "outside the pool"),
    ("src_row_stride", 0, "src_row_stride"),
])
def test_quantize_store_validation(lib, field, value, needle):
    p, keep = _qstore(**{field: value})
    assert lib.kvb_quantize_store(ctypes.byref(p), None) == _lib.KVB_ERR_INVALID
    assert needle in lib.kvb_last_error().decode()


def test_quantize_store_rejects_repeated_blocks(lib):
    p, keep = _qstore()
    p.block_ids[3] = p.block_ids[0]
    assert lib.kvb_quantize_store(ctypes.byref(p), None) == _lib.KVB_ERR_INVALID
    assert b"repeat" in lib.kvb_last_error()


def _blend(**kw):
    import ctypes as C
    p = _lib.KvbCacheBlendParams()
    p.dtype, p.head_dim, p.num_layers, p.num_kv_heads = 0, 128, 2, 2
    p.num_tokens, p.num_select, p.min_deviation, p.patch = 256, 38, 0.01, 1
    ptrs = _lib.pointer_array([4096, 8192])
    for f in ("cached_k", "cached_v", "fresh_k", "fresh_v"):
        setattr(p, f, C.cast(ptrs, _lib._pp))
    p.cached_head_stride, p.cached_row_stride = 256 * 128, 128
    p.fresh_head_stride, p.fresh_row_stride = 256 * 128, 128
    p.deviation = p.selected = p.num_selected = 4096
    for k_, v_ in kw.items():
        setattr(p, k_, v_)
    return p, ptrs


@pytest.mark.parametrize("field,value,needle", [
    ("head_dim", 48, "head_dim"),
    ("num_select", 0, "num_select"),
    ("patch", 2, "patch"),
    ("cached_row_stride", 100, "multiples of 8"),
    ("fresh_row_stride", 0, "non-zero"),
    ("cached_v", None, "cached_v"),
    ("deviation", None, "deviation"),
])
def test_cacheblend_validation(lib, field, value, needle):
    p, keep = _blend(**{field: value})
    assert lib.kvb_cacheblend_fwd(ctypes.byref(p), None) == _lib.KVB_ERR_INVALID
    assert needle in lib.kvb_last_error().decode()


def test_cacheblend_rejects_unaligned_pointers(lib):
    import ctypes as C
    bad = _lib.pointer_array([4096 + 2, 8192])
    p, keep = _blend()
    p.fresh_k = C.cast(bad, _lib._pp)
    assert lib.kvb_cacheblend_fwd(ctypes.byref(p), None) == _lib.KVB_ERR_INVALID
    assert b"16-byte aligned" in lib.kvb_last_error()


@pytest.mark.parametrize("field,value,needle", [
    ("num_chunks", 0, "num_chunks"),
    ("num_chunks", 2000, "num_chunks"),
    ("max_chunk_blocks", 129, "max_chunk_blocks"),
    ("num_pool_blocks", 0, "num_pool_blocks"),
    ("src", None, "non-null"),
    ("head_dim", 72, "head_dim"),
])
def test_quantize_store_batch_validation(lib, field, value, needle):
    p = _lib.KvbQuantizeStoreBatch()
    p.dtype, p.head_dim, p.num_layers, p.num_kv_heads = 0, 128, 36, 2
    p.num_chunks, p.max_chunk_blocks, p.num_pool_blocks = 24, 8, 1024
    p.num_tokens = p.block_ids = p.src = p.src_strides = p.tables = 4096
    setattr(p, field, value)
    assert lib.kvb_quantize_store_batch(ctypes.byref(p), None) == _lib.KVB_ERR_INVALID
    assert needle in lib.kvb_last_error().decode()


@pytest.mark.parametrize("field,value,needle", [
    ("world", 0, "world must be in"), ("world", 9, "world must be in"),
    ("rank", 2, "rank must be in"), ("slot", None, "non-null and 4-byte"),
])
def test_peer_barrier_validation(lib, field, value, needle):
    """Argument errors come back before anything launches (no device needed)."""
    sig = _lib.KvbPeerSignals()
    sig.world, sig.rank = 2, 0
    sig.slot[0], sig.slot[1] = 4096, 8192
    if field == "slot":
        sig.slot[1] = value
    else:
        setattr(sig, field, value)
    rc = lib.kvb_peer_barrier(ctypes.byref(sig), 1, 1_000_000, None, None)
    assert rc == _lib.KVB_ERR_INVALID or rc == _lib.KVB_ERR_UNSUPPORTED
    assert needle in lib.kvb_last_error().decode()


def test_peer_barrier_rejects_epoch_zero_and_bad_timeouts(lib):
    sig = _lib.KvbPeerSignals()
    sig.world, sig.rank, sig.slot[0] = 1, 0, 4096
    assert lib.kvb_peer_barrier(ctypes.byref(sig), 0, 1_000_000, None, None) == _lib.KVB_ERR_INVALID
    assert lib.kvb_peer_barrier(ctypes.byref(sig), 1, 0, None, None) == _lib.KVB_ERR_INVALID
    assert lib.kvb_peer_barrier(ctypes.byref(sig), 1, 61 * 10**9, None, None) == \
        _lib.KVB_ERR_INVALID
