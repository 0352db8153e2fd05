"""ctypes binding of the C ABI in ``include/kvb_attn.h``.

The library is loaded from the package directory (built in-tree by
``kvboost_b200._build``).  There is no fallback: if the library is missing
or fails to load, every op raises.
"""

from __future__ import annotations

import ctypes
import os
import re
import threading

from . import _build

KVB_DTYPE_BF16 = 0
KVB_DTYPE_FP16 = 1
KVB_OK = 0
KVB_ERR_INVALID = 1
KVB_ERR_UNSUPPORTED = 2
KVB_ERR_CUDA = -1
KVB_NOALLOC_SCRATCH_BYTES = 32 << 20
KVB_POOL_INT8_KIVI, KVB_POOL_COMPUTE = 0, 1
KVB_STATUS_BAD_BLOCK, KVB_STATUS_BAD_LENGTH, KVB_STATUS_PEER_WAIT = 16, 32, 64

_i32, _i64, _f32, _vp = ctypes.c_int32, ctypes.c_int64, ctypes.c_float, ctypes.c_void_p


class KvbPrefillParams(ctypes.Structure):
    """Mirror of ``KvbPrefillParams`` (field order and types must match the header)."""

    _fields_ = [
        ("dtype", _i32), ("head_dim", _i32), ("batch", _i32),
        ("num_q_heads", _i32), ("num_kv_heads", _i32),
        ("q_len", _i32), ("kv_len", _i32), ("causal", _i32),
        ("softmax_scale", _f32), ("total_q", _i32), ("total_k", _i32),
        ("q", _vp), ("k", _vp), ("v", _vp), ("o", _vp), ("lse", _vp),
        ("q_batch_stride", _i64), ("q_head_stride", _i64), ("q_row_stride", _i64),
        ("k_batch_stride", _i64), ("k_head_stride", _i64), ("k_row_stride", _i64),
        ("v_batch_stride", _i64), ("v_head_stride", _i64), ("v_row_stride", _i64),
        ("o_batch_stride", _i64), ("o_head_stride", _i64), ("o_row_stride", _i64),
        ("lse_batch_stride", _i64), ("lse_head_stride", _i64),
        ("cu_seqlens_q", _vp), ("cu_seqlens_k", _vp), ("status", _vp),
    ]


class KvbPeerShards(ctypes.Structure):
    """Mirror of ``KvbPeerShards``."""

    _fields_ = [("base", _vp * 8), ("world", _i32), ("shard_blocks", _i32),
                ("zigzag_rows", _i32), ("reserved0", _i32)]


class KvbPeerSignals(ctypes.Structure):
    """Mirror of ``KvbPeerSignals``."""

    _fields_ = [("slot", _vp * 8), ("world", _i32), ("rank", _i32)]


class KvbPagedPrefillParams(ctypes.Structure):
    """Mirror of ``KvbPagedPrefillParams`` (field order and types must match the header)."""

    _fields_ = [
        ("dtype", _i32), ("head_dim", _i32), ("batch", _i32),
        ("num_q_heads", _i32), ("num_kv_heads", _i32), ("q_len", _i32), ("causal", _i32),
        ("softmax_scale", _f32),
        ("q", _vp), ("o", _vp), ("lse", _vp),
        ("q_batch_stride", _i64), ("q_head_stride", _i64), ("q_row_stride", _i64),
        ("o_batch_stride", _i64), ("o_head_stride", _i64), ("o_row_stride", _i64),
        ("lse_batch_stride", _i64), ("lse_head_stride", _i64),
        ("k_new", _vp), ("v_new", _vp),
        ("k_new_batch_stride", _i64), ("k_new_head_stride", _i64), ("k_new_row_stride", _i64),
        ("v_new_batch_stride", _i64), ("v_new_head_stride", _i64), ("v_new_row_stride", _i64),
        ("kv_pool", _vp), ("k_scale", _vp), ("v_scale", _vp),
        ("num_blocks", _i32), ("block_size", _i32),
        ("block_tables", _vp), ("max_blocks_per_seq", _i32), ("prefix_len", _i32),
        ("prefix_lens", _vp), ("status", _vp),
        ("workspace", _vp), ("workspace_bytes", _i64),
        ("pool_format", _i32), ("reserved0", _i32),
    ]


_lock = threading.Lock()
_lib = None


KVB_MAX_LAYERS = 128
KVB_MAX_CHUNK_BLOCKS = 128
_pp = ctypes.POINTER(ctypes.c_void_p)


class KvbQuantizeStoreParams(ctypes.Structure):
    """Mirror of ``KvbQuantizeStoreParams``."""

    _fields_ = [
        ("dtype", _i32), ("head_dim", _i32), ("num_layers", _i32), ("num_kv_heads", _i32),
        ("num_tokens", _i32), ("num_chunk_blocks", _i32),
        ("block_ids", _i32 * KVB_MAX_CHUNK_BLOCKS),
        ("num_pool_blocks", _i64),
        ("src_k", _pp), ("src_v", _pp),
        ("src_head_stride", _i64), ("src_row_stride", _i64),
        ("pool", _pp), ("k_scale16", _pp), ("v_scale16", _pp), ("k_scale", _pp), ("v_scale", _pp),
    ]


class KvbCacheBlendParams(ctypes.Structure):
    """Mirror of ``KvbCacheBlendParams``."""

    _fields_ = [
        ("dtype", _i32), ("head_dim", _i32), ("num_layers", _i32), ("num_kv_heads", _i32),
        ("num_tokens", _i32), ("num_select", _i32), ("min_deviation", ctypes.c_float),
        ("patch", _i32),
        ("cached_k", _pp), ("cached_v", _pp), ("fresh_k", _pp), ("fresh_v", _pp),
        ("cached_head_stride", _i64), ("cached_row_stride", _i64),
        ("fresh_head_stride", _i64), ("fresh_row_stride", _i64),
        ("deviation", _vp), ("selected", _vp), ("num_selected", _vp),
    ]


class KvbQuantizeStoreBatch(ctypes.Structure):
    """Mirror of ``KvbQuantizeStoreBatch``."""

    _fields_ = [
        ("dtype", _i32), ("head_dim", _i32), ("num_layers", _i32), ("num_kv_heads", _i32),
        ("num_chunks", _i32), ("max_chunk_blocks", _i32), ("num_pool_blocks", _i64),
        ("num_tokens", _vp), ("block_ids", _vp), ("src", _vp), ("src_strides", _vp),
        ("tables", _vp), ("status", _vp),
    ]


def pointer_array(ptrs):
    """A ctypes ``void*[n]`` of device addresses (keep it alive across the call)."""
    arr = (ctypes.c_void_p * len(ptrs))(*[int(p) if p else None for p in ptrs])
    return arr


def lib_path() -> str:
    """The in-tree library, or the build named by ``KVB_LIB`` (the traced build that
    ``kvboost_b200._trace`` loads)."""
    return os.environ.get("KVB_LIB") or _build.LIB_PATH


def load() -> ctypes.CDLL:
    """Load (once) and return the CUDA library; raises if it is not built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = lib_path()
        if not os.path.exists(path):
            raise RuntimeError(
                f"kvboost_b200 CUDA library not found at {path}; build it with "
                "`python -m kvboost_b200._build` (nvcc, sm_100a)")
        lib = ctypes.CDLL(path)
        lib.kvb_prefill_fwd.argtypes = [ctypes.POINTER(KvbPrefillParams), _vp]
        lib.kvb_prefill_fwd.restype = ctypes.c_int
        lib.kvb_flash_attn_fwd.argtypes = [_vp, _vp, _vp, _vp, _vp, ctypes.c_int, ctypes.c_int,
                                           ctypes.c_int, ctypes.c_int, ctypes.c_int, _f32,
                                           ctypes.c_int, _vp]
        lib.kvb_flash_attn_fwd.restype = ctypes.c_int
        lib.kvb_paged_prefill_fwd.argtypes = [ctypes.POINTER(KvbPagedPrefillParams), _vp]
        lib.kvb_paged_prefill_fwd.restype = ctypes.c_int
        lib.kvb_paged_materialize_peers.argtypes = [ctypes.POINTER(KvbPagedPrefillParams),
                                                    ctypes.POINTER(KvbPeerShards), _vp]
        lib.kvb_paged_materialize_peers.restype = ctypes.c_int
        lib.kvb_peer_barrier.argtypes = [ctypes.POINTER(KvbPeerSignals), ctypes.c_uint32,
                                         ctypes.c_int64, _vp, _vp]
        lib.kvb_peer_barrier.restype = ctypes.c_int
        lib.kvb_peer_shard_layout.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                              ctypes.c_int, ctypes.POINTER(ctypes.c_int64)]
        lib.kvb_peer_shard_layout.restype = ctypes.c_int64
        lib.kvb_decode_fwd.argtypes = [ctypes.POINTER(KvbPrefillParams), ctypes.c_int, _vp,
                                       ctypes.c_int64, _vp]
        lib.kvb_decode_fwd.restype = ctypes.c_int
        lib.kvb_decode_workspace_bytes.argtypes = [ctypes.POINTER(KvbPrefillParams), ctypes.c_int]
        lib.kvb_decode_workspace_bytes.restype = ctypes.c_int64
        lib.kvb_paged_materialize.argtypes = [ctypes.POINTER(KvbPagedPrefillParams), _vp]
        lib.kvb_paged_materialize.restype = ctypes.c_int
        lib.kvb_paged_prefill_fwd_noalloc.argtypes = [ctypes.POINTER(KvbPagedPrefillParams), _vp]
        lib.kvb_paged_prefill_fwd_noalloc.restype = ctypes.c_int
        lib.kvb_paged_prefill_workspace_bytes.argtypes = [ctypes.POINTER(KvbPagedPrefillParams)]
        lib.kvb_paged_prefill_workspace_bytes.restype = ctypes.c_int64
        lib.kvb_quantize_store.argtypes = [ctypes.POINTER(KvbQuantizeStoreParams), _vp]
        lib.kvb_quantize_store.restype = ctypes.c_int
        lib.kvb_quantize_store_batch.argtypes = [ctypes.POINTER(KvbQuantizeStoreBatch), _vp]
        lib.kvb_quantize_store_batch.restype = ctypes.c_int
        lib.kvb_cacheblend_fwd.argtypes = [ctypes.POINTER(KvbCacheBlendParams), _vp]
        lib.kvb_cacheblend_fwd.restype = ctypes.c_int
        lib.kvb_last_error.argtypes = []
        lib.kvb_last_error.restype = ctypes.c_char_p
        lib.kvb_abi_version.argtypes = []
        lib.kvb_abi_version.restype = ctypes.c_int
        _lib = lib
        return lib


calls_ok = 0   # successful attention entry-point calls (each launches the kernels once)


def check(rc: int, what: str) -> None:
    global calls_ok
    if rc == KVB_OK:
        calls_ok += 1
    else:
        msg = load().kvb_last_error().decode("utf-8", "replace")
        kind = {KVB_ERR_INVALID: "invalid argument", KVB_ERR_UNSUPPORTED: "unsupported",
                KVB_ERR_CUDA: "CUDA error"}.get(rc, f"error {rc}")
        raise RuntimeError(f"{what}: {kind}: {msg}")


def header_symbols(header_dir: str = None):
    """Function names declared in ``include/*.h`` (used to check the exports)."""
    header_dir = header_dir or _build.INCLUDE
    names = []
    for fn in sorted(os.listdir(header_dir)):
        if not fn.endswith(".h"):
            continue
        text = open(os.path.join(header_dir, fn)).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        for m in re.finditer(r"^\s*(?:const\s+)?[A-Za-z_][\w\s\*]*?\b(kvb_\w+)\s*\(", text, re.M):
            names.append(m.group(1))
    return sorted(set(names))
