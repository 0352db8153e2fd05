"""Drop-in for ``kvboost.flash_attn_ext`` backed by the sm_100a kernels.

Same public names and behaviour as ``src/kvboost/flash_attn_ext.py``:

* ``get_tier()`` / ``flash_attention_available()`` (``:34-61``): the tier is
  ``"kvboost_cuda"`` when the sm_100a library loads.
* ``_kvboost_flash_attn(Q, K, V, scale, causal, attn_mask)`` (``:68-103``): CUDA
  fp16/bf16 tensors run on the kernel; CPU tensors and fp32 keep the
  reference's vanilla SDPA behaviour (its CPU tier, unchanged).
* ``install_flash_attention`` / ``uninstall_flash_attention`` (``:141-212``):
  wrap the forward of modules whose class name ends in ``Attention`` /
  ``SdpaAttention`` / ``FlashAttention2`` (``:109-113``), return the number
  patched, idempotent through the ``_kvboost_attn_fn`` attribute.

What differs is that the patch actually routes.  The reference only swaps a
module-global ``scaled_dot_product_attention`` name, which HF >= 4.48 never
reads (attention goes through ``ALL_ATTENTION_FUNCTIONS``), so on current
transformers it patches nothing in effect.  Here the patched forward also
points the model's registry entry (``config._attn_implementation``) at
``kvboost_attention_forward`` for the duration of the call -- the same
registry-swap technique the reference's own paged interceptor uses
(``flash_attn_ext.py:407-420``).

Masks: HF hands reuse prefill an explicit boolean ``[B, 1, q, kv]`` mask
that is bottom-right causal.  ``classify_mask`` recognises it (and the
all-visible mask of a decode step); any other mask raises instead of
silently taking another path.
"""

from __future__ import annotations

import logging
import math
import sys
import types
import weakref
from typing import Optional

import torch
import torch.nn.functional as F

log = logging.getLogger(__name__)

# ── Tier detection ────────────────────────────────────────────────────────────

_TIER: str = "vanilla"
_LOAD_ERROR: Optional[BaseException] = None
try:
    from . import _lib
    _lib.load()
    _TIER = "kvboost_cuda"
except Exception as e:  # the library is required for every CUDA call below
    _LOAD_ERROR = e
    log.warning("kvboost_b200: CUDA library unavailable (%s)", e)


def flash_attention_available() -> bool:
    """Return True if an accelerated tier is active (``flash_attn_ext.py:56-58``)."""
    return _TIER != "vanilla"


def get_tier() -> str:
    """Return the active attention tier name (``flash_attn_ext.py:61-63``)."""
    return _TIER


def _require_library():
    if _TIER != "kvboost_cuda":
        raise RuntimeError(f"kvboost_b200 CUDA library is not available: {_LOAD_ERROR}")


# ── Mask recognition ──────────────────────────────────────────────────────────

# id(mask) -> (weakref to the mask, version, (q_len, kv_len), result); a hit
# requires the weakref to resolve to the very same tensor object.
_mask_cache: dict = {}
_MASK_CACHE_MAX = 16


def classify_mask(mask: Optional[torch.Tensor], q_len: int, kv_len: int) -> Optional[bool]:
    """Return ``True`` for a bottom-right causal mask, ``False`` for all-visible.

    ``mask`` is HF's boolean keep-mask or additive float mask, broadcastable to
    ``[B, H, q_len, kv_len]``.  ``None`` returns ``None`` (caller decides).  Any
    other pattern raises ``NotImplementedError``: the kernels implement exactly
    these two masks and nothing is silently routed elsewhere.  The result is
    cached per mask tensor (HF passes one mask object to every layer of a
    forward), so the device check runs once per forward.
    """
    if mask is None:
        return None
    ver = getattr(mask, "_version", 0)
    hit = _mask_cache.get(id(mask))
    if hit is not None and hit[0]() is mask and hit[1] == ver and hit[2] == (q_len, kv_len):
        return hit[3]
    if mask.shape[-2] not in (1, q_len) or mask.shape[-1] != kv_len:
        raise NotImplementedError(
            f"kvboost_b200: attention mask of shape {tuple(mask.shape)} does not match "
            f"q_len={q_len}, kv_len={kv_len}")
    keep = mask if mask.dtype == torch.bool else (mask == 0)
    keep = keep.reshape(-1, keep.shape[-2], kv_len)
    causal = torch.ones(q_len, kv_len, dtype=torch.bool, device=mask.device).tril(kv_len - q_len)
    if keep.shape[-2] == 1 and q_len > 1:
        raise NotImplementedError("kvboost_b200: a 1-row mask only fits a single-query step")
    is_causal = bool(torch.equal(keep, causal.expand_as(keep)))
    if is_causal:
        result = True
    elif bool(keep.all()):
        result = False
    else:
        raise NotImplementedError(
            "kvboost_b200: attention mask is neither bottom-right causal nor all-visible "
            "(padding / custom masks are not supported by the prefill kernels)")
    if len(_mask_cache) >= _MASK_CACHE_MAX:
        for k in [k for k, v in _mask_cache.items() if v[0]() is None] or list(_mask_cache)[:1]:
            _mask_cache.pop(k, None)
    _mask_cache[id(mask)] = (weakref.ref(mask), ver, (q_len, kv_len), result)
    return result


# ── Core attention function ───────────────────────────────────────────────────

def _kvboost_flash_attn(Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, scale: float,
                        causal: bool = True, attn_mask: Optional[torch.Tensor] = None,
                        ) -> torch.Tensor:
    """Unified dispatch (``flash_attn_ext.py:68-103``).  Q/K/V: ``[B, H, S, D]``.

    CUDA fp16/bf16 inputs run on the sm_100a kernel: ``attn_mask`` may be a
    bottom-right causal or all-visible mask (anything else raises), K/V may
    carry fewer heads than Q (GQA).  With no mask and ``causal=True`` the mask
    is bottom-right, which for ``S_q == S_kv`` is SDPA's ``is_causal``.  CPU and
    fp32 tensors take the reference's vanilla SDPA path unchanged.
    """
    if Q.is_cuda and Q.dtype in (torch.float16, torch.bfloat16):
        _require_library()
        from .ops import prefill_attention
        Sq, Skv = Q.size(2), K.size(2)
        if attn_mask is not None:
            causal = bool(classify_mask(attn_mask, Sq, Skv))
        elif causal and Sq != Skv:
            # SDPA's is_causal (what the reference would compute) is top-left.
            O, _ = prefill_attention(Q, K, V, float(scale), True, return_lse=False, top_left=True)
            return O
        O, _ = prefill_attention(Q, K, V, float(scale), causal, return_lse=False)
        return O
    return F.scaled_dot_product_attention(
        Q, K, V, attn_mask=attn_mask, scale=scale, is_causal=(causal and attn_mask is None))


def kvboost_attention_forward(module: torch.nn.Module, query: torch.Tensor, key: torch.Tensor,
                              value: torch.Tensor, attention_mask: Optional[torch.Tensor],
                              dropout: float = 0.0, scaling: Optional[float] = None,
                              is_causal: Optional[bool] = None, **kwargs):
    """HF attention-registry function (signature of ``sdpa_attention_forward``).

    query ``[B, Hq, q, D]``, key/value ``[B, Hkv, kv, D]`` (un-repeated GQA
    heads, any strides); returns ``(attn_output [B, q, Hq, D], None)``.
    Dropout is ignored (inference only, as in the reference's patched SDPA).
    """
    if kwargs.get("sliding_window") is not None or kwargs.get("softcap") is not None:
        raise NotImplementedError("kvboost_b200: sliding-window / softcapped attention")
    if not query.is_cuda:
        raise RuntimeError("kvboost_b200 attention runs on CUDA tensors only")
    _require_library()
    from .ops import prefill_attention
    q_len, kv_len = query.size(2), key.size(2)
    if scaling is None:
        scaling = 1.0 / math.sqrt(query.size(-1))
    if attention_mask is not None:
        causal = bool(classify_mask(attention_mask, q_len, kv_len))
    else:
        is_causal = is_causal if is_causal is not None else getattr(module, "is_causal", True)
        causal = bool(is_causal) and q_len > 1
    # decode steps, seams and short suffixes over long prefixes go to the
    # split-key kernel inside prefill_attention (ops.split_key_plan)
    out, _ = prefill_attention(query, key, value, float(scaling), causal, return_lse=False,
                               out_layout="bshd")
    return out, None


DECODE_MAX_Q = 16     # paged pools: query rows per step up to which attention reads the pool


# ── HuggingFace module patching ───────────────────────────────────────────────

_ATTN_MODULE_SUFFIXES = ("Attention", "SdpaAttention", "FlashAttention2")
_SDPA_ATTR = "_kvboost_attn_fn"
_LEGACY_SDPA_NAME = "scaled_dot_product_attention"


def _patched_sdpa(query, key, value, attn_mask=None, dropout_p=0.0, is_causal=False,
                  scale=None, **kwargs):
    """Replacement for a module-global ``scaled_dot_product_attention`` (HF <= 4.47)."""
    if scale is None:
        scale = 1.0 / math.sqrt(query.size(-1))
    return _kvboost_flash_attn(query, key, value, scale, is_causal, attn_mask)


def _registry_of(fn):
    g = getattr(fn, "__globals__", {})
    reg = g.get("ALL_ATTENTION_FUNCTIONS")
    if reg is not None and hasattr(reg, "get_interface"):
        return reg
    return None


def _patch_module(module: torch.nn.Module) -> bool:
    """Wrap one attention module's forward; False if it was already patched."""
    if hasattr(module, _SDPA_ATTR):
        return False
    original_forward = module.forward
    module.__dict__[_SDPA_ATTR] = _kvboost_flash_attn
    module.__dict__["_original_forward"] = original_forward
    fn = getattr(original_forward, "__func__", original_forward)
    registry = _registry_of(fn)

    def patched_forward(self, *args, **kwargs):
        if _PAGED_ATTR in self.__dict__:
            # a paged interceptor wraps this forward and has put its own function in
            # the registry for this call: leave it there
            return original_forward(*args, **kwargs)
        g = fn.__globals__ if hasattr(fn, "__globals__") else {}
        old_sdpa = g.get(_LEGACY_SDPA_NAME, None)
        had_sdpa = _LEGACY_SDPA_NAME in g
        key = None
        if registry is not None:
            cfg = getattr(self, "config", None)
            key = getattr(cfg, "_attn_implementation", None) or "sdpa"
            had_local = key in registry._local_mapping
            old_local = registry._local_mapping.get(key)
            registry[key] = kvboost_attention_forward
        if had_sdpa:
            g[_LEGACY_SDPA_NAME] = _patched_sdpa
        try:
            return original_forward(*args, **kwargs)
        finally:
            if had_sdpa:
                g[_LEGACY_SDPA_NAME] = old_sdpa
            if registry is not None:
                if had_local:
                    registry[key] = old_local
                else:
                    del registry[key]

    module.forward = types.MethodType(patched_forward, module)
    return True


def install_flash_attention(model: torch.nn.Module) -> int:
    """Patch every attention module of *model*; returns the number patched.

    Mirrors ``flash_attn_ext.py:179-198``.  Raises if the CUDA library is
    missing (the reference returned 0 on its vanilla tier; here there is no
    second tier to fall back to).
    """
    _require_library()
    patched = 0
    for name, module in model.named_modules():
        cls_name = type(module).__name__
        if any(cls_name.endswith(suffix) for suffix in _ATTN_MODULE_SUFFIXES):
            if _patch_module(module):
                patched += 1
                log.debug("flash_attn: patched %s (%s)", name, cls_name)
    if patched:
        log.info("flash_attn: patched %d attention module(s) -> tier=%s", patched, _TIER)
    return patched


def uninstall_flash_attention(model: torch.nn.Module) -> int:
    """Restore all patched attention modules (``flash_attn_ext.py:201-212``)."""
    restored = 0
    for module in model.modules():
        if "_original_forward" in module.__dict__:
            module.forward = module.__dict__.pop("_original_forward")
            module.__dict__.pop(_SDPA_ATTR, None)
            restored += 1
    return restored


# ── Paged attention (flash_attn_ext.py:240-453) ───────────────────────────────

_PAGED_ATTR = "_kvboost_paged_layer"


def _make_paged_attn_fn(layer_idx: int, state: dict):
    """Registry attention function reading K/V from the state's block pool.

    Same protocol as the reference's ``sdpa_style`` function
    (``flash_attn_ext.py:273-328``): the new tokens' K/V (everything past
    ``state["_write_slot"]`` when HF concatenated a cache, else all of ``key``)
    are appended to the pool at the write slot, extending ``state["block_table"]``;
    the queries then attend to the pool.  Here the append is one device scatter,
    the tokens before the write slot are read from the pool through the block
    table and the new K/V straight from the call (``kvb_paged_prefill_fwd``), with
    bottom-right causality; ``state["top_left"] = True`` selects the reference's
    SDPA ``is_causal`` alignment instead.
    """
    from .paged import block_table_tensor, paged_attention_fwd, paged_prefill_attention

    def paged_fn(module, query, key, value, attention_mask=None, dropout=0.0, scaling=None,
                 is_causal=None, **kwargs):
        allocator = state["allocator"]
        write_slot = int(state["_write_slot"])
        if query.size(0) != 1:
            raise NotImplementedError("paged attention serves one sequence per forward")
        if scaling is None:
            scaling = 1.0 / math.sqrt(query.size(-1))
        if key.size(2) > write_slot:
            k_new, v_new = key[:, :, write_slot:], value[:, :, write_slot:]
        else:
            k_new, v_new = key, value
        table, _ = allocator.append_kv(layer_idx, state["block_table"], write_slot,
                                       k_new[0], v_new[0])
        state["block_table"] = table
        n = write_slot + k_new.size(2)
        if state.get("top_left") or query.size(2) <= DECODE_MAX_Q:
            # decode steps (and the reference's mask alignment): attend over the pool
            out = paged_attention_fwd(query, allocator, [table], [n], layer_idx,
                                      causal=query.size(2) > 1, scale=scaling,
                                      top_left=bool(state.get("top_left")))
        else:
            out, _ = paged_prefill_attention(
                query, k_new.to(query.dtype).contiguous(), v_new.to(query.dtype).contiguous(),
                allocator, layer_idx, block_table_tensor([table], query.device), write_slot,
                softmax_scale=scaling, causal=True, return_lse=False)
        return out.transpose(1, 2), None

    return paged_fn


def install_paged_attention(model: torch.nn.Module, state: dict) -> int:
    """Point every attention module of *model* at the state's block pool
    (``flash_attn_ext.py:367-440``); returns the number of modules patched.

    ``state``: ``allocator`` (a 16-bit ``DeviceBlockAllocator`` with one pool per
    layer), ``block_table`` (list of block ids, extended in place), ``_write_slot``
    (logical slot of the next token, advanced by the caller after each forward).
    Layers are numbered in module order, as in the reference.
    """
    _require_library()
    patched = 0
    layer_idx = 0
    for name, module in model.named_modules():
        cls_name = type(module).__name__
        if not any(cls_name.endswith(s) for s in _ATTN_MODULE_SUFFIXES):
            continue
        if _PAGED_ATTR in module.__dict__:
            continue
        original_forward = module.forward
        module.__dict__[_PAGED_ATTR] = layer_idx
        module.__dict__["_paged_original_forward"] = original_forward
        # a module already routed by install_flash_attention keeps the model's own
        # forward under _original_forward: the registry is found through that
        base = module.__dict__.get("_original_forward", original_forward)
        fn = getattr(base, "__func__", base)
        registry = _registry_of(fn)
        if registry is None:
            raise NotImplementedError("paged attention needs transformers' attention registry")
        paged_fn = _make_paged_attn_fn(layer_idx, state)

        def paged_forward(self, *args, _fn=paged_fn, _orig=original_forward, **kw):
            cfg = getattr(self, "config", None)
            key = getattr(cfg, "_attn_implementation", None) or "sdpa"
            had = key in registry._local_mapping
            old = registry._local_mapping.get(key)
            registry[key] = _fn
            try:
                return _orig(*args, **kw)
            finally:
                if had:
                    registry[key] = old
                else:
                    del registry[key]

        module.forward = types.MethodType(paged_forward, module)
        layer_idx += 1
        patched += 1
    return patched


def uninstall_paged_attention(model: torch.nn.Module) -> int:
    """Restore the modules ``install_paged_attention`` patched (``flash_attn_ext.py:443-453``)."""
    restored = 0
    for module in model.modules():
        if "_paged_original_forward" in module.__dict__:
            module.forward = module.__dict__.pop("_paged_original_forward")
            module.__dict__.pop(_PAGED_ATTR, None)
            restored += 1
    return restored


# ── Reference injection ───────────────────────────────────────────────────────

def inject_into_reference() -> None:
    """Register the sm_100a op as ``kvboost._flash_attn_cuda``.

    Call before importing ``kvboost``: the reference's import-time probe
    (``flash_attn_ext.py:37-39``) then finds the module, reports tier
    ``"kvboost_cuda"`` and routes ``_kvboost_flash_attn`` to
    ``flash_attn_fwd`` (``:80-84``).
    """
    from . import _flash_attn_cuda
    sys.modules["kvboost._flash_attn_cuda"] = _flash_attn_cuda
    pkg = sys.modules.get("kvboost")
    if pkg is not None:
        setattr(pkg, "_flash_attn_cuda", _flash_attn_cuda)
