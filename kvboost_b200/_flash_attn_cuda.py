"""Drop-in for the reference extension module ``kvboost._flash_attn_cuda``.

Same name, signature, outputs and error behaviour as the pybind op in
``src/kvboost/csrc/flash_attn.cpp:58-102``::

    flash_attn_fwd(Q, K, V, scale, causal=True) -> (O, L)

* Q, K, V: contiguous CUDA ``[B, H, S, D]`` float16/bfloat16, D in {64, 96, 128}.
* O: ``empty_like(Q)``; L: float32 ``[B, H, S_q]`` natural-log logsumexp of the
  scaled scores (``flash_attn_kernel.cu:236-245``).
* Argument errors raise ``RuntimeError`` with the reference's messages
  (``check_inputs``, ``flash_attn.cpp:16-54``).

Where the reference silently indexed K/V with Q's length (it never checks
``Q.size(2) == K.size(2)``, ``flash_attn.cpp:24-25``), this op accepts
``S_q != S_kv`` and applies the bottom-right causal mask; for ``S_q == S_kv``
that is exactly the reference's top-left mask.  The launch goes on the
current torch stream instead of the legacy default stream.

``kvboost_b200.flash_attn_ext.inject_into_reference()`` registers this module
as ``kvboost._flash_attn_cuda`` so an unmodified KVBoost reports tier
``"kvboost_cuda"`` and calls it.
"""

from __future__ import annotations

from typing import Tuple

import torch

from . import _lib


def _check_inputs(Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor) -> None:
    """Restates ``check_inputs`` (``flash_attn.cpp:16-54``) with its messages."""
    if Q.dim() != 4:
        raise RuntimeError(f"Q must be 4-D [B, H, S, D], got {Q.dim()}")
    if K.dim() != 4:
        raise RuntimeError(f"K must be 4-D [B, H, S, D], got {K.dim()}")
    if V.dim() != 4:
        raise RuntimeError(f"V must be 4-D [B, H, S, D], got {V.dim()}")
    if not (Q.size(0) == K.size(0) and Q.size(0) == V.size(0)):
        raise RuntimeError(
            f"Batch dimension mismatch: Q={Q.size(0)} K={K.size(0)} V={V.size(0)}")
    if not (Q.size(1) == K.size(1) and Q.size(1) == V.size(1)):
        raise RuntimeError("Head dimension mismatch")
    if K.size(2) != V.size(2):
        raise RuntimeError(f"K/V sequence length mismatch: K={K.size(2)} V={V.size(2)}")
    if not (Q.size(3) == K.size(3) and Q.size(3) == V.size(3)):
        raise RuntimeError("Head-dim mismatch")
    if Q.dtype not in (torch.float16, torch.bfloat16):
        raise RuntimeError(f"flash_attn only supports float16 or bfloat16, got {Q.dtype}")
    if not (Q.dtype == K.dtype and Q.dtype == V.dtype):
        raise RuntimeError("Q, K, V must have the same dtype")
    if not Q.is_cuda:
        raise RuntimeError("Q must be on CUDA")
    if not K.is_cuda:
        raise RuntimeError("K must be on CUDA")
    if not V.is_cuda:
        raise RuntimeError("V must be on CUDA")
    if not Q.is_contiguous():
        raise RuntimeError("Q must be contiguous")
    if not K.is_contiguous():
        raise RuntimeError("K must be contiguous")
    if not V.is_contiguous():
        raise RuntimeError("V must be contiguous")
    D = Q.size(3)
    if D not in (64, 96, 128):
        raise RuntimeError(f"flash_attn supports head_dim ∈ {{64, 96, 128}}, got {D}")


def flash_attn_fwd(Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, scale: float,
                   causal: bool = True) -> Tuple[torch.Tensor, torch.Tensor]:
    """FlashAttention forward.  Returns ``(O [B,H,S,D], L [B,H,S] float32)``."""
    _check_inputs(Q, K, V)
    B, H, S, D = Q.shape
    O = torch.empty_like(Q)
    L = torch.empty(B, H, S, dtype=torch.float32, device=Q.device)
    if B == 0 or H == 0 or S == 0:
        return O, L
    lib = _lib.load()
    with torch.cuda.device(Q.device):
        stream = torch.cuda.current_stream(Q.device).cuda_stream
        if K.size(2) == S:
            rc = lib.kvb_flash_attn_fwd(
                Q.data_ptr(), K.data_ptr(), V.data_ptr(), O.data_ptr(), L.data_ptr(),
                B, H, S, D, _lib.KVB_DTYPE_BF16 if Q.dtype == torch.bfloat16 else _lib.KVB_DTYPE_FP16,
                float(scale), 1 if causal else 0, stream)
            _lib.check(rc, "flash_attn_fwd")
            return O, L
    from .ops import prefill_attention
    O, L = prefill_attention(Q, K, V, softmax_scale=float(scale), causal=causal, out=O)
    return O, L
