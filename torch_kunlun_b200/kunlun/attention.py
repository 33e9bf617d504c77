"""Scaled-dot-product attention on the kunlun device.

Same signature and semantics as the reference's
torch_kunlun/kunlun/attention.py:36-107 -- shapes follow PyTorch SDPA
(query (..., L, E), key (..., S, E), value (..., S, Ev)), a boolean mask is
True where attention is *masked out* (contributing -1e4), ``is_causal`` adds
-1e4 above the diagonal, no dropout -- computed by the backend's native
``sdpa`` (per-slice quantised QK^T with the scale and mask applied in the GEMM
epilogue, softmax, per-slice quantised PV).
"""

from __future__ import annotations

from typing import Optional

import torch

from .. import _C


def scaled_dot_product_attention(
    query: torch.Tensor,
    key: torch.Tensor,
    value: torch.Tensor,
    attn_mask: Optional[torch.Tensor] = None,
    dropout_p: float = 0.0,
    is_causal: bool = False,
    scale: Optional[float] = None,
) -> torch.Tensor:
    if dropout_p != 0.0:
        raise NotImplementedError("kunlun attention dropout is not implemented (no device RNG)")
    if query.dim() < 2 or key.dim() < 2 or value.dim() < 2:
        raise ValueError("attention expects tensors with at least 2 dimensions")
    if query.shape[-1] != key.shape[-1]:
        raise ValueError("query/key head dimensions must match")
    if key.shape[-2] != value.shape[-2]:
        raise ValueError("key/value sequence lengths must match")
    return _C.sdpa(query, key, value, attn_mask, bool(is_causal),
                   None if scale is None else float(scale))


__all__ = ["scaled_dot_product_attention"]
