"""Drop-in import name: ``import torch_kunlun`` loads the B200 backend
(torch_kunlun_b200) and exposes the reference's module layout
(torch_kunlun.kunlun, torch_kunlun.xccl, torch_kunlun.scaled_dot_product_attention)."""

import sys as _sys

import torch_kunlun_b200 as _impl
from torch_kunlun_b200 import kunlun, ops, xccl  # noqa: F401

_sys.modules[__name__ + ".kunlun"] = kunlun
_sys.modules[__name__ + ".kunlun.attention"] = kunlun.attention
_sys.modules[__name__ + ".xccl"] = xccl
_sys.modules[__name__ + ".ops"] = ops

__version__ = _impl.__version__
scaled_dot_product_attention = _impl.scaled_dot_product_attention

__all__ = ["kunlun", "xccl", "ops", "scaled_dot_product_attention"]
