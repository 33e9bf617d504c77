"""torch_kunlun on B200: the int16-quantised dense-op path of torch_kunlun
(mm / linear / addmm / bmm / baddbmm / matmul / conv2d, softmax, layer_norm,
scaled-dot-product attention and the ``bkcl`` collectives) on hand-written
sm_100a kernels, behind the same ``kunlun`` PrivateUse1 device.

Importing the package registers the device exactly as the reference's
``torch_kunlun/__init__.py:9-24`` does: the C++ extension registers the
PrivateUse1 backend, allocator, guard and hooks; Python renames PrivateUse1 to
``kunlun``, registers ``torch.kunlun`` and generates ``Tensor.kunlun()``-style
methods.  There is no CPU fallback for the named ops: if the native libraries
are missing the import fails.
"""

from __future__ import annotations

import ctypes
import os

import torch
from torch.utils.backend_registration import (
    generate_methods_for_privateuse1_backend,
    rename_privateuse1_backend,
)

_HERE = os.path.dirname(os.path.abspath(__file__))
_KERNEL_LIB = os.path.join(_HERE, "libtk_kernels.so")
if not os.path.exists(_KERNEL_LIB):
    raise ImportError(
        f"torch_kunlun_b200: {_KERNEL_LIB} is missing; build the native libraries with "
        "`python torch_kunlun_b200/_build.py`")
# _C links libtk_kernels.so by soname; load it first so the link resolves
# wherever the package directory lives.
_kernels = ctypes.CDLL(_KERNEL_LIB, mode=ctypes.RTLD_GLOBAL)

from . import _C  # noqa: E402,F401  (registers PrivateUse1, allocator, guard, hooks)
from . import kunlun  # noqa: E402
from . import xccl  # noqa: E402
from . import ops  # noqa: E402
from . import tp  # noqa: E402

__version__ = "0.1.0"

if torch._C._get_privateuse1_backend_name() != "kunlun":
    rename_privateuse1_backend("kunlun")
if not hasattr(torch, "kunlun"):
    torch._register_device_module("kunlun", kunlun)
if not hasattr(torch.Tensor, "kunlun"):
    generate_methods_for_privateuse1_backend()

scaled_dot_product_attention = kunlun.scaled_dot_product_attention

__all__ = ["kunlun", "xccl", "ops", "tp", "scaled_dot_product_attention"]
