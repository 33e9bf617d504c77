"""ctypes binding of the C ABI in include/tk_kernels.h (libtk_kernels.so).

The PrivateUse1 backend (_C) links the library directly; this binding exists
for callers that drive the kernels with raw device pointers (the parity
tests, the benchmark's C-ABI leg, and non-torch embedders).  It performs no
computation of its own and fails loudly when the library is missing.
"""

from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libtk_kernels.so")

TK_OK = 0
TK_DTYPE_F16 = 0
TK_DTYPE_F32 = 1
ACT = {"none": 0, "relu": 1, "gelu": 2, "gelu_tanh": 3, "silu": 4}

# Every entry point declared in include/tk_kernels.h.
EXPORTED = [
    "tk_abi_version", "tk_last_error_string", "tk_device_error", "tk_amax",
    "tk_quantize_limbs", "tk_qgemm_workspace_size", "tk_qgemm", "tk_qgemm_simt",
    "tk_qgemm_debug", "tk_qgemm_from_limbs", "tk_copy_strided", "tk_fill_strided",
    "tk_binary", "tk_unary", "tk_silu_mul", "tk_conv2d_workspace_size", "tk_conv2d_q16",
    "tk_softmax", "tk_layer_norm", "tk_qgemm_noalloc", "tk_sdpa_workspace_size", "tk_sdpa_q16",
    "tk_reduce_sum", "tk_conv3d_workspace_size", "tk_conv3d_q16", "tk_qgemm_scatter_rows",
    "tk_conv3d_wgrad_workspace_size", "tk_conv3d_wgrad_q16", "tk_silu_mul_amax",
]


class QGemmDesc(ctypes.Structure):
    """Mirror of tk_qgemm_desc_t."""
    _fields_ = [
        ("dtype", ctypes.c_int),
        ("batch", ctypes.c_int64), ("m", ctypes.c_int64), ("n", ctypes.c_int64),
        ("k", ctypes.c_int64),
        ("a", ctypes.c_void_p),
        ("a_sb", ctypes.c_int64), ("a_sm", ctypes.c_int64), ("a_sk", ctypes.c_int64),
        ("b", ctypes.c_void_p),
        ("b_sb", ctypes.c_int64), ("b_sn", ctypes.c_int64), ("b_sk", ctypes.c_int64),
        ("out", ctypes.c_void_p),
        ("out_sb", ctypes.c_int64), ("out_sm", ctypes.c_int64),
        ("bias", ctypes.c_void_p),
        ("addend", ctypes.c_void_p),
        ("add_sb", ctypes.c_int64), ("add_sm", ctypes.c_int64), ("add_sn", ctypes.c_int64),
        ("alpha", ctypes.c_float), ("beta", ctypes.c_float),
        ("act", ctypes.c_int),
        ("per_slice_scales", ctypes.c_int),
        ("amax_a", ctypes.c_void_p),
        ("amax_b", ctypes.c_void_p),
        ("amax_out", ctypes.c_void_p),
    ]


_lib = None


class SdpaDesc(ctypes.Structure):
    """Mirror of tk_sdpa_desc_t."""
    _fields_ = [
        ("dtype", ctypes.c_int),
        ("batch", ctypes.c_int64), ("heads", ctypes.c_int64), ("l", ctypes.c_int64),
        ("s", ctypes.c_int64), ("e", ctypes.c_int64), ("ev", ctypes.c_int64),
        ("q", ctypes.c_void_p), ("q_strides", ctypes.c_int64 * 4),
        ("k", ctypes.c_void_p), ("k_strides", ctypes.c_int64 * 4),
        ("v", ctypes.c_void_p), ("v_strides", ctypes.c_int64 * 4),
        ("out", ctypes.c_void_p), ("out_strides", ctypes.c_int64 * 4),
        ("mask", ctypes.c_void_p), ("mask_strides", ctypes.c_int64 * 4),
        ("causal", ctypes.c_int),
        ("scale", ctypes.c_float),
    ]


class ConvWgradDesc(ctypes.Structure):
    """Mirror of tk_conv3d_wgrad_desc_t."""
    _fields_ = [("dtype", ctypes.c_int)] + [
        (n, ctypes.c_int64) for n in (
            "n", "c", "d", "h", "w", "f", "kd", "kh", "kw", "stride_d", "stride_h", "stride_w",
            "pad_d", "pad_h", "pad_w", "dil_d", "dil_h", "dil_w", "groups")] + [
        ("x", ctypes.c_void_p), ("grad_out", ctypes.c_void_p), ("grad_weight", ctypes.c_void_p),
        ("amax_x", ctypes.c_void_p), ("amax_g", ctypes.c_void_p)]


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"torch_kunlun_b200: {LIB_PATH} is missing; build it with "
                "`python torch_kunlun_b200/_build.py` (there is no CPU fallback)")
        L = ctypes.CDLL(LIB_PATH)
        vp, i64, i32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
        L.tk_abi_version.restype = i32
        L.tk_last_error_string.restype = ctypes.c_char_p
        L.tk_device_error.argtypes = [i32, ctypes.POINTER(ctypes.c_uint)]
        L.tk_amax.argtypes = [i32, vp, i64, i64, i64, vp, vp]
        L.tk_quantize_limbs.argtypes = [i32, vp, i64, i64, i64, i64, i64, i64, vp, i64, vp, vp]
        L.tk_qgemm_workspace_size.argtypes = [ctypes.POINTER(QGemmDesc)]
        L.tk_sdpa_workspace_size.argtypes = [ctypes.POINTER(SdpaDesc)]
        L.tk_sdpa_workspace_size.restype = ctypes.c_size_t
        L.tk_sdpa_q16.argtypes = [ctypes.POINTER(SdpaDesc), vp, ctypes.c_size_t, vp]
        L.tk_qgemm_workspace_size.restype = ctypes.c_size_t
        for name in ("tk_qgemm", "tk_qgemm_simt"):
            getattr(L, name).argtypes = [ctypes.POINTER(QGemmDesc), vp, ctypes.c_size_t, vp]
        L.tk_qgemm_from_limbs.argtypes = [ctypes.POINTER(QGemmDesc), vp, vp, vp, vp, vp]
        L.tk_qgemm_noalloc.argtypes = [ctypes.POINTER(QGemmDesc), vp]
        L.tk_qgemm_debug.argtypes = [ctypes.POINTER(QGemmDesc), vp, ctypes.c_size_t, vp, vp]
        L.tk_conv3d_wgrad_workspace_size.argtypes = [ctypes.POINTER(ConvWgradDesc)]
        L.tk_conv3d_wgrad_workspace_size.restype = ctypes.c_size_t
        L.tk_conv3d_wgrad_q16.argtypes = [ctypes.POINTER(ConvWgradDesc), vp, ctypes.c_size_t, vp]
        _lib = L
    return _lib


def check(rc: int, what: str) -> None:
    if rc != TK_OK:
        msg = lib().tk_last_error_string().decode(errors="replace")
        raise RuntimeError(f"{what} failed (status {rc}): {msg}")


def device_error(device: int = 0) -> int:
    code = ctypes.c_uint(0)
    check(lib().tk_device_error(device, ctypes.byref(code)), "tk_device_error")
    return int(code.value)
