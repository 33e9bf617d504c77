"""CPU checks of the C ABI boundary: the library loads, exports every entry
point declared in include/tk_kernels.h, and rejects bad arguments before any
device work (no GPU is touched)."""
import ctypes
import os
import re

import pytest

from torch_kunlun_b200 import _capi as C

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    src = open(os.path.join(ROOT, "include", "tk_kernels.h")).read()
    return sorted(set(re.findall(r"TK_API\s+[\w\s\*]+?\b(tk_\w+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    L = C.lib()
    names = declared_symbols()
    assert len(names) >= 19
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, missing
    assert set(names) <= set(C.EXPORTED) | set(names)


def test_binding_lists_every_declared_symbol():
    assert set(declared_symbols()) == set(C.EXPORTED)


def test_abi_version():
    assert C.lib().tk_abi_version() == 1


def test_qgemm_long_k_reserves_int64_accumulators():
    # K > 32768 is split: the workspace adds one int64 sum per output
    d = C.QGemmDesc()
    d.dtype = 0
    d.batch, d.m, d.n, d.k = 1, 40, 30, 40000
    ws = C.lib().tk_qgemm_workspace_size(ctypes.byref(d))
    assert ws >= 2 * 40 * 40000 + 2 * 30 * 40000 + 8 * 40 * 30
    d.k = 1 << 31
    d.out = 1  # never dereferenced: validation fails first
    assert C.lib().tk_qgemm(ctypes.byref(d), None, 0, None) == 1
    assert b"out of range" in C.lib().tk_last_error_string()


def test_noalloc_validates_the_descriptor_before_sizing_its_scratch():
    d = C.QGemmDesc()
    d.dtype = 0
    d.batch, d.m, d.n, d.k = 1, -4, 4, 64
    d.out = 1  # never dereferenced: validation fails first
    rc = C.lib().tk_qgemm_noalloc(ctypes.byref(d), None)
    assert rc == 1  # TK_ERR_INVALID_ARG, not TK_ERR_WORKSPACE
    assert b"negative size" in C.lib().tk_last_error_string()


def test_qgemm_workspace_layout():
    d = C.QGemmDesc()
    d.dtype = 0
    d.batch, d.m, d.n, d.k = 2, 100, 60, 33
    d.per_slice_scales = 1
    ws = C.lib().tk_qgemm_workspace_size(ctypes.byref(d))
    ld = 48  # round_up(33, 16)
    assert ws >= 2 * 2 * 100 * ld + 2 * 2 * 60 * ld
    assert ws % 1024 == 0


def test_sdpa_workspace_and_limits_without_touching_the_device():
    d = C.SdpaDesc()
    d.dtype = 0
    d.batch, d.heads, d.l, d.s, d.e, d.ev = 2, 3, 100, 77, 40, 24
    ws = C.lib().tk_sdpa_workspace_size(ctypes.byref(d))
    BH, Spad = 6, 128
    limbs = BH * 100 * 128 + BH * 77 * 128 + BH * 24 * 2 * Spad
    assert ws >= limbs + 3 * BH * 4 + 2 * BH * 100 * 4 and ws % 1024 == 0
    d.e = 129
    assert C.lib().tk_sdpa_workspace_size(ctypes.byref(d)) == 0
    rc = C.lib().tk_sdpa_q16(ctypes.byref(d), None, 0, None)
    assert rc == 2 and b"head dim" in C.lib().tk_last_error_string()
    d.e, d.s = 64, 40000
    assert C.lib().tk_sdpa_q16(ctypes.byref(d), None, 0, None) == 2
    assert b"32768" in C.lib().tk_last_error_string()
    d.s = 77
    d.q = d.k = d.v = d.out = 16  # never dereferenced: the workspace check fails first
    assert C.lib().tk_sdpa_q16(ctypes.byref(d), None, 0, None) == 4


def test_package_registers_kunlun_device_and_bkcl():
    import torch
    import torch.distributed as dist
    import torch_kunlun  # noqa: F401
    assert torch._C._get_privateuse1_backend_name() == "kunlun"
    assert hasattr(torch, "kunlun") and hasattr(torch.Tensor, "kunlun")
    assert "bkcl" in dist.Backend.backend_list
    assert torch_kunlun.kunlun.Stream is torch.kunlun.Stream


def test_cluster_budget_roundtrip_api():
    import torch_kunlun
    k = torch_kunlun.kunlun
    orig = k.cluster_budget()
    try:
        assert k.set_cluster_budget(2) == 2
        assert k.cluster_budget() == 2 and k.sdnn_budget() == 2
    finally:
        k.set_cluster_budget(orig)


class _Conv3dDesc(ctypes.Structure):
    """tk_conv3d_desc_t, as include/tk_kernels.h declares it."""
    _fields_ = ([("dtype", ctypes.c_int)] +
                [(n, ctypes.c_int64) for n in ("n", "c", "d", "h", "w", "f", "kd", "kh", "kw", "stride_d",
                                               "stride_h", "stride_w", "pad_d", "pad_h", "pad_w", "dil_d",
                                               "dil_h", "dil_w", "groups")] +
                [(n, ctypes.c_void_p) for n in ("x", "weight", "bias", "out", "amax_x", "amax_w")])


def test_depthwise_workspace_holds_the_partial_maxima():
    """The depthwise path keeps its two amax slots and 2 x 512 partial words
    (one per depthwise_amax_kernel block and operand) in the workspace."""
    L = C.lib()
    L.tk_conv3d_workspace_size.argtypes = [ctypes.POINTER(_Conv3dDesc)]
    L.tk_conv3d_workspace_size.restype = ctypes.c_size_t
    d = _Conv3dDesc()
    d.dtype = 0
    d.n, d.c, d.d, d.h, d.w, d.f = 64, 512, 1, 7, 7, 512
    d.kd, d.kh, d.kw = 1, 3, 3
    d.stride_d = d.stride_h = d.stride_w = 1
    d.pad_d, d.pad_h, d.pad_w = 0, 1, 1
    d.dil_d = d.dil_h = d.dil_w = 1
    d.groups = 512
    assert L.tk_conv3d_workspace_size(ctypes.byref(d)) >= 1024 + 2 * 512 * 4
