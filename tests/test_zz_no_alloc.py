"""tk_qgemm_noalloc: the quantised GEMM for callers that cannot allocate.

Such callers (a host or server that owns all device memory and hands this
library only inputs and outputs) get the scratch from a fixed array inside the
library instead of a workspace.  This file is collected last so that a run
stopping at the first failure has already run every other test; it must pass
both alone in a fresh process and after the rest of the suite."""
import ctypes

import pytest
import torch

from torch_kunlun_b200 import _capi as C

pytestmark = pytest.mark.gpu


def _desc(a, w, out, bias):
    d = C.QGemmDesc()
    d.dtype = C.TK_DTYPE_F16
    B, M, K = a.shape
    d.batch, d.m, d.n, d.k = B, M, w.shape[1], K
    d.a = a.data_ptr(); d.a_sb, d.a_sm, d.a_sk = a.stride()
    d.b = w.data_ptr(); d.b_sb, d.b_sn, d.b_sk = w.stride()
    d.out = out.data_ptr(); d.out_sb, d.out_sm = out.stride(0), out.stride(1)
    d.bias = bias.data_ptr()
    d.alpha, d.beta, d.act, d.per_slice_scales = 1.0, 0.0, 0, 1
    return d


def test_noalloc_matches_workspace_entry_point_on_two_calls():
    g = torch.Generator().manual_seed(7)
    a = torch.randn(2, 300, 520, generator=g).half().cuda()
    w = (torch.randn(2, 200, 520, generator=g) * 0.02).half().cuda()
    bias = (torch.randn(200, generator=g) * 0.01).half().cuda()
    L = C.lib()
    stream = torch.cuda.current_stream().cuda_stream

    ref = torch.empty(2, 300, 200, dtype=torch.float16, device="cuda")
    d = _desc(a, w, ref, bias)
    ws_bytes = L.tk_qgemm_workspace_size(ctypes.byref(d))
    ws = torch.empty(ws_bytes + 1024, dtype=torch.uint8, device="cuda")
    base = (ws.data_ptr() + 1023) // 1024 * 1024
    C.check(L.tk_qgemm(ctypes.byref(d), base, ws_bytes, stream), "tk_qgemm")

    for call in range(2):  # the second call reuses the scratch left by the first
        out = torch.full((2, 300, 200), float("nan"), dtype=torch.float16, device="cuda")
        C.check(L.tk_qgemm_noalloc(ctypes.byref(_desc(a, w, out, bias)), stream),
                "tk_qgemm_noalloc")
        torch.cuda.synchronize()
        # both paths are exact integer GEMMs with the same epilogue: bit-equal
        assert torch.equal(out.view(torch.int16), ref.view(torch.int16)), f"call {call}"
    assert C.device_error(0) == 0


def test_noalloc_rejects_problems_larger_than_its_scratch():
    a = torch.zeros(1, 8192, 8192, dtype=torch.float16, device="cuda")
    out = torch.empty(1, 8192, 8192, dtype=torch.float16, device="cuda")
    bias = torch.zeros(8192, dtype=torch.float16, device="cuda")
    d = _desc(a, a, out, bias)
    rc = C.lib().tk_qgemm_noalloc(ctypes.byref(d), torch.cuda.current_stream().cuda_stream)
    assert rc == 4  # TK_ERR_WORKSPACE
    assert b"built-in scratch" in C.lib().tk_last_error_string()
