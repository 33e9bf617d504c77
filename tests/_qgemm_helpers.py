"""Helpers shared by the GPU parity tests: drive tk_qgemm through the C ABI with
torch.cuda memory, and compute the matching oracle result on the CPU."""
import ctypes

import numpy as np
import torch

from oracle import oracle as O
from torch_kunlun_b200 import _capi as C


def _np(t):
    return t.detach().cpu().numpy()


def dtype_code(dt):
    return C.TK_DTYPE_F16 if dt == torch.float16 else C.TK_DTYPE_F32


def qgemm(a, b_nk, *, bias=None, addend=None, alpha=1.0, beta=0.0, act="none",
          per_slice=True, path="tc", debug=False):
    """out[b] = epilogue(q(a[b]) @ q(b_nk[b])^T) through the C ABI.

    a is [B,M,K] (any strides); b_nk is a [B,N,K] view (for a row-major W[N,K]
    pass W, for a row-major [K,N] operand pass its transpose view)."""
    assert a.is_cuda and b_nk.is_cuda and a.dim() == 3 and b_nk.dim() == 3
    B, M, K = a.shape
    N = b_nk.shape[1]
    out = torch.empty((B, M, N), dtype=a.dtype, device=a.device)
    d = C.QGemmDesc()
    d.dtype = dtype_code(a.dtype)
    d.batch, d.m, d.n, d.k = B, M, N, K
    d.a = a.data_ptr(); d.a_sb, d.a_sm, d.a_sk = a.stride()
    d.b = b_nk.data_ptr(); d.b_sb, d.b_sn, d.b_sk = b_nk.stride()
    d.out = out.data_ptr(); d.out_sb, d.out_sm = out.stride(0), out.stride(1)
    d.bias = bias.data_ptr() if bias is not None else None
    if addend is not None:
        d.addend = addend.data_ptr()
        d.add_sb, d.add_sm, d.add_sn = addend.stride()
    d.alpha, d.beta = float(alpha), float(beta)
    d.act = C.ACT[act]
    d.per_slice_scales = 1 if per_slice else 0
    L = C.lib()
    ws_bytes = L.tk_qgemm_workspace_size(ctypes.byref(d))
    ws = torch.empty(ws_bytes + 1024, dtype=torch.uint8, device=a.device)
    base = (ws.data_ptr() + 1023) // 1024 * 1024
    stream = torch.cuda.current_stream(a.device).cuda_stream
    dbg = None
    if debug:
        dbg = torch.zeros((3, M, N), dtype=torch.int32, device=a.device)
        C.check(L.tk_qgemm_debug(ctypes.byref(d), base, ws_bytes, dbg.data_ptr(), stream),
                "tk_qgemm_debug")
    elif path == "tc":
        C.check(L.tk_qgemm(ctypes.byref(d), base, ws_bytes, stream), "tk_qgemm")
    else:
        C.check(L.tk_qgemm_simt(ctypes.byref(d), base, ws_bytes, stream), "tk_qgemm_simt")
    torch.cuda.synchronize(a.device)
    return (out, dbg) if debug else out


def oracle_qgemm(a, b_nk, *, bias=None, addend=None, alpha=1.0, beta=0.0, act="none",
                 per_slice=True):
    """Oracle result for the same call (CPU)."""
    an = _np(a)
    bn = _np(b_nk)
    B = an.shape[0]
    act_code = O.ACT_CODES[act]
    outs = []
    if per_slice:
        amax_a = [O.amax(an[i]) for i in range(B)]
        amax_b = [O.amax(bn[i]) for i in range(B)]
    else:
        amax_a = [O.amax(an)] * B
        amax_b = [O.amax(bn)] * B
    bias_n = None if bias is None else _np(bias)
    add_n = None if addend is None else _np(addend)
    for i in range(B):
        qa = O.quant(an[i], amax_a[i])
        qb = O.quant(bn[i], amax_b[i])
        acc = O.gemm_i16_exact(qa, qb.T)
        outs.append(O.epilogue(acc, amax_a[i], amax_b[i], an.dtype, alpha, bias_n,
                               None if add_n is None else add_n[i], beta, act_code))
    return np.stack(outs)


def limb_accumulators(a2d, b_nk2d):
    """Oracle HH / MID / LL accumulators of one slice (int64)."""
    an, bn = _np(a2d), _np(b_nk2d)
    qa, qb = O.quant(an), O.quant(bn)
    ha, la = O.limbs(qa)
    hb, lb = O.limbs(qb)
    f = lambda x, y: (x.astype(np.float64) @ y.astype(np.float64).T).astype(np.int64)
    return f(ha, hb), f(ha, lb) + f(la, hb), f(la, lb)


def assert_bits_equal(got, want, what=""):
    """Bit-exact comparison; NaNs compare by NaN-ness."""
    g = np.asarray(got)
    w = np.asarray(want)
    assert g.shape == w.shape, (g.shape, w.shape)
    gn, wn = np.isnan(g), np.isnan(w)
    assert np.array_equal(gn, wn), f"{what}: NaN pattern differs"
    it = np.uint16 if g.dtype == np.float16 else np.uint32
    gb = np.where(gn, 0, g).view(it) if g.dtype != np.float16 else np.where(gn, np.float16(0), g).view(it)
    wb = np.where(wn, 0, w).astype(g.dtype).view(it)
    bad = np.nonzero(gb != wb)
    if bad[0].size:
        idx = tuple(b[:5] for b in bad)
        raise AssertionError(
            f"{what}: {bad[0].size} of {g.size} elements differ; first at {list(zip(*idx))}: "
            f"got {g[idx]} want {w[idx]}")
