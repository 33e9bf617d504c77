"""CPU oracle for the int16-quantised dense path (test infrastructure only).

Nothing in the shipped package imports this module: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s ``cpu_baseline`` leg do, and
only as the checker.  The arithmetic contract is stated in ``tk_oracle.c``;
this module wraps the C restatement with numpy and composes the reference's
operator-level dataflow from it:

* ``fc``       -- csrc/ops.cpp:210-230 (per-tensor quantised fc), with the bias
                  added after rounding as in csrc/ops.cpp:480-495 and the
                  addmm alpha/beta order of csrc/autograd.cpp:192-218.
* ``bmm``      -- csrc/ops_nn.cpp:199-221 (one fc per batch slice, so every
                  slice has its own scales).
* ``baddbmm``  -- csrc/linalg_extra.cpp:85-93.
* ``conv2d``   -- csrc/ops.cpp:237-285 (whole-tensor scales, bias afterwards).
* ``sdpa``     -- torch_kunlun/kunlun/attention.py:36-107 (bmm, scale, mask
                  add, softmax, bmm).

Parity status: unpinned at bit level -- the reference's arithmetic is in a
closed vendor library with no golden vectors; see tk_oracle.c.

Large GEMMs use an exact shortcut: int16 x int16 products are < 2^30 and, for
K < 2^23, every partial sum is an integer below 2^53, so a float64 matmul of
the integer-valued matrices is exact.  ``tests/test_oracle.py`` checks the
shortcut against the scalar int64 loop.
"""

from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libtk_oracle.so")
_lib = None

F16 = 0
F32 = 1
ACT_NONE = 0
ACT_RELU = 1
ACT_GELU = 2
ACT_GELU_TANH = 3
ACT_SILU = 4
ACT_CODES = {"none": ACT_NONE, "relu": ACT_RELU, "gelu": ACT_GELU, "gelu_tanh": ACT_GELU_TANH,
             "silu": ACT_SILU}
Q = 32767.0


def build() -> str:
    """Compile the C oracle with its Makefile (strict IEEE flags)."""
    src = os.path.join(_HERE, "tk_oracle.c")
    if not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(src):
        subprocess.check_call(["make", "-s", "-C", _HERE])
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(_LIB_PATH)
        p, i64, f32, f64, i32 = (ctypes.c_void_p, ctypes.c_int64, ctypes.c_float,
                                 ctypes.c_double, ctypes.c_int)
        L.tko_f16_to_f32.argtypes = [ctypes.c_uint16]
        L.tko_f16_to_f32.restype = f32
        L.tko_f64_to_f16.argtypes = [f64]
        L.tko_f64_to_f16.restype = ctypes.c_uint16
        L.tko_f32_to_f16.argtypes = [f32]
        L.tko_f32_to_f16.restype = ctypes.c_uint16
        L.tko_amax2d.argtypes = [p, i32, i64, i64, i64, i64]
        L.tko_amax2d.restype = f32
        L.tko_amax.argtypes = [p, i32, i64]
        L.tko_amax.restype = f32
        L.tko_quant_inv.argtypes = [f32]
        L.tko_quant_inv.restype = f32
        L.tko_quant2d.argtypes = [p, i32, i64, i64, i64, i64, f32, p]
        L.tko_quant.argtypes = [p, i32, i64, f32, p]
        L.tko_limbs.argtypes = [p, i64, p, p]
        L.tko_gemm_i16.argtypes = [i64, i64, i64, p, i64, i64, p, i64, i64, p]
        L.tko_dequant_scale.argtypes = [f32, f32]
        L.tko_dequant_scale.restype = f64
        L.tko_epilogue.argtypes = [i32, i64, i64, p, f32, f32, f32, p, p, i64, i64,
                                   f32, i32, p, i64]
        L.tko_conv2d_i16.argtypes = [i64] * 14 + [p, p, p]
        L.tko_act64.argtypes = [f64, i32]
        L.tko_act64.restype = f64
        L.tko_act.argtypes = [p, i32, i64, i32, p]
        L.tko_silu_mul.argtypes = [p, p, i32, i64, p]
        L.tko_softmax.argtypes = [p, i32, i64, i64, i32, p]
        L.tko_layer_norm.argtypes = [p, i32, i64, i64, p, p, i32, f64, p, p, p]
        L.tko_num_threads.restype = i32
        _lib = L
    return _lib


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


def _dt(a: np.ndarray) -> int:
    if a.dtype == np.float16:
        return F16
    if a.dtype == np.float32:
        return F32
    raise TypeError(f"oracle supports float16/float32, got {a.dtype}")


# ---- scalar helpers --------------------------------------------------------


def f64_to_f16_bits(v: float) -> int:
    return int(lib().tko_f64_to_f16(float(v)))


def amax(x: np.ndarray) -> np.float32:
    x = np.ascontiguousarray(x)
    return np.float32(lib().tko_amax(_ptr(x), _dt(x), x.size))


def quant(x: np.ndarray, a: float | None = None) -> np.ndarray:
    """int16 quantisation of a whole tensor with one scale."""
    x = np.ascontiguousarray(x)
    if a is None:
        a = amax(x)
    q = np.empty(x.shape, dtype=np.int16)
    lib().tko_quant(_ptr(x), _dt(x), x.size, float(a), _ptr(q))
    return q


def limbs(q: np.ndarray):
    q = np.ascontiguousarray(q, dtype=np.int16)
    hi = np.empty(q.shape, dtype=np.int8)
    lo = np.empty(q.shape, dtype=np.uint8)
    lib().tko_limbs(_ptr(q), q.size, _ptr(hi), _ptr(lo))
    return hi, lo


def dequant_scale(amax_a: float, amax_b: float) -> float:
    return float(lib().tko_dequant_scale(float(amax_a), float(amax_b)))


# ---- integer GEMM ------------------------------------------------------------


def gemm_i16_exact(qa: np.ndarray, qb: np.ndarray) -> np.ndarray:
    """acc = qa @ qb in int64 via the exact float64 shortcut (K < 2^23)."""
    assert qa.shape[-1] == qb.shape[-2] and qa.shape[-1] < (1 << 23)
    return np.matmul(qa.astype(np.float64), qb.astype(np.float64)).astype(np.int64)


def gemm_i16_strided(qa: np.ndarray, qb: np.ndarray) -> np.ndarray:
    """acc = qa @ qb with the C int64 loop on the arrays' own strides (no
    copies; host threads over output elements).  Used for skinny products
    (few rows), where converting the big operand to float64 would dominate."""
    assert qa.dtype == np.int16 and qb.dtype == np.int16 and qa.ndim == 2 and qb.ndim == 2
    M, K = qa.shape
    K2, N = qb.shape
    assert K == K2
    acc = np.empty((M, N), dtype=np.int64)
    sa = [st // 2 for st in qa.strides]
    sb = [st // 2 for st in qb.strides]
    lib().tko_gemm_i16(M, N, K, _ptr(qa), sa[0], sa[1], _ptr(qb), sb[0], sb[1], _ptr(acc))
    return acc


def gemm_i16_scalar(qa: np.ndarray, qb: np.ndarray) -> np.ndarray:
    """acc = qa @ qb with the C int64 loop (slow; used to pin the shortcut)."""
    qa = np.ascontiguousarray(qa, dtype=np.int16)
    qb = np.ascontiguousarray(qb, dtype=np.int16)
    M, K = qa.shape
    K2, N = qb.shape
    assert K == K2
    acc = np.empty((M, N), dtype=np.int64)
    lib().tko_gemm_i16(M, N, K, _ptr(qa), K, 1, _ptr(qb), N, 1, _ptr(acc))
    return acc


def epilogue(acc: np.ndarray, amax_a, amax_b, dtype, alpha=1.0, bias=None,
             addend=None, beta=0.0, act=ACT_NONE) -> np.ndarray:
    """Apply the dequant/bias/addend/activation contract to an int64 tile."""
    acc = np.ascontiguousarray(acc, dtype=np.int64)
    M, N = acc.shape
    dt = F16 if np.dtype(dtype) == np.float16 else F32
    out = np.empty((M, N), dtype=np.float16 if dt == F16 else np.float32)
    bias_p = None
    if bias is not None:
        bias = np.ascontiguousarray(bias, dtype=out.dtype).reshape(-1)
        assert bias.size == N
        bias_p = _ptr(bias)
    add_p, sm, sn = None, 0, 0
    if addend is not None and beta != 0.0:
        addend = np.ascontiguousarray(np.broadcast_to(
            np.asarray(addend, dtype=out.dtype), (M, N)))
        add_p, sm, sn = _ptr(addend), N, 1
    lib().tko_epilogue(dt, M, N, _ptr(acc), float(amax_a), float(amax_b), float(alpha),
                       bias_p, add_p, sm, sn, float(beta), int(act), _ptr(out), N)
    return out


# ---- operator-level compositions ---------------------------------------------


def fc(x: np.ndarray, w: np.ndarray, w_trans: bool, bias=None, alpha=1.0,
       addend=None, beta=0.0, act=ACT_NONE, scalar=False):
    """Quantised fc: y = epilogue(q16(x) @ op(q16(w))).

    x is [M,K]; w is [N,K] when w_trans (linear) and [K,N] otherwise (mm).
    Returns (y, acc, amax_x, amax_w).
    """
    ax, aw = amax(x), amax(w)
    qx, qw = quant(x, ax), quant(w, aw)
    qb = qw.T if w_trans else qw
    if scalar:
        acc = gemm_i16_scalar(qx, qb)
    elif qx.shape[0] <= 64:
        acc = gemm_i16_strided(qx, qb)
    else:
        acc = gemm_i16_exact(qx, qb)
    y = epilogue(acc, ax, aw, x.dtype, alpha, bias, addend, beta, act)
    return y, acc, ax, aw


def linear(x, w, bias=None, act=ACT_NONE):
    return fc(x, w, True, bias=bias, act=act)[0]


def mm(a, b):
    return fc(a, b, False)[0]


def addmm(self_, a, b, beta=1.0, alpha=1.0):
    return fc(a, b, False, alpha=alpha, addend=self_, beta=beta)[0]


def bmm(a: np.ndarray, b: np.ndarray, alpha=1.0, addend=None, beta=0.0) -> np.ndarray:
    """Per-slice quantised batched matmul: a [B,M,K] @ b [B,K,N]."""
    B = a.shape[0]
    outs = []
    for i in range(B):
        add_i = None if addend is None else np.broadcast_to(addend, (B,) + addend.shape[-2:])[i]
        outs.append(fc(a[i], b[i], False, alpha=alpha, addend=add_i, beta=beta)[0])
    return np.stack(outs)


def baddbmm(self_, a, b, beta=1.0, alpha=1.0):
    return bmm(a, b, alpha=alpha, addend=self_, beta=beta)


def conv_out_hw(H, W, KH, KW, stride, pad, dil):
    OH = (H + 2 * pad[0] - dil[0] * (KH - 1) - 1) // stride[0] + 1
    OW = (W + 2 * pad[1] - dil[1] * (KW - 1) - 1) // stride[1] + 1
    return OH, OW


def conv2d_acc(qx: np.ndarray, qw: np.ndarray, stride, pad, dil, groups, scalar=False):
    """int64 conv accumulators of quantised NCHW input and OIHW weight."""
    NB, C, H, W = qx.shape
    F, cg, KH, KW = qw.shape
    OH, OW = conv_out_hw(H, W, KH, KW, stride, pad, dil)
    if scalar:
        acc = np.empty((NB, F, OH, OW), dtype=np.int64)
        lib().tko_conv2d_i16(NB, C, H, W, F, KH, KW, stride[0], stride[1], pad[0], pad[1],
                             dil[0], dil[1], groups, _ptr(np.ascontiguousarray(qx)),
                             _ptr(np.ascontiguousarray(qw)), _ptr(acc))
        return acc
    xp = np.zeros((NB, C, H + 2 * pad[0], W + 2 * pad[1]), dtype=np.float64)
    xp[:, :, pad[0]:pad[0] + H, pad[1]:pad[1] + W] = qx
    fg = F // groups
    acc = np.zeros((NB, F, OH, OW), dtype=np.float64)
    for g in range(groups):
        wg = qw[g * fg:(g + 1) * fg].astype(np.float64).reshape(fg, cg * KH * KW)
        cols = np.empty((NB, cg, KH, KW, OH, OW), dtype=np.float64)
        for r in range(KH):
            for s in range(KW):
                h0, w0 = r * dil[0], s * dil[1]
                cols[:, :, r, s] = xp[:, g * cg:(g + 1) * cg,
                                      h0:h0 + stride[0] * (OH - 1) + 1:stride[0],
                                      w0:w0 + stride[1] * (OW - 1) + 1:stride[1]]
        cols = cols.reshape(NB, cg * KH * KW, OH * OW)
        acc[:, g * fg:(g + 1) * fg] = np.einsum("fk,bkp->bfp", wg, cols).reshape(NB, fg, OH, OW)
    return acc.astype(np.int64)


def conv2d(x: np.ndarray, w: np.ndarray, bias=None, stride=(1, 1), pad=(0, 0), dil=(1, 1),
           groups=1, scalar=False) -> np.ndarray:
    ax, aw = amax(x), amax(w)
    acc = conv2d_acc(quant(x, ax), quant(w, aw), stride, pad, dil, groups, scalar)
    NB, F, OH, OW = acc.shape
    # bias broadcasts over [N, F, OH, OW] along F: flatten so F*OH*OW is one row
    # per image and expand the bias to match (csrc/ops.cpp:271-283).
    flat = acc.transpose(0, 1, 2, 3).reshape(NB * F, OH * OW)
    add = None
    if bias is not None:
        add = np.repeat(np.asarray(bias, dtype=x.dtype).reshape(1, F), NB, 0).reshape(NB * F, 1)
        add = np.broadcast_to(add, flat.shape)
    y = epilogue(flat, ax, aw, x.dtype, addend=add, beta=1.0 if add is not None else 0.0)
    return y.reshape(NB, F, OH, OW)


def convnd_acc(qx: np.ndarray, qw: np.ndarray, stride, pad, dil, groups) -> np.ndarray:
    """int64 accumulators of a quantised convolution with any number of
    spatial axes (NC... input, OI... weight): the conv2d gather above per
    kernel tap, float64 sums of integers below 2^53 (exact)."""
    import itertools
    k = qx.ndim - 2
    NB, C = qx.shape[:2]
    F, cg = qw.shape[:2]
    ks = qw.shape[2:]
    outs = [(qx.shape[2 + i] + 2 * pad[i] - dil[i] * (ks[i] - 1) - 1) // stride[i] + 1 for i in range(k)]
    xp = np.zeros((NB, C) + tuple(qx.shape[2 + i] + 2 * pad[i] for i in range(k)), dtype=np.float64)
    xp[(slice(None), slice(None)) + tuple(slice(pad[i], pad[i] + qx.shape[2 + i]) for i in range(k))] = qx
    fg = F // groups
    acc = np.zeros((NB, F) + tuple(outs), dtype=np.float64)
    for g in range(groups):
        xs = xp[:, g * cg:(g + 1) * cg]
        for tap in itertools.product(*[range(t) for t in ks]):
            sl = tuple(slice(tap[i] * dil[i], tap[i] * dil[i] + stride[i] * (outs[i] - 1) + 1, stride[i])
                       for i in range(k))
            win = xs[(slice(None), slice(None)) + sl]                      # [NB, cg, O...]
            wt = qw[(slice(g * fg, (g + 1) * fg), slice(None)) + tap].astype(np.float64)  # [fg, cg]
            acc[:, g * fg:(g + 1) * fg] += np.einsum("fc,nc...->nf...", wt, win)
    return acc.astype(np.int64)


def _conv_epilogue(acc, x, ax, aw, bias):
    NB, F = acc.shape[:2]
    flat = acc.reshape(NB * F, -1)
    add = None
    if bias is not None:
        add = np.repeat(np.asarray(bias, dtype=x.dtype).reshape(1, F), NB, 0).reshape(NB * F, 1)
        add = np.broadcast_to(add, flat.shape)
    y = epilogue(flat, ax, aw, x.dtype, addend=add, beta=1.0 if add is not None else 0.0)
    return y.reshape(acc.shape)


def conv3d(x: np.ndarray, w: np.ndarray, bias=None, stride=(1, 1, 1), pad=(0, 0, 0), dil=(1, 1, 1),
           groups=1) -> np.ndarray:
    """conv3d with the conv2d contract (csrc/ops_nn_extra.cpp:88-121: xdnn
    conv3d with TGEMM = int16 and null maxptrs, then a separately rounded bias
    add)."""
    ax, aw = amax(x), amax(w)
    acc = convnd_acc(quant(x, ax), quant(w, aw), stride, pad, dil, groups)
    return _conv_epilogue(acc, x, ax, aw, bias)


def conv1d(x: np.ndarray, w: np.ndarray, bias=None, stride=1, pad=0, dil=1, groups=1) -> np.ndarray:
    """conv1d as conv2d on [N, C, 1, L] (csrc/ops_nn_extra.cpp:70-86)."""
    y = conv2d(x[:, :, None, :], w[:, :, None, :], bias, (1, stride), (0, pad), (1, dil), groups)
    return y[:, :, 0, :]


def conv_transpose_acc(qx: np.ndarray, qw: np.ndarray, stride, pad, out_pad, dil, groups) -> np.ndarray:
    """int64 accumulators of a transposed convolution by its definition: input
    element i scatters x[i] * w[tap] to output position i*stride - pad +
    tap*dil (weight [C_in, C_out/groups, K...])."""
    import itertools
    k = qx.ndim - 2
    NB, Cin = qx.shape[:2]
    cog = qw.shape[1]
    ks = qw.shape[2:]
    cig = Cin // groups
    ins = qx.shape[2:]
    outs = [(ins[i] - 1) * stride[i] - 2 * pad[i] + dil[i] * (ks[i] - 1) + 1 + out_pad[i] for i in range(k)]
    full = [(ins[i] - 1) * stride[i] + dil[i] * (ks[i] - 1) + 1 + out_pad[i] for i in range(k)]
    acc = np.zeros((NB, cog * groups) + tuple(full), dtype=np.float64)
    for g in range(groups):
        xs = qx[:, g * cig:(g + 1) * cig].astype(np.float64)
        for tap in itertools.product(*[range(t) for t in ks]):
            wt = qw[(slice(g * cig, (g + 1) * cig), slice(None)) + tap].astype(np.float64)  # [cig, cog]
            contrib = np.einsum("nc...,co->no...", xs, wt)
            sl = tuple(slice(tap[i] * dil[i], tap[i] * dil[i] + stride[i] * (ins[i] - 1) + 1, stride[i])
                       for i in range(k))
            acc[(slice(None), slice(g * cog, (g + 1) * cog)) + sl] += contrib
    crop = tuple(slice(pad[i], pad[i] + outs[i]) for i in range(k))
    return acc[(slice(None), slice(None)) + crop].astype(np.int64)


def conv_transpose(x: np.ndarray, w: np.ndarray, bias=None, stride=None, pad=None, out_pad=None, dil=None,
                   groups=1) -> np.ndarray:
    """Transposed convolution (csrc/ops_nn_extra.cpp:123-159: xdnn
    conv2d_transpose with TGEMM = int16, null maxptrs, then the bias add) with
    the conv2d contract: one scale per tensor, exact sum, one rounding."""
    k = x.ndim - 2
    stride = stride or (1,) * k
    pad = pad or (0,) * k
    out_pad = out_pad or (0,) * k
    dil = dil or (1,) * k
    ax, aw = amax(x), amax(w)
    acc = conv_transpose_acc(quant(x, ax), quant(w, aw), stride, pad, out_pad, dil, groups)
    return _conv_epilogue(acc, x, ax, aw, bias)


def conv_weight_grad_acc(qx: np.ndarray, qg: np.ndarray, w_shape, stride, pad, dil, groups) -> np.ndarray:
    """int64 accumulators of the weight gradient of a convolution with any
    number of spatial axes: acc[f][c][tap] = sum over images and output
    positions o of qg[n][f][o] * qx[n][g*cg + c][o*stride + tap*dil - pad]
    (zero outside the input), per kernel tap as float64 sums of integers below
    2^53 (exact)."""
    import itertools
    k = qx.ndim - 2
    NB, C = qx.shape[:2]
    F, cg = w_shape[:2]
    ks = tuple(w_shape[2:])
    outs = qg.shape[2:]
    xp = np.zeros((NB, C) + tuple(qx.shape[2 + i] + 2 * pad[i] for i in range(k)), dtype=np.float64)
    xp[(slice(None), slice(None)) + tuple(slice(pad[i], pad[i] + qx.shape[2 + i]) for i in range(k))] = qx
    fg = F // groups
    acc = np.zeros((F, cg) + ks, dtype=np.float64)
    gd = qg.astype(np.float64)
    for g in range(groups):
        xs = xp[:, g * cg:(g + 1) * cg]
        gs = gd[:, g * fg:(g + 1) * fg]
        for tap in itertools.product(*[range(t) for t in ks]):
            sl = tuple(slice(tap[i] * dil[i], tap[i] * dil[i] + stride[i] * (outs[i] - 1) + 1, stride[i])
                       for i in range(k))
            win = xs[(slice(None), slice(None)) + sl]                      # [NB, cg, O...]
            acc[(slice(g * fg, (g + 1) * fg), slice(None)) + tap] = np.einsum(
                "nfp,ncp->fc", gs.reshape(NB, fg, -1), win.reshape(NB, cg, -1))
    return acc.astype(np.int64)


def conv_weight_grad(x: np.ndarray, grad_out: np.ndarray, w_shape, stride, pad, dil,
                     groups=1) -> np.ndarray:
    """Weight gradient of the quantised convolution: the weight half of the
    reference's conv2d_grad (csrc/autograd.cpp:621-682) under the forward's
    contract -- x and grad_out each quantised with one per-tensor scale, the
    exact integer sum over every image and output pixel, one dequantising
    rounding to T."""
    ax, ag = amax(x), amax(grad_out)
    acc = conv_weight_grad_acc(quant(x, ax), quant(grad_out, ag), w_shape, stride, pad, dil, groups)
    y = epilogue(acc.reshape(acc.shape[0], -1), ax, ag, x.dtype)
    return y.reshape(acc.shape)


# ---- floating-point ops: the textbook formulas in float64 (C, libm) -----------
# The device evaluates the same formulas in binary32; tests compare at the
# bounds they state (one or two binary16 ulps plus the binary32 error of the
# libm-class functions the device calls).


def _out_like(x, dtype=None):
    return np.empty(x.shape, dtype=x.dtype if dtype is None else dtype)


def act(x: np.ndarray, kind: str) -> np.ndarray:
    """T(act(x)) elementwise: relu, gelu (erf), gelu_tanh, silu."""
    x = np.ascontiguousarray(x)
    out = _out_like(x)
    lib().tko_act(_ptr(x), _dt(x), x.size, ACT_CODES[kind], _ptr(out))
    return out


def gelu(x: np.ndarray, approximate: str = "none") -> np.ndarray:
    return act(x, "gelu_tanh" if approximate == "tanh" else "gelu")


def silu(x: np.ndarray) -> np.ndarray:
    return act(x, "silu")


def silu_mul(gate: np.ndarray, up: np.ndarray) -> np.ndarray:
    """T(T(silu(gate)) * up): swish stored as T, then mul."""
    gate = np.ascontiguousarray(gate)
    up = np.ascontiguousarray(up, dtype=gate.dtype)
    assert gate.shape == up.shape
    out = _out_like(gate)
    lib().tko_silu_mul(_ptr(gate), _ptr(up), _dt(gate), gate.size, _ptr(out))
    return out


def softmax(x: np.ndarray, axis=-1, out_dtype=None) -> np.ndarray:
    """Softmax along the last axis (axis must be -1 or the last)."""
    assert axis in (-1, x.ndim - 1)
    x = np.ascontiguousarray(x)
    od = np.dtype(out_dtype) if out_dtype is not None else x.dtype
    out = np.empty(x.shape, dtype=od)
    cols = x.shape[-1]
    lib().tko_softmax(_ptr(x), _dt(x), x.size // max(cols, 1), cols, F16 if od == np.float16 else F32, _ptr(out))
    return out


def layer_norm(x: np.ndarray, gamma, beta, eps, return_stats=False):
    x = np.ascontiguousarray(x)
    cols = x.shape[-1]
    rows = x.size // max(cols, 1)
    wdt = x.dtype
    g = None if gamma is None else np.ascontiguousarray(gamma)
    b = None if beta is None else np.ascontiguousarray(beta)
    if g is not None:
        wdt = g.dtype
    if b is not None:
        b = b.astype(wdt)
    out = _out_like(x)
    mean = np.empty(rows, dtype=np.float32)
    rstd = np.empty(rows, dtype=np.float32)
    lib().tko_layer_norm(_ptr(x), _dt(x), rows, cols, None if g is None else _ptr(g),
                         None if b is None else _ptr(b), F16 if wdt == np.float16 else F32, float(eps),
                         _ptr(out), _ptr(mean), _ptr(rstd))
    return (out, mean, rstd) if return_stats else out


def round_t(v: np.ndarray, dtype) -> np.ndarray:
    """Round float64 values to T (nearest-even) through the C helper for fp16."""
    v = np.asarray(v, dtype=np.float64)
    if np.dtype(dtype) == np.float32:
        return v.astype(np.float32)
    L = lib()
    flat = v.reshape(-1)
    bits = np.fromiter((L.tko_f64_to_f16(float(t)) for t in flat), dtype=np.uint16,
                       count=flat.size)
    return bits.view(np.float16).reshape(v.shape)


def sdpa(q: np.ndarray, k: np.ndarray, v: np.ndarray, mask=None, scale=None, causal=False,
         return_p=False):
    """The reference's SDPA composition over [BH, L, E] slices.

    Steps (torch_kunlun/kunlun/attention.py:85-106): per-slice quantised bmm
    q @ k^T, multiply by the scale (rounded to T), add the additive mask
    (rounded to T), softmax along the last axis, per-slice quantised bmm with v.
    The softmax step is computed in float64 here, so results are compared with
    a tolerance.
    """
    BH, L, E = q.shape
    kt = np.ascontiguousarray(np.swapaxes(k, 1, 2))
    s = bmm(q, kt)
    factor = (1.0 / np.sqrt(E)) if scale is None else float(scale)
    if factor != 1.0:
        s = round_t(s.astype(np.float32) * np.float32(factor), q.dtype)
    if causal:
        # -1e4 strictly above the diagonal, added as its own rounded step
        # (torch_kunlun/kunlun/attention.py:89-95)
        S = k.shape[1]
        tri = np.triu(np.full((L, S), -1.0e4, dtype=np.float32), 1)
        s = round_t(s.astype(np.float32) + tri, q.dtype)
    if mask is not None:
        s = round_t(s.astype(np.float32) + np.broadcast_to(mask, s.shape).astype(np.float32),
                    q.dtype)
    p = softmax(s, -1)
    out = bmm(p, v)
    return (out, p) if return_p else out
