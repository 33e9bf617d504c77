"""conv1d, conv3d and the transposed convolutions on the kunlun device, with
the quantised-conv contract (one max-abs int16 scale per whole input and per
whole weight, exact integer MAC, T(acc * s), bias added after rounding):

- conv1d is conv2d on [N, C, 1, L] (reference csrc/ops_nn_extra.cpp:70-86);
- conv3d (csrc/ops_nn_extra.cpp:88-121) runs on the implicit-GEMM core for
  groups 1 / stride 1 (5-D TMA boxes over N·D·H·W limb rows) and on the
  patch-gather GEMM otherwise;
- conv_transpose{1,2,3}d (csrc/ops_nn_extra.cpp:123-159) is one quantised
  correlation of the zero-inserted input with the flipped weight, checked
  against the oracle's scatter definition of the transposed convolution.
All forward results are bit-identical to the oracle.  Backward: the
reference's own autograd tests (tests/test_nn_extra.py:177-244) at their
tolerances, and bit-exact gradients where each is one quantised op."""
import math

import numpy as np
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

torch_kunlun = pytest.importorskip("torch_kunlun")
kunlun = torch_kunlun.kunlun
from oracle import oracle as O  # noqa: E402
from tests._qgemm_helpers import assert_bits_equal  # noqa: E402

DEV = "kunlun"


def rnd(shape, seed, scale=1.0, dtype=torch.float16):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(shape, generator=g) * scale).to(dtype)


def _np(t):
    return None if t is None else t.numpy()


def _dev(t):
    return None if t is None else t.to(DEV)


C1_CASES = [
    # N, C, L, F, k, stride, pad, dil, groups, bias
    (2, 3, 8, 4, 3, 1, 1, 1, 1, True),
    (2, 64, 100, 64, 5, 1, 2, 1, 1, False),
    (3, 6, 31, 9, 3, 2, 1, 1, 3, True),
    (1, 8, 40, 16, 3, 1, 2, 2, 1, False),
]


@pytest.mark.parametrize("case", C1_CASES)
def test_conv1d_bit_exact(case):
    N, C, L, Fo, k, s, p, d, g, has_b = case
    x = rnd((N, C, L), 50)
    w = rnd((Fo, C // g, k), 51, 0.3)
    b = rnd((Fo,), 52, 0.05) if has_b else None
    y = F.conv1d(x.to(DEV), w.to(DEV), _dev(b), stride=s, padding=p, dilation=d, groups=g).cpu()
    want = O.conv1d(x.numpy(), w.numpy(), _np(b), s, p, d, g)
    assert y.shape == want.shape
    assert_bits_equal(y.numpy(), want, f"conv1d {case}")


C3_CASES = [
    # N, C, D, H, W, F, k, stride, pad, dil, groups, bias, dtype
    (1, 2, 4, 5, 5, 3, (2, 2, 2), 1, 1, 1, 1, True, torch.float16),    # the reference's test shape
    (2, 70, 5, 9, 10, 40, (3, 3, 3), 1, 1, 1, 1, False, torch.float16),  # implicit, ragged channel group
    (1, 32, 4, 12, 12, 150, (3, 3, 3), 1, (1, 1, 1), 1, 1, True, torch.float16),  # two filter tiles
    (2, 16, 6, 7, 8, 24, (3, 1, 3), 1, (2, 0, 1), (2, 1, 1), 1, False, torch.float16),  # dilation in depth
    (1, 8, 5, 6, 7, 12, (1, 1, 1), 1, 0, 1, 1, True, torch.float32),   # pointwise, fp32
    (2, 6, 7, 8, 9, 10, (3, 3, 3), 2, 1, 1, 2, True, torch.float16),   # strided, grouped: patch-gather GEMM
    (1, 4, 5, 5, 6, 8, (2, 3, 3), (2, 1, 2), (0, 1, 1), 1, 1, False, torch.float32),
]


def _t3(v):
    return tuple(v) if isinstance(v, tuple) else (v, v, v)


@pytest.mark.parametrize("case", C3_CASES)
def test_conv3d_bit_exact(case):
    N, C, D, H, W, Fo, k, s, p, d, g, has_b, dt = case
    x = torch.relu(rnd((N, C, D, H, W), 53, dtype=dt))
    w = rnd((Fo, C // g) + k, 54, math.sqrt(2.0 / (C // g * np.prod(k))), dtype=dt)
    b = rnd((Fo,), 55, 0.05, dtype=dt) if has_b else None
    y = F.conv3d(x.to(DEV), w.to(DEV), _dev(b), stride=s, padding=p, dilation=d, groups=g).cpu()
    want = O.conv3d(x.numpy(), w.numpy(), _np(b), _t3(s), _t3(p), _t3(d), g)
    assert y.shape == want.shape
    assert_bits_equal(y.numpy(), want, f"conv3d {case}")


CT_CASES = [
    # shape of x, weight [Cin, Cout/g, K...], stride, pad, output_padding, dil, groups, bias
    ((1, 3, 5, 5), (3, 2, 3, 3), 2, 1, 0, 1, 1, True),             # the reference's test shape
    ((2, 8, 7, 6), (8, 5, 4, 4), 2, 1, 1, 1, 1, False),
    ((2, 6, 5, 5), (6, 4, 3, 3), (2, 3), (0, 1), (1, 2), (1, 2), 2, True),
    ((2, 4, 9, 9), (4, 6, 3, 3), 1, 3, 0, 1, 1, False),             # padding wider than the kernel: a crop
    ((2, 6, 17), (6, 4, 5), 3, 2, 2, 1, 1, True),                    # conv_transpose1d
    ((1, 4, 3, 4, 5), (4, 3, 2, 3, 3), 2, 1, (1, 0, 1), 1, 1, True),  # conv_transpose3d
]


def _tk(v, k):
    return tuple(v) if isinstance(v, tuple) else (v,) * k


@pytest.mark.parametrize("case", CT_CASES)
def test_conv_transpose_bit_exact(case):
    xs, ws, s, p, op, d, g, has_b = case
    k = len(xs) - 2
    x = rnd(xs, 56)
    w = rnd(ws, 57, 0.3)
    b = rnd((ws[1] * g,), 58, 0.05) if has_b else None
    fn = {1: F.conv_transpose1d, 2: F.conv_transpose2d, 3: F.conv_transpose3d}[k]
    y = fn(x.to(DEV), w.to(DEV), _dev(b), stride=s, padding=p, output_padding=op, groups=g, dilation=d).cpu()
    want = O.conv_transpose(x.numpy(), w.numpy(), _np(b), _tk(s, k), _tk(p, k), _tk(op, k), _tk(d, k), g)
    assert y.shape == want.shape, (y.shape, want.shape)
    assert_bits_equal(y.numpy(), want, f"conv_transpose {case}")


def _ones(t):
    out = torch.empty_like(t)
    out.fill_(1.0)
    return out


def _grads(fn, tensors, dev):
    ts = [t.clone().to(dev).requires_grad_() for t in tensors]
    y = fn(*ts)
    y.backward(_ones(y))
    if dev == DEV:
        kunlun.synchronize()
    return y.detach().cpu(), [t.grad.cpu() for t in ts]


@pytest.mark.parametrize("which", ["conv1d", "conv3d", "conv_transpose2d"])
def test_reference_autograd_cases(which):
    """tests/test_nn_extra.py:177-244 of the reference, same shapes and
    tolerances."""
    if which == "conv1d":
        ts = [torch.randn(2, 3, 8, dtype=torch.float16), torch.randn(4, 3, 3, dtype=torch.float16),
              torch.randn(4, dtype=torch.float16)]
        fn = lambda x, w, b: F.conv1d(x, w, b, padding=1)  # noqa: E731
    elif which == "conv3d":
        ts = [torch.randn(1, 2, 4, 5, 5, dtype=torch.float16), torch.randn(3, 2, 2, 2, 2, dtype=torch.float16),
              torch.randn(3, dtype=torch.float16)]
        fn = lambda x, w, b: F.conv3d(x, w, b, padding=1)  # noqa: E731
    else:
        ts = [torch.randn(1, 3, 5, 5, dtype=torch.float16), torch.randn(3, 2, 3, 3, dtype=torch.float16),
              torch.randn(2, dtype=torch.float16)]
        fn = lambda x, w, b: F.conv_transpose2d(x, w, b, stride=2, padding=1)  # noqa: E731
    yr, gr = _grads(fn, ts, "cpu")
    yk, gk = _grads(fn, ts, DEV)
    assert torch.allclose(yk, yr, atol=5e-2, rtol=5e-2)
    for a, b in zip(gk, gr):
        assert torch.allclose(a, b, atol=5e-2, rtol=5e-2)


def test_conv3d_backward_is_quantised():
    """grad_input of conv3d is the transposed convolution of grad_output
    (bit-exact against the oracle's scatter definition); grad_weight is the
    quantised correlation of input and grad_output."""
    N, C, D, H, Fo, k, s, p = 2, 4, 6, 7, 5, 3, 2, 1
    x = rnd((N, C, D, H, H), 60)
    w = rnd((Fo, C, k, k, k), 61, 0.2)
    xk = x.to(DEV).requires_grad_()
    wk = w.to(DEV).requires_grad_()
    y = F.conv3d(xk, wk, stride=s, padding=p)
    gy = rnd(tuple(y.shape), 62)
    y.backward(gy.to(DEV))
    e = [(n + 2 * p - (k - 1) - 1) - (o - 1) * s for n, o in zip((D, H, H), y.shape[2:])]
    want_gi = O.conv_transpose(gy.numpy(), w.numpy(), None, (s,) * 3, (p,) * 3, tuple(e), (1,) * 3, 1)
    assert_bits_equal(xk.grad.cpu().numpy(), want_gi, "conv3d grad_input")
    xt = np.ascontiguousarray(np.swapaxes(x.numpy(), 0, 1)).astype(np.float32)
    gt = np.ascontiguousarray(np.swapaxes(gy.numpy(), 0, 1)).astype(np.float32)
    gw = O.conv3d(xt, gt, None, (1,) * 3, (p,) * 3, (s,) * 3, 1)[:, :, :k, :k, :k]
    want_gw = np.ascontiguousarray(np.swapaxes(gw, 0, 1)).astype(np.float16)
    assert_bits_equal(wk.grad.cpu().numpy(), want_gw, "conv3d grad_weight")


def test_conv_transpose2d_backward_is_quantised():
    """grad_input of a transposed convolution is the forward convolution of
    grad_output with the same weight, bit-exact."""
    x = rnd((2, 6, 5, 6), 63)
    w = rnd((6, 4, 3, 3), 64, 0.3)
    xk = x.to(DEV).requires_grad_()
    wk = w.to(DEV).requires_grad_()
    y = F.conv_transpose2d(xk, wk, stride=2, padding=1, output_padding=1, groups=2)
    gy = rnd(tuple(y.shape), 65)
    y.backward(gy.to(DEV))
    want = O.conv2d(gy.numpy(), w.numpy(), None, (2, 2), (1, 1), (1, 1), 2)
    assert_bits_equal(xk.grad.cpu().numpy(), want, "conv_transpose2d grad_input")
    yr = F.conv_transpose2d(x.float().requires_grad_(), w.float().requires_grad_(), stride=2, padding=1,
                            output_padding=1, groups=2)
    wr = w.float().requires_grad_()
    yr = F.conv_transpose2d(x.float(), wr, stride=2, padding=1, output_padding=1, groups=2)
    yr.backward(gy.float())
    scale = max(1.0, wr.grad.abs().max().item())
    assert (wk.grad.cpu().float() - wr.grad).abs().max().item() <= 2e-2 * scale
