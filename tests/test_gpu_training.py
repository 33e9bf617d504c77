"""Backward through the quantised dense ops (the next row of the hot path):
torch's autograd formulas for mm / addmm / linear / bmm run their gradient
products on the same int16-quantised GEMM, so the input and weight gradients
are bit-exact against the oracle's quantised product of the same operands;
the bias gradient is a deterministic fp32 sum.  Plus the reference's own
training test (tests/test_training.py:17-39: MLP + ReLU + MSE + SGD, loss
must decrease) and the ops it needs (threshold_backward, sum, mse_loss)."""
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


def test_linear_backward_uses_the_quantised_gemm():
    x, w, b = rnd((96, 64), 1), rnd((48, 64), 2, 0.05), rnd((48,), 3, 0.05)
    gy = rnd((96, 48), 4)
    xd = x.to(DEV).requires_grad_()
    wd = w.to(DEV).requires_grad_()
    bd = b.to(DEV).requires_grad_()
    y = F.linear(xd, wd, bd)
    y.backward(gy.to(DEV))
    # dX = dY @ W and dW = dY^T @ X, each one quantised product (per-tensor scales)
    assert_bits_equal(xd.grad.cpu().numpy(), O.mm(gy.numpy(), w.numpy()), "grad_input")
    assert_bits_equal(wd.grad.cpu().numpy(),
                      O.mm(np.ascontiguousarray(gy.numpy().T), x.numpy()), "grad_weight")
    want_b = gy.double().sum(0)
    assert torch.allclose(bd.grad.cpu().double(), want_b, atol=2e-2, rtol=2e-3)


def test_mm_and_bmm_backward():
    a, b = rnd((40, 72), 5), rnd((72, 24), 6, 0.1)
    ad, bd = a.to(DEV).requires_grad_(), b.to(DEV).requires_grad_()
    g = rnd((40, 24), 7)
    (ad @ bd).backward(g.to(DEV))
    assert_bits_equal(ad.grad.cpu().numpy(), O.mm(g.numpy(), np.ascontiguousarray(b.numpy().T)), "mm dA")
    assert_bits_equal(bd.grad.cpu().numpy(), O.mm(np.ascontiguousarray(a.numpy().T), g.numpy()), "mm dB")
    A, B = rnd((3, 16, 32), 8), rnd((3, 32, 8), 9, 0.2)
    Ad, Bd = A.to(DEV).requires_grad_(), B.to(DEV).requires_grad_()
    G = rnd((3, 16, 8), 10)
    torch.bmm(Ad, Bd).backward(G.to(DEV))
    want = O.bmm(G.numpy(), np.ascontiguousarray(np.swapaxes(B.numpy(), 1, 2)))
    assert_bits_equal(Ad.grad.cpu().numpy(), want, "bmm dA")


@pytest.mark.parametrize("dims,keepdim", [((0,), False), ((1,), True), ((0, 2), False), (None, False),
                                          ((-1,), False), ((1, 2), True)])
@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_sum_over_dims(dims, keepdim, dtype):
    x = rnd((5, 7, 33), 11, dtype=dtype)
    xd = x.to(DEV)
    got = (xd.sum() if dims is None else xd.sum(dim=dims, keepdim=keepdim)).cpu()
    want = x.double().sum() if dims is None else x.double().sum(dim=dims, keepdim=keepdim)
    assert got.shape == want.shape and got.dtype == dtype
    tol = 5e-3 if dtype == torch.float16 else 1e-5
    assert torch.allclose(got.double(), want, atol=tol * 10, rtol=tol)
    f32 = xd.sum(dim=0, dtype=torch.float32).cpu() if dtype == torch.float16 else None
    if f32 is not None:
        assert f32.dtype == torch.float32
        assert torch.allclose(f32.double(), x.double().sum(0), atol=1e-4, rtol=1e-5)


def test_relu_and_mse_backward():
    x, t = rnd((32, 16), 12), rnd((32, 16), 13)
    xd = x.to(DEV).requires_grad_()
    loss = F.mse_loss(torch.relu(xd), t.to(DEV))
    loss.backward()
    xr = x.float().requires_grad_()
    lr = F.mse_loss(torch.relu(xr), t.float())
    lr.backward()
    assert abs(loss.cpu().item() - lr.item()) < 2e-3 * max(1.0, lr.item())
    assert torch.allclose(xd.grad.cpu().float(), xr.grad, atol=1e-4, rtol=1e-2)
    for red in ("sum", "none"):
        got = F.mse_loss(xd.detach(), t.to(DEV), reduction=red).cpu().float()
        want = F.mse_loss(x.float(), t.float(), reduction=red)
        assert torch.allclose(got, want, atol=5e-2, rtol=3e-3)


def test_mlp_mse_sgd_training():
    """The reference's tests/test_training.py:17-39 on the kunlun device."""
    torch.manual_seed(0)
    model = torch.nn.Sequential(
        torch.nn.Linear(8, 16),
        torch.nn.ReLU(),
        torch.nn.Linear(16, 1),
    ).half().to(DEV)
    opt = torch.optim.SGD(model.parameters(), lr=0.05, foreach=False)
    loss_fn = torch.nn.MSELoss()
    x = torch.randn(32, 8, dtype=torch.float16).to(DEV)
    target = torch.randn(32, 1, dtype=torch.float16).to(DEV)
    losses = []
    for _ in range(20):
        opt.zero_grad()
        loss = loss_fn(model(x), target)
        loss.backward()
        opt.step()
        losses.append(float(loss.detach().cpu().item()))
    assert losses[-1] < losses[0], f"loss did not decrease: {losses[0]} -> {losses[-1]}"


def _ones_like(x):
    out = torch.empty_like(x)
    out.fill_(1.0)
    return out


def test_conv2d_backward_reference_case():
    """The reference's tests/test_autograd_nn.py:20-40."""
    x = torch.randn(1, 2, 5, 5, dtype=torch.float16)
    w = torch.randn(3, 2, 3, 3, dtype=torch.float16)
    b = torch.randn(3, dtype=torch.float16)
    xr, wr, br = x.clone().requires_grad_(), w.clone().requires_grad_(), b.clone().requires_grad_()
    ref = F.conv2d(xr, wr, br, padding=1)
    ref.backward(_ones_like(ref))
    xk = x.clone().to(DEV).requires_grad_()
    wk = w.clone().to(DEV).requires_grad_()
    bk = b.clone().to(DEV).requires_grad_()
    out = F.conv2d(xk, wk, bk, padding=1)
    out.backward(_ones_like(out))
    kunlun.synchronize()
    assert torch.allclose(out.cpu(), ref.detach(), atol=5e-2, rtol=5e-2)
    assert torch.allclose(xk.grad.cpu(), xr.grad, atol=5e-2, rtol=5e-2)
    assert torch.allclose(wk.grad.cpu(), wr.grad, atol=5e-2, rtol=5e-2)
    assert torch.allclose(bk.grad.cpu(), br.grad, atol=5e-2, rtol=5e-2)


def test_conv2d_backward_is_quantised_conv():
    """grad_input and grad_weight are themselves quantised convolutions of the
    contract: bit-exact against the oracle on the same operands."""
    N, C, H, F_, k, pad = 2, 6, 9, 5, 3, 1
    x = rnd((N, C, H, H), 20)
    w = rnd((F_, C, k, k), 21, 0.2)
    gy = rnd((N, F_, H, H), 22)
    xk = x.to(DEV).requires_grad_()
    wk = w.to(DEV).requires_grad_()
    F.conv2d(xk, wk, padding=pad).backward(gy.to(DEV))
    wt = np.ascontiguousarray(np.flip(np.swapaxes(w.numpy(), 0, 1), (2, 3)))
    want_gi = O.conv2d(gy.numpy(), wt, None, (1, 1), (k - 1 - pad, k - 1 - pad), (1, 1), 1)
    assert_bits_equal(xk.grad.cpu().numpy(), want_gi, "conv grad_input")
    want_gw = O.conv_weight_grad(x.numpy(), gy.numpy(), w.shape, (1, 1), (pad, pad), (1, 1), 1)
    assert_bits_equal(wk.grad.cpu().numpy(), want_gw, "conv grad_weight")


@pytest.mark.parametrize("stride,groups,dil", [(2, 1, 1), (1, 2, 1), (2, 2, 1), (1, 1, 2)])
def test_conv2d_backward_strided_grouped(stride, groups, dil):
    x = rnd((2, 4, 11, 10), 23)
    w = rnd((6, 4 // groups, 3, 3), 24, 0.3)
    b = rnd((6,), 25, 0.1)
    gy = None
    xr, wr, br = x.float().requires_grad_(), w.float().requires_grad_(), b.float().requires_grad_()
    ref = F.conv2d(xr, wr, br, stride=stride, padding=1, dilation=dil, groups=groups)
    gy = rnd(tuple(ref.shape), 26)
    ref.backward(gy.float())
    xk = x.to(DEV).requires_grad_()
    wk = w.to(DEV).requires_grad_()
    bk = b.to(DEV).requires_grad_()
    out = F.conv2d(xk, wk, bk, stride=stride, padding=1, dilation=dil, groups=groups)
    out.backward(gy.to(DEV))
    for got, want in ((xk.grad, xr.grad), (wk.grad, wr.grad), (bk.grad, br.grad)):
        scale = max(1.0, want.abs().max().item())
        assert (got.cpu().float() - want).abs().max().item() <= 2e-2 * scale
    # the weight gradient is one exact quantised sum: bit-exact against the oracle
    want_gw = O.conv_weight_grad(x.numpy(), gy.numpy(), w.shape, (stride, stride), (1, 1), (dil, dil), groups)
    assert_bits_equal(wk.grad.cpu().numpy(), want_gw, "strided/grouped grad_weight")


def test_cat_out_variants_and_inplace_division():
    """Ops the data-parallel reducer and coalesced broadcast run on the device:
    cat (flatten of a bucket), mul.out into a strided bucket view with a
    wrapped scalar, div_ / sub_ in place."""
    a, b, c = rnd((3, 5), 30), rnd((2, 5), 31), rnd((4, 5), 32, dtype=torch.float32)
    got = torch.cat([a.to(DEV), b.to(DEV), torch.empty(0, dtype=torch.float16).to(DEV), c.to(DEV)]).cpu()
    assert torch.equal(got, torch.cat([a.float(), b.float(), c]))
    got1 = torch.cat([a.to(DEV), a.to(DEV)], dim=1).cpu()
    assert torch.equal(got1, torch.cat([a, a], dim=1))
    bucket = torch.zeros(40, dtype=torch.float16).to(DEV)
    view = bucket.narrow(0, 5, 15).view(3, 5)
    torch.mul(a.to(DEV), 0.5, out=view)
    want = torch.zeros(40, dtype=torch.float16)
    want[5:20] = (a.float() * 0.5).half().reshape(-1)
    assert torch.equal(bucket.cpu(), want)
    x = a.to(DEV)
    x.div_(4)
    assert torch.equal(x.cpu(), (a.float() * 0.25).half())
    x.sub_(b[:1].to(DEV), alpha=2)
    assert torch.allclose(x.cpu().float(), (a.float() * 0.25).half().float() - 2 * b[:1].float(), atol=2e-3)


@pytest.mark.parametrize("H,stride,pad,dil", [(200, 1, 1, 1), (401, 2, 1, 1), (190, 1, 2, 2)])
def test_conv2d_weight_grad_large_image(H, stride, pad, dil):
    """One image's output plane longer than the exact limb limit (32768
    terms): the reduction is split into exact chunks whose int64 sums are
    added before the one rounding, so the weight gradient stays bit-exact."""
    x = rnd((1, 2, H, H), 70)
    w = rnd((3, 2, 3, 3), 71, 0.3)
    xr, wr = x.float().requires_grad_(), w.float().requires_grad_()
    ref = F.conv2d(xr, wr, stride=stride, padding=pad, dilation=dil)
    gy = rnd(tuple(ref.shape), 72)
    ref.backward(gy.float())
    xk, wk = x.to(DEV).requires_grad_(), w.to(DEV).requires_grad_()
    F.conv2d(xk, wk, stride=stride, padding=pad, dilation=dil).backward(gy.to(DEV))
    scale = max(1.0, wr.grad.abs().max().item())
    assert (wk.grad.cpu().float() - wr.grad).abs().max().item() <= 2e-2 * scale
    want_gw = O.conv_weight_grad(x.numpy(), gy.numpy(), w.shape, (stride, stride), (pad, pad), (dil, dil), 1)
    assert_bits_equal(wk.grad.cpu().numpy(), want_gw, f"grad_weight H={H}")
    scale = max(1.0, xr.grad.abs().max().item())
    assert (xk.grad.cpu().float() - xr.grad).abs().max().item() <= 2e-2 * scale


def _wgrad_capi(x, gy, w_shape, stride, pad, dil, groups):
    """tk_conv3d_wgrad_q16 through the C ABI on torch.cuda memory (2-D shapes
    are passed with depth 1)."""
    import ctypes
    from torch_kunlun_b200 import _capi as C
    x5 = x if x.dim() == 5 else x.unsqueeze(2)
    g5 = gy if gy.dim() == 5 else gy.unsqueeze(2)
    ws = tuple(w_shape) if len(w_shape) == 5 else (w_shape[0], w_shape[1], 1) + tuple(w_shape[2:])
    st = tuple(stride) if len(stride) == 3 else (1,) + tuple(stride)
    pd = tuple(pad) if len(pad) == 3 else (0,) + tuple(pad)
    dl = tuple(dil) if len(dil) == 3 else (1,) + tuple(dil)
    xd, gd = x5.contiguous().cuda(), g5.contiguous().cuda()
    out = torch.full(w_shape, float("nan"), dtype=x.dtype, device="cuda")
    d = C.ConvWgradDesc()
    d.dtype = C.TK_DTYPE_F16 if x.dtype == torch.float16 else C.TK_DTYPE_F32
    d.n, d.c, d.d, d.h, d.w = x5.shape
    d.f, _, d.kd, d.kh, d.kw = ws
    d.stride_d, d.stride_h, d.stride_w = st
    d.pad_d, d.pad_h, d.pad_w = pd
    d.dil_d, d.dil_h, d.dil_w = dl
    d.groups = groups
    d.x, d.grad_out, d.grad_weight = xd.data_ptr(), gd.data_ptr(), out.data_ptr()
    L = C.lib()
    nbytes = L.tk_conv3d_wgrad_workspace_size(ctypes.byref(d))
    assert nbytes > 0
    buf = torch.empty(nbytes + 1024, dtype=torch.uint8, device="cuda")
    base = (buf.data_ptr() + 1023) // 1024 * 1024
    C.check(L.tk_conv3d_wgrad_q16(ctypes.byref(d), base, nbytes, torch.cuda.current_stream().cuda_stream),
            "tk_conv3d_wgrad_q16")
    torch.cuda.synchronize()
    assert C.device_error(0) == 0
    return out.cpu().numpy()


@pytest.mark.parametrize("case", [
    # (x shape, F, kernel, stride, pad, dil, groups, dtype)
    ((4, 64, 20, 20), 64, (3, 3), (1, 1), (1, 1), (1, 1), 1, torch.float16),
    ((3, 32, 15, 17), 48, (1, 1), (1, 1), (0, 0), (1, 1), 1, torch.float16),
    ((2, 12, 13, 11), 8, (3, 2), (2, 1), (1, 0), (1, 2), 4, torch.float32),
    ((4, 16, 7, 7), 16, (3, 3), (1, 1), (1, 1), (1, 1), 16, torch.float16),      # depthwise
    ((1, 3, 230, 150), 5, (5, 5), (1, 1), (2, 2), (1, 1), 1, torch.float16),     # P = 34500 > 32768
    ((2, 4, 6, 9, 8), 6, (3, 1, 3), (1, 2, 1), (1, 0, 1), (1, 1, 1), 2, torch.float16),  # 3-D
])
def test_conv_weight_grad_capi_bit_exact(case):
    xs, F_, ks, st, pd, dl, groups, dt = case
    x = torch.relu(rnd(xs, 40, dtype=torch.float32)).to(dt)
    k = len(ks)
    outs = [(xs[2 + i] + 2 * pd[i] - dl[i] * (ks[i] - 1) - 1) // st[i] + 1 for i in range(k)]
    gy = rnd((xs[0], F_) + tuple(outs), 41, dtype=torch.float32).to(dt)
    w_shape = (F_, xs[1] // groups) + tuple(ks)
    got = _wgrad_capi(x, gy, w_shape, st, pd, dl, groups)
    want = O.conv_weight_grad(x.numpy(), gy.numpy(), w_shape, st, pd, dl, groups)
    assert_bits_equal(got, want, f"wgrad {case}")
