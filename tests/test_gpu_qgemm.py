"""GPU parity of the quantise kernels and the tensor-core limb GEMM, called
through the C ABI, against the CPU oracle.  Integer work and the whole
dequant/bias/alpha/beta/relu epilogue are required to be bit-exact."""
import ctypes

import numpy as np
import pytest
import torch

from oracle import oracle as O
from torch_kunlun_b200 import _capi as C
from tests._qgemm_helpers import (assert_bits_equal, limb_accumulators, oracle_qgemm,
                                  qgemm)

pytestmark = pytest.mark.gpu


def _rand(shape, dtype, seed, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(shape, generator=g) * scale).to(dtype).cuda()


@pytest.fixture(autouse=True)
def _no_device_error():
    yield
    assert C.device_error(0) == 0, "a kernel recorded a device-side timeout"


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
@pytest.mark.parametrize("shape", [(1, 1), (3, 1000), (64, 4096), (257, 1031)])
def test_amax_and_limbs(dtype, shape):
    x = _rand(shape, dtype, 1)
    x.view(-1)[7 % x.numel()] = -3.5
    L = C.lib()
    amax = torch.empty(1, dtype=torch.float32, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    dc = C.TK_DTYPE_F16 if dtype == torch.float16 else C.TK_DTYPE_F32
    C.check(L.tk_amax(dc, x.data_ptr(), 1, 0, x.numel(), amax.data_ptr(), st), "amax")
    rows, cols = shape
    ld = (cols + 15) // 16 * 16
    limbs = torch.empty((2, rows, ld), dtype=torch.int8, device="cuda")
    C.check(L.tk_quantize_limbs(dc, x.data_ptr(), 1, rows, cols, 0, cols, 1, amax.data_ptr(), 0,
                                limbs.data_ptr(), st), "quantize")
    torch.cuda.synchronize()
    xn = x.cpu().numpy()
    assert amax.item() == O.amax(xn)
    q = O.quant(xn)
    hi, lo = O.limbs(q)
    ln = limbs.cpu().numpy()
    assert np.array_equal(ln[0, :, :cols], hi)
    assert np.array_equal(ln[1, :, :cols].view(np.uint8), lo)
    assert np.all(ln[:, :, cols:] == 0)


def test_quantize_transposed_view():
    x = _rand((300, 200), torch.float16, 2)
    xt = x.t()  # [200, 300] view with row stride 1
    L = C.lib()
    amax = torch.empty(1, dtype=torch.float32, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    C.check(L.tk_amax(0, x.data_ptr(), 1, 0, x.numel(), amax.data_ptr(), st), "amax")
    ld = 304
    limbs = torch.empty((2, 200, ld), dtype=torch.int8, device="cuda")
    C.check(L.tk_quantize_limbs(0, xt.data_ptr(), 1, 200, 300, 0, xt.stride(0), xt.stride(1),
                                amax.data_ptr(), 0, limbs.data_ptr(), st), "quantize")
    torch.cuda.synchronize()
    hi, lo = O.limbs(O.quant(xt.cpu().numpy()))
    ln = limbs.cpu().numpy()
    assert np.array_equal(ln[0, :, :300], hi) and np.array_equal(ln[1, :, :300].view(np.uint8), lo)


SHAPES = [(128, 128, 128), (1, 1, 1), (7, 5, 33), (129, 130, 257), (256, 384, 1024),
          (300, 200, 4096)]


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_limb_accumulators_exact(M, N, K):
    a = _rand((1, M, K), torch.float16, 10)
    w = _rand((1, N, K), torch.float16, 11, 0.02)
    out, dbg = qgemm(a, w, debug=True)
    hh, mid, ll = limb_accumulators(a[0], w[0])
    d = dbg.cpu().numpy().astype(np.int64)
    assert np.array_equal(d[0], hh), "HH accumulator differs"
    assert np.array_equal(d[1], mid), "MID accumulator differs"
    assert np.array_equal(d[2], ll), "LL accumulator differs"
    assert_bits_equal(out.cpu().numpy(), oracle_qgemm(a, w), "out")


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
@pytest.mark.parametrize("M,N,K", SHAPES)
def test_linear_layout_bit_exact(dtype, M, N, K):
    a = _rand((1, M, K), dtype, 20)
    w = _rand((1, N, K), dtype, 21, 0.02)
    bias = _rand((N,), dtype, 22, 0.01)
    got = qgemm(a, w, bias=bias)
    assert_bits_equal(got.cpu().numpy(), oracle_qgemm(a, w, bias=bias), "linear")


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
@pytest.mark.parametrize("M,N,K", [(64, 96, 160), (200, 136, 520)])
def test_mm_layout_addmm_epilogue(dtype, M, N, K):
    a = _rand((1, M, K), dtype, 30)
    b_kn = _rand((1, K, N), dtype, 31)
    b_nk = b_kn.transpose(1, 2)  # [1, N, K] view with n-stride 1
    addend = _rand((1, M, N), dtype, 32)
    got = qgemm(a, b_nk, addend=addend, alpha=0.5, beta=-1.25, act="relu")
    want = oracle_qgemm(a, b_nk, addend=addend, alpha=0.5, beta=-1.25, act="relu")
    assert_bits_equal(got.cpu().numpy(), want, "addmm")


@pytest.mark.parametrize("B,M,N,K", [(4, 64, 80, 48), (3, 130, 129, 128)])
def test_bmm_per_slice_scales(B, M, N, K):
    a = _rand((B, M, K), torch.float16, 40)
    b = _rand((B, K, N), torch.float16, 41)
    # make slice scales differ strongly
    a[1] *= 100
    b[2] *= 0.001
    b_nk = b.transpose(1, 2)
    got = qgemm(a, b_nk, per_slice=True)
    assert_bits_equal(got.cpu().numpy(), oracle_qgemm(a, b_nk, per_slice=True), "bmm")


def test_tensor_core_matches_simt_kernel():
    a = _rand((2, 190, 300), torch.float16, 50)
    w = _rand((2, 70, 300), torch.float16, 51)
    tc = qgemm(a, w)
    simt = qgemm(a, w, path="simt")
    assert torch.equal(tc.view(torch.int16), simt.view(torch.int16))


def test_edge_values():
    a = torch.zeros((1, 16, 64), dtype=torch.float16, device="cuda")
    w = _rand((1, 32, 64), torch.float16, 60)
    assert torch.all(qgemm(a, w) == 0)
    a = _rand((1, 16, 64), torch.float16, 61)
    a[0, 3, 5] = float("inf")
    out = qgemm(a, w)
    assert torch.all(torch.isnan(out))
    # extremes of the int16 range in every limb: +-amax everywhere
    a = torch.full((1, 128, 32768), 1.0, dtype=torch.float16, device="cuda")
    a[0, ::2] = -1.0
    w = torch.full((1, 128, 32768), -2.0, dtype=torch.float16, device="cuda")
    assert_bits_equal(qgemm(a, w).cpu().numpy(), oracle_qgemm(a, w), "extreme K")


@pytest.mark.parametrize("M,N,K", [(130, 70, 40000), (64, 200, 65536), (33, 17, 131072)])
def test_long_k_split_bit_exact(M, N, K):
    # K > 32768: the reduction is split into exact int32-limb chunks whose
    # int64 sums are added in a workspace, then dequantised once
    a = _rand((1, M, K), torch.float16, 70)
    w = _rand((1, N, K), torch.float16, 71, 0.02)
    bias = _rand((N,), torch.float16, 72, 0.01)
    got = qgemm(a, w, bias=bias)
    assert_bits_equal(got.cpu().numpy(), oracle_qgemm(a, w, bias=bias), f"K={K}")


def test_long_k_split_mm_layout_and_epilogue():
    # [K, N] operand (transposed quantiser), alpha, beta * addend, relu
    a = _rand((1, 96, 70000), torch.float16, 73)
    b_kn = _rand((1, 70000, 40), torch.float16, 74)
    add = _rand((1, 96, 40), torch.float16, 75)
    got = qgemm(a, b_kn.transpose(1, 2), addend=add, alpha=0.75, beta=-1.5, act="relu")
    want = oracle_qgemm(a, b_kn.transpose(1, 2), addend=add, alpha=0.75, beta=-1.5, act="relu")
    assert_bits_equal(got.cpu().numpy(), want, "split mm epilogue")


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_long_k_split_batched_per_slice(dtype):
    a = _rand((3, 100, 40000), dtype, 76)
    w = _rand((3, 50, 40000), dtype, 77)
    assert_bits_equal(qgemm(a, w).cpu().numpy(), oracle_qgemm(a, w), "split bmm")


def test_few_tiles_long_k_split_equals_unsplit_result():
    # 4 output tiles with K = 8192: the reduction is spread over K chunks to
    # occupy the SMs; the int64 sums make it identical to the oracle
    a = _rand((1, 256, 8192), torch.float16, 78)
    w = _rand((1, 256, 8192), torch.float16, 79)
    got = qgemm(a, w)
    assert_bits_equal(got.cpu().numpy(), oracle_qgemm(a, w), "few-tile split")
    simt = qgemm(a, w, path="simt")
    assert torch.equal(got.view(torch.int16), simt.view(torch.int16))


def test_linear_weight_gradient_over_131072_tokens():
    # the weight gradient of a linear reduces over the tokens: K = 131072
    import torch_kunlun  # noqa: F401
    g = torch.Generator().manual_seed(80)
    x = torch.randn(131072, 64, generator=g).half()
    w = (torch.randn(32, 64, generator=g) * 0.02).half()
    gy = (torch.randn(131072, 32, generator=g) * 0.1).half()
    xd = x.to("kunlun:0").requires_grad_(True)
    wd = w.to("kunlun:0").requires_grad_(True)
    y = torch.nn.functional.linear(xd, wd)
    y.backward(gy.to("kunlun:0"))
    got = wd.grad.cpu().numpy()
    want = O.mm(x.numpy().T.copy(), gy.numpy()).T  # (x^T g)^T, one scale per operand
    assert_bits_equal(got, want, "linear wgrad K=131072")


def test_mid_accumulator_worst_case():
    # q = -32513 gives hi = -128, lo = 255: the largest |hi*lo + lo*hi| per
    # product (65280); at K = 32768 the MID accumulator reaches -2139095040.
    v = np.float32(-32513.0 / 32767.0)
    a = torch.full((1, 128, 32768), float(v), dtype=torch.float32, device="cuda")
    a[0, 0, 0] = 1.0
    w = a.clone()
    got, dbg = qgemm(a, w, debug=True)
    q = O.quant(np.array([v, 1.0], np.float32))
    assert q[0] == -32513
    assert_bits_equal(got.cpu().numpy(), oracle_qgemm(a, w), "worst-case MID")


def test_supplied_amax_below_max_clamps_like_the_oracle():
    # A caller-supplied amax below max|x| scales some values past the code
    # range: they clamp to +-32767 (and +-inf with it), NaN gives code 0,
    # exactly as the oracle's quantiser.
    import torch_kunlun  # noqa: F401
    from torch_kunlun_b200 import ops
    g = torch.Generator().manual_seed(91)
    x = torch.randn(130, 520, generator=g).half()
    w = (torch.randn(200, 520, generator=g) * 0.02).half()
    x[3, 7] = float("inf")
    x[5, 9] = float("-inf")
    x[8, 1] = float("nan")
    finite = x[torch.isfinite(x)]
    ax = np.float32(0.5 * float(finite.abs().max()))
    xd, wd = x.to("kunlun:0"), w.to("kunlun:0")
    ax_t = torch.tensor([ax], dtype=torch.float32).to("kunlun:0")
    got = ops.linear_scaled(xd, wd, amax_x=ax_t).cpu().numpy()
    xn, wn = x.numpy(), w.numpy()
    aw = O.amax(wn)
    qx = O.quant(xn, ax)
    assert qx[3, 7] == 32767 and qx[5, 9] == -32767 and qx[8, 1] == 0
    assert (qx == 32767).sum() > 10 and (qx == -32767).sum() > 10
    acc = O.gemm_i16_exact(qx, O.quant(wn, aw).T)
    want = O.epilogue(acc, ax, aw, np.float16)
    assert_bits_equal(got, want, "linear_scaled with amax_x = max|x| / 2")
