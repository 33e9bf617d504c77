"""GPU tests of the kunlun device through torch (the reference's own test
style: tests/test_runtime.py, test_numeric_semantics.py, test_transformer_ops.py,
test_attention.py, test_stream_event.py), with the quantised ops checked
bit-for-bit against the CPU oracle and everything else against float64
references at stated tolerances."""
import math

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

torch_kunlun = pytest.importorskip("torch_kunlun")
kunlun = torch_kunlun.kunlun
from oracle import oracle as O  # noqa: E402
from tests._qgemm_helpers import assert_bits_equal  # noqa: E402

DEV = "kunlun"


def rnd(shape, dtype=torch.float16, seed=0, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(shape, generator=g) * scale).to(dtype)


@pytest.fixture(autouse=True)
def _no_device_error():
    yield
    from torch_kunlun_b200 import _capi
    assert _capi.device_error(0) == 0


# ---- runtime (reference tests/test_runtime.py) -------------------------------

def test_device_count_and_properties():
    assert kunlun.is_available() and kunlun.device_count() > 0
    p = kunlun.get_device_properties(0)
    assert p.multi_processor_count >= 100 and p.warp_size == 32 and p.total_memory > 100e9


def test_empty_fill_copy():
    x = torch.empty(1024, dtype=torch.float16, device=DEV)
    assert x.device.type == "kunlun"
    x.fill_(1.0)
    y = torch.empty_like(x)
    y.copy_(x)
    kunlun.synchronize()
    assert torch.all(y.cpu() == 1.0)


def test_add_relu_exact():
    a, b = rnd(128, seed=1), rnd(128, seed=2)
    c = torch.add(a.to(DEV), b.to(DEV))
    r = torch.relu(c)
    assert torch.equal(c.cpu(), a + b)
    assert torch.equal(r.cpu(), torch.relu(a + b))


def test_add_broadcast_both_orders():
    a, b = rnd((4, 8), seed=3), rnd(8, seed=4)
    ad, bd = a.to(DEV), b.to(DEV)
    assert torch.equal(torch.add(ad, bd).cpu(), a + b)
    assert torch.equal(torch.add(bd, ad).cpu(), a + b)


def test_scalar_arith_and_item():
    a = rnd((5, 7), torch.float32, seed=5)
    ad = a.to(DEV)
    assert torch.allclose((ad * 3.0).cpu(), a * 3.0)
    assert torch.allclose((ad + 2.0).cpu(), a + 2.0)
    assert torch.allclose((ad - 1.5).cpu(), a - 1.5)
    assert torch.allclose((ad / 4.0).cpu(), a / 4.0)
    assert ad[1, 2].item() == a[1, 2].item()


def test_empty_strided_zero():
    x = torch.empty_strided((4, 8), (8, 1), dtype=torch.float16, device=DEV)
    assert x.stride() == (8, 1)
    x.zero_()
    assert torch.all(x.cpu() == 0)


@pytest.mark.parametrize("dtype,value", [(torch.bool, True), (torch.uint8, 200), (torch.int8, -7),
                                         (torch.int16, -3000), (torch.int32, 123456),
                                         (torch.int64, -1234567890123), (torch.float64, 1.5)])
def test_fill_non_float_dtypes(dtype, value):
    x = torch.empty(1000, dtype=dtype, device=DEV)
    x.fill_(value)
    assert torch.equal(x.cpu(), torch.full((1000,), value, dtype=dtype))


def test_fill_rejects_overflowing_scalar():
    x = torch.empty(4, dtype=torch.int8, device=DEV)
    with pytest.raises(RuntimeError):
        x.fill_(1000)


def test_copy_overlapping_views_and_transpose():
    x = torch.arange(16, dtype=torch.float16).to(DEV)
    x[1:].copy_(x[:-1])
    e = torch.arange(16, dtype=torch.float16)
    e[1:] = e[:-1].clone()
    assert torch.equal(x.cpu(), e)
    src = torch.arange(12, dtype=torch.float16).reshape(3, 4).to(DEV)
    dst = torch.empty(4, 3, dtype=torch.float16, device=DEV)
    dst.copy_(src.t())
    assert torch.equal(dst.cpu(), src.cpu().t())
    assert torch.equal(src.t().contiguous().cpu(), src.cpu().t().contiguous())


def test_dtype_conversion_on_device():
    a = rnd((33, 17), torch.float32, seed=6)
    ad = a.to(DEV)
    assert torch.equal(ad.half().cpu(), a.half())
    assert torch.equal(ad.half().float().cpu(), a.half().float())
    assert torch.equal(ad.to(torch.float64).cpu(), a.double())


def test_large_allocation_has_no_2gib_cap():
    x = torch.empty(3 * (1 << 30), dtype=torch.uint8, device=DEV)
    assert x.numel() == 3 * (1 << 30)
    del x
    kunlun.empty_cache()


def test_cpu_fallback_denied_by_default():
    x = torch.ones(8, dtype=torch.float32, device=DEV)
    with pytest.raises(RuntimeError, match="generic CPU fallback is disabled"):
        torch.cumsum(x, 0)


# ---- quantised dense ops vs the oracle (bit-exact) ---------------------------

@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
@pytest.mark.parametrize("M,K,N", [(16, 32, 24), (129, 257, 130), (512, 768, 256)])
def test_mm_linear_addmm_bit_exact(dtype, M, K, N):
    a, b = rnd((M, K), dtype, 10), rnd((K, N), dtype, 11)
    w, bias = rnd((N, K), dtype, 12, 0.02), rnd((N,), dtype, 13, 0.01)
    an, bn, wn, biasn = a.numpy(), b.numpy(), w.numpy(), bias.numpy()
    assert_bits_equal(torch.mm(a.to(DEV), b.to(DEV)).cpu().numpy(), O.mm(an, bn), "mm")
    assert_bits_equal(torch.nn.functional.linear(a.to(DEV), w.to(DEV), bias.to(DEV)).cpu().numpy(),
                      O.linear(an, wn, biasn), "linear")
    s = rnd((M, N), dtype, 14)
    got = torch.addmm(s.to(DEV), a.to(DEV), b.to(DEV), beta=0.5, alpha=2.0).cpu().numpy()
    assert_bits_equal(got, O.addmm(s.numpy(), an, bn, beta=0.5, alpha=2.0), "addmm")


def test_linear_3d_input_and_autograd_path():
    x = rnd((2, 5, 64), seed=15)
    w, b = rnd((32, 64), seed=16, scale=0.05), rnd((32,), seed=17, scale=0.01)
    want = O.linear(x.reshape(-1, 64).numpy(), w.numpy(), b.numpy()).reshape(2, 5, 32)
    y = torch.nn.functional.linear(x.to(DEV), w.to(DEV), b.to(DEV))
    assert y.shape == (2, 5, 32)
    assert_bits_equal(y.cpu().numpy(), want, "linear 3d")
    wd = w.to(DEV).requires_grad_()
    y2 = torch.nn.functional.linear(x.to(DEV), wd, b.to(DEV))
    assert y2.requires_grad
    assert_bits_equal(y2.detach().cpu().numpy(), want, "linear 3d with grad")


def test_reference_fp16_mm_accuracy_bound():
    # reference tests/test_numeric_semantics.py:49-57
    torch.manual_seed(0)
    x = torch.randn(64, 128, dtype=torch.float16)
    w = torch.randn(128, 64, dtype=torch.float16)
    exact = x.float() @ w.float()
    out = (x.to(DEV) @ w.to(DEV)).cpu().float()
    assert ((out - exact).norm() / exact.norm()) < 5e-3


def test_reference_fp32_probe_value():
    x = torch.tensor([[1e-5, 1.0]], dtype=torch.float32, device=DEV)
    w = torch.tensor([[1.0], [1e5]], dtype=torch.float32, device=DEV)
    assert (x @ w).cpu().item() == np.float32(1e5)


@pytest.mark.parametrize("B,M,K,N", [(4, 33, 65, 17), (64, 512, 128, 512)])
def test_bmm_baddbmm_matmul_bit_exact(B, M, K, N):
    a, b = rnd((B, M, K), seed=20), rnd((B, K, N), seed=21)
    a[1] *= 50
    an, bn = a.numpy(), b.numpy()
    assert_bits_equal(torch.bmm(a.to(DEV), b.to(DEV)).cpu().numpy(), O.bmm(an, bn), "bmm")
    s = rnd((B, M, N), seed=22)
    got = torch.baddbmm(s.to(DEV), a.to(DEV), b.to(DEV), beta=1.0, alpha=0.125).cpu().numpy()
    assert_bits_equal(got, O.baddbmm(s.numpy(), an, bn, beta=1.0, alpha=0.125), "baddbmm")
    assert_bits_equal(torch.matmul(a.to(DEV), b.to(DEV)).cpu().numpy(), O.bmm(an, bn), "matmul 3d")
    a4, b4 = a.reshape(2, B // 2, M, K), b.reshape(2, B // 2, K, N)
    got4 = torch.matmul(a4.to(DEV), b4.to(DEV)).cpu().numpy().reshape(B, M, N)
    assert_bits_equal(got4, O.bmm(an, bn), "matmul 4d")


CONV_CASES = [
    # N, C, H, W, F, k, stride, pad, dil, groups, bias
    (2, 8, 9, 7, 16, 3, 1, 1, 1, 1, True),
    (2, 16, 12, 12, 8, 1, 1, 0, 1, 1, False),
    (1, 6, 11, 13, 12, 3, 2, 0, 1, 3, True),
    (2, 8, 7, 7, 8, 3, 1, 1, 1, 8, True),
    (1, 4, 10, 10, 6, 5, 1, 2, 2, 1, False),
]


@pytest.mark.parametrize("case", CONV_CASES)
def test_conv2d_bit_exact(case):
    N, C, H, W, F, k, s, p, d, g, has_b = case
    x = torch.relu(rnd((N, C, H, W), seed=30))
    w = rnd((F, C // g, k, k), seed=31, scale=math.sqrt(2.0 / (C // g * k * k)))
    b = rnd((F,), seed=32, scale=0.01) if has_b else None
    y = torch.nn.functional.conv2d(x.to(DEV), w.to(DEV), b.to(DEV) if has_b else None,
                                   stride=s, padding=p, dilation=d, groups=g)
    want = O.conv2d(x.numpy(), w.numpy(), None if b is None else b.numpy(), (s, s), (p, p),
                    (d, d), g)
    assert_bits_equal(y.cpu().numpy(), want, f"conv2d {case}")


def test_conv2d_reference_tolerance():
    # reference tests/test_runtime.py:62-69
    x = torch.randn(1, 4, 8, 8, dtype=torch.float16)
    w = torch.randn(8, 4, 3, 3, dtype=torch.float16)
    b = torch.randn(8, dtype=torch.float16)
    y = torch.conv2d(x.to(DEV), w.to(DEV), b.to(DEV), padding=1).cpu()
    assert torch.allclose(y, torch.conv2d(x.float(), w.float(), b.float(), padding=1).half(),
                          atol=5e-2, rtol=5e-2)


# ---- row ops and activations (float64 references, stated tolerances) ----------

def test_softmax_layer_norm_gelu_silu():
    x = rnd((64, 768), seed=40)
    xd = x.to(DEV)
    y = torch.softmax(xd, dim=-1).cpu()
    assert torch.allclose(y.float(), torch.softmax(x.double(), -1).float(), atol=1e-3, rtol=2e-3)
    g, bb = rnd(768, seed=41), rnd(768, seed=42)
    z = torch.nn.functional.layer_norm(xd, (768,), g.to(DEV), bb.to(DEV), 1e-12).cpu()
    ref = torch.nn.functional.layer_norm(x.double(), (768,), g.double(), bb.double(), 1e-12)
    assert (z.double() - ref).abs().max() < 1e-2
    assert torch.allclose(torch.nn.functional.gelu(xd).cpu().float(),
                          torch.nn.functional.gelu(x.double()).float(), atol=2e-3, rtol=2e-3)
    assert torch.allclose(torch.nn.functional.silu(xd).cpu().float(),
                          torch.nn.functional.silu(x.double()).float(), atol=2e-3, rtol=2e-3)
    y32 = torch.softmax(xd.float(), dim=0).cpu()
    assert torch.allclose(y32, torch.softmax(x.float(), 0), atol=1e-6, rtol=1e-5)


# ---- attention (reference tests/test_attention.py) ------------------------------

@pytest.mark.parametrize("shape", [(2, 3, 5, 4), (2, 4, 5, 8), (2, 12, 128, 64)])
def test_sdpa_matches_oracle_composition(shape):
    q, k, v = rnd(shape, seed=50), rnd(shape, seed=51), rnd(shape, seed=52)
    L = shape[2]
    mask = torch.zeros(shape[0], 1, L, L, dtype=torch.float16)
    mask[..., L - max(1, L // 8):] = -1e4
    out = kunlun.scaled_dot_product_attention(q.to(DEV), k.to(DEV), v.to(DEV),
                                              attn_mask=mask.to(DEV)).cpu()
    BH = shape[0] * shape[1]
    m3 = mask.expand(shape[0], shape[1], L, L).reshape(BH, L, L).numpy()
    want = O.sdpa(q.reshape(BH, L, -1).numpy(), k.reshape(BH, L, -1).numpy(),
                  v.reshape(BH, L, -1).numpy(), mask=m3)
    got = out.reshape(BH, L, -1).float().numpy()
    # softmax is the only non-integer step; its fp16 output may differ by one
    # ulp from the float64 oracle, which the second quantised bmm can amplify
    assert np.abs(got - want.astype(np.float32)).max() < 2e-2
    ref = torch.softmax((q.float() @ k.float().transpose(-1, -2)) / math.sqrt(shape[-1]) + mask.float(),
                        -1) @ v.float()
    assert torch.allclose(out.float(), ref, atol=5e-2, rtol=5e-2)


def test_sdpa_causal_and_bool_mask():
    q, k, v = rnd((1, 2, 16, 8), seed=53), rnd((1, 2, 16, 8), seed=54), rnd((1, 2, 16, 8), seed=55)
    out = kunlun.scaled_dot_product_attention(q.to(DEV), k.to(DEV), v.to(DEV), is_causal=True).cpu()
    ref = torch.nn.functional.scaled_dot_product_attention(q.float(), k.float(), v.float(),
                                                           is_causal=True)
    assert torch.allclose(out.float(), ref, atol=5e-2, rtol=5e-2)
    bm = torch.zeros(16, 16, dtype=torch.bool)
    bm[:, 12:] = True
    out2 = kunlun.scaled_dot_product_attention(q.to(DEV), k.to(DEV), v.to(DEV), attn_mask=bm.to(DEV)).cpu()
    ref2 = torch.nn.functional.scaled_dot_product_attention(q.float(), k.float(), v.float(),
                                                            attn_mask=~bm)
    assert torch.allclose(out2.float(), ref2, atol=5e-2, rtol=5e-2)


# ---- streams and events (reference tests/test_stream_event.py) -------------------

def test_stream_event_roundtrip():
    s = kunlun.Stream()
    assert isinstance(s, torch.Stream)
    e0, e1 = kunlun.Event(enable_timing=True), kunlun.Event(enable_timing=True)
    a = rnd((1024, 1024), seed=60).to(DEV)
    with kunlun.stream(s):
        assert kunlun.current_stream().stream_id == s.stream_id
        e0.record()
        c = a @ a
        e1.record()
        c.record_stream(s)
    assert kunlun.current_stream().stream_id == 0
    e1.synchronize()
    assert e1.query() and s.query()
    assert e0.elapsed_time(e1) >= 0.0
    s.synchronize()
    ds = kunlun.default_stream()
    ds.wait_stream(s)
    assert torch.isfinite(c.cpu().float()).all()


def test_memory_stats():
    kunlun.synchronize()
    before = kunlun.memory_allocated()
    x = torch.empty(1 << 20, dtype=torch.float32, device=DEV)
    assert kunlun.memory_allocated() >= before + (1 << 22)
    assert kunlun.memory_reserved() >= kunlun.memory_allocated()
    del x
    kunlun.synchronize()
    assert kunlun.memory_allocated() == before
