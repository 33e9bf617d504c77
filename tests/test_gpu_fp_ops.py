"""The floating-point ops of the path against the oracle's binary64
restatement (oracle/tk_oracle.c: tko_act64, tko_silu_mul, tko_softmax,
tko_layer_norm), at bounds derived from how the device evaluates them.

The device evaluates the same formulas in binary32 with CUDA's erff / tanhf /
expf (documented maximum error 2 ulp) and IEEE-rounded arithmetic, then
rounds once to T; the oracle evaluates them in binary64 and rounds once.
Both roundings to T agree unless the binary32 value lies within its own
error of a rounding boundary of T, where they differ by one ulp of T.  The
bounds below are that one ulp plus the binary32 error itself:

* gelu (erf / tanh) and silu:   |d| <= ulp_T(|y|) + 2^-21 (|x| + |y|)
  (|x| 2^-21 covers the cancellation in 1 + erf(x / sqrt 2) for x << 0:
  erf's 2-ulp error is absolute there, about 2^-22, times 0.5 |x|);
* silu(gate) * up:              |d| <= 2 ulp_16(|y|) + 2^-24
  (T(silu) may differ by one ulp, the product then rounds once more);
* softmax over n columns:       |d| <= ulp_T(|y|) + (n + 8) 2^-24 |y| + 2^-24
  (binary32 exp, a sum of n terms and one division);
* layer_norm over n columns:    |d| <= ulp_T(|y|) + (n + 8) 2^-24 (|y| + |gamma| (1 + |x - mean| rstd)) + 2^-24
  (binary32 two-pass mean / variance, rsqrtf, the affine step).

The fused GEMM epilogues (linear + GELU for BERT's FFN1, linear + SiLU) are
exact up to the activation: the pre-activation value is the bit-exact
integer result, so they take the activation's bound."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

torch_kunlun = pytest.importorskip("torch_kunlun")
from oracle import oracle as O  # noqa: E402
from torch_kunlun_b200 import ops  # noqa: E402

DEV = "kunlun"


def rnd(shape, seed, dtype=torch.float16, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(shape, generator=g) * scale).to(dtype)


def ulp(a, dtype):
    a = np.abs(np.asarray(a, dtype=np.float64))
    if dtype == np.float16:
        e = np.floor(np.log2(np.maximum(a, 2.0 ** -14)))
        return 2.0 ** (e - 10)
    e = np.floor(np.log2(np.maximum(a, 2.0 ** -126)))
    return 2.0 ** (e - 23)


def assert_within(got, want, bound, what):
    g = np.asarray(got, dtype=np.float64)
    w = np.asarray(want, dtype=np.float64)
    assert g.shape == w.shape
    err = np.abs(g - w)
    bad = ~(err <= bound)
    assert not bad.any(), (f"{what}: {int(bad.sum())} of {g.size} beyond the bound; first at "
                           f"{np.argwhere(bad)[:3].tolist()} got {g[bad][:3]} want {w[bad][:3]}")


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
@pytest.mark.parametrize("kind", ["gelu", "gelu_tanh", "silu"])
def test_activations_within_bound(dtype, kind):
    x = rnd((256, 1024), 1, dtype, 3.0)
    x[0, :8] = torch.tensor([0.0, -0.0, 1e-4, -1e-4, 12.0, -12.0, 30.0, -30.0], dtype=dtype)
    xd = x.to(DEV)
    if kind == "silu":
        got = torch.nn.functional.silu(xd)
    else:
        got = torch.nn.functional.gelu(xd, approximate="tanh" if kind == "gelu_tanh" else "none")
    xn = x.numpy()
    want = O.act(xn, kind)
    nd = np.float16 if dtype == torch.float16 else np.float32
    bound = ulp(want, nd) + 2.0 ** -21 * (np.abs(xn.astype(np.float64)) + np.abs(want.astype(np.float64)))
    assert_within(got.cpu().numpy(), want, bound, kind)


@pytest.mark.parametrize("act", ["gelu", "silu", "gelu_tanh"])
def test_fused_linear_activation_epilogue(act):
    """linear + activation in the GEMM epilogue: the pre-activation is the
    bit-exact quantised result, the activation is within its bound."""
    x, w, b = rnd((300, 768), 2), rnd((512, 768), 3, scale=0.02), rnd((512,), 4, scale=0.01)
    got = ops.linear(x.to(DEV), w.to(DEV), b.to(DEV), act=act).cpu().numpy()
    pre = O.linear(x.numpy(), w.numpy(), b.numpy())
    want = O.linear(x.numpy(), w.numpy(), b.numpy(), act=O.ACT_CODES[act])
    assert np.array_equal(want, O.act(pre, act))  # the oracle's epilogue is act(T(pre))
    bound = ulp(want, np.float16) + 2.0 ** -21 * (np.abs(pre.astype(np.float64)) + np.abs(want.astype(np.float64)))
    assert_within(got, want, bound, f"linear+{act}")


def test_bert_ffn1_epilogue_full_size():
    """BERT-base FFN1 at full size: h [16384, 768] x W1 [3072, 768]^T + b1,
    GELU in the epilogue; checked on 1024 sampled rows with the whole h's
    scale."""
    g = torch.Generator().manual_seed(5)
    h = torch.randn(16384, 768, generator=g).half()
    w = (torch.randn(3072, 768, generator=g) * 0.02).half()
    b = (torch.randn(3072, generator=g) * 0.02).half()
    got = ops.linear(h.to(DEV), w.to(DEV), b.to(DEV), act="gelu").cpu().numpy()
    rows = np.random.default_rng(6).choice(16384, 1024, replace=False)
    hn, wn, bn = h.numpy(), w.numpy(), b.numpy()
    ah, aw = O.amax(hn), O.amax(wn)
    acc = O.gemm_i16_exact(O.quant(hn[rows], ah), O.quant(wn, aw).T)
    pre = O.epilogue(acc, ah, aw, np.float16, bias=bn)
    want = O.epilogue(acc, ah, aw, np.float16, bias=bn, act=O.ACT_GELU)
    bound = ulp(want, np.float16) + 2.0 ** -21 * (np.abs(pre.astype(np.float64)) + np.abs(want.astype(np.float64)))
    assert_within(got[rows], want, bound, "FFN1 gelu epilogue")


def test_silu_gate_tp_shard_size():
    """The SiLU gate of the tensor-parallel MLP on one TP-8 shard's width:
    T(T(silu(gate)) * up) over [16384, 3584]."""
    g = rnd((16384, 3584), 7, scale=0.5)
    u = rnd((16384, 3584), 8, scale=0.5)
    got = ops.silu_mul(g.to(DEV), u.to(DEV)).cpu().numpy()
    want = O.silu_mul(g.numpy(), u.numpy())
    assert_within(got, want, 2 * ulp(want, np.float16) + 2.0 ** -24, "silu * up")
    frac = float(np.mean(got.view(np.uint16) != want.view(np.uint16)))
    assert frac < 1e-3, frac  # the binary32 error rarely reaches a binary16 boundary


@pytest.mark.parametrize("shape,out32", [((64 * 512, 512), False), ((1024, 768), False), ((512, 3000), False),
                                         ((1024, 512), True)])
def test_softmax_within_bound(shape, out32):
    x = rnd(shape, 9, scale=2.0)
    xd = x.to(DEV)
    got = (torch.softmax(xd, -1, dtype=torch.float32) if out32 else torch.softmax(xd, -1)).cpu().numpy()
    want = O.softmax(x.numpy(), out_dtype=np.float32 if out32 else np.float16)
    n = shape[-1]
    nd = np.float32 if out32 else np.float16
    w64 = np.abs(want.astype(np.float64))
    assert_within(got, want, ulp(want, nd) + (n + 8) * 2.0 ** -24 * w64 + 2.0 ** -24, "softmax")


@pytest.mark.parametrize("rows,cols,wdt", [(16384, 768, torch.float16), (333, 1024, torch.float32),
                                           (64, 5000, torch.float16)])
def test_layer_norm_within_bound(rows, cols, wdt):
    x = rnd((rows, cols), 10, wdt, scale=1.5)
    gamma = (1 + 0.2 * rnd((cols,), 11, torch.float32)).to(wdt)
    beta = (0.2 * rnd((cols,), 12, torch.float32)).to(wdt)
    got = torch.nn.functional.layer_norm(x.to(DEV), (cols,), gamma.to(DEV), beta.to(DEV), 1e-12).cpu().numpy()
    want, mean, rstd = O.layer_norm(x.numpy(), gamma.numpy(), beta.numpy(), 1e-12, return_stats=True)
    xc = np.abs(x.numpy().astype(np.float64) - mean.astype(np.float64)[:, None]) * rstd.astype(np.float64)[:, None]
    g64 = np.abs(gamma.numpy().astype(np.float64))[None, :]
    w64 = np.abs(want.astype(np.float64))
    nd = np.float16 if wdt == torch.float16 else np.float32
    bound = ulp(want, nd) + (cols + 8) * 2.0 ** -24 * (w64 + g64 * (1 + xc)) + 2.0 ** -24
    assert_within(got, want, bound, "layer_norm")
