"""Parity at the benchmark configurations' full sizes.

The device runs each workload whole; the oracle recomputes a sample of the
outputs exactly -- the per-tensor (or per-slice) max-abs of the WHOLE operands,
the int16 codes of only the sampled rows / columns / receptive fields, exact
int64 dot products, and the oracle's epilogue -- so the comparison is bit-exact
at sizes the oracle could not finish whole in seconds.  Samples include the
first and last rows, columns and border pixels.  Attention is checked on whole
slices of the BERT-size batch at the attention tests' stated tolerance."""
import math

import numpy as np
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

torch_kunlun = pytest.importorskip("torch_kunlun")
from oracle import oracle as O  # noqa: E402
from tests._qgemm_helpers import assert_bits_equal  # noqa: E402

DEV = "kunlun"


def _sample(n, k, seed):
    rng = np.random.default_rng(seed)
    idx = set(rng.choice(n, size=min(n, k), replace=False).tolist()) | {0, n - 1}
    return np.array(sorted(idx))


def _linear_case(M, N, K, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, K, generator=g).half()
    w = (torch.randn(N, K, generator=g) * 0.02).half()
    b = (torch.randn(N, generator=g) * 0.01).half()
    y = F.linear(x.to(DEV), w.to(DEV), b.to(DEV)).cpu().numpy()
    xn, wn, bn = x.numpy(), w.numpy(), b.numpy()
    ax, aw = O.amax(xn), O.amax(wn)
    rows, cols = _sample(M, 14, seed + 1), _sample(N, 126, seed + 2)
    qx = O.quant(xn[rows], ax).astype(np.int64)
    qw = O.quant(wn[cols], aw).astype(np.int64)
    want = O.epilogue(qx @ qw.T, ax, aw, np.float16, bias=bn[cols])
    assert_bits_equal(y[np.ix_(rows, cols)], want, f"linear {M}x{N}x{K}")


def test_linear_cfg1_2048x4096x4096():
    _linear_case(2048, 4096, 4096, 0)


def test_linear_4096_cubed():
    _linear_case(4096, 4096, 4096, 10)


def test_bmm_cfg2_per_slice_scales():
    g = torch.Generator().manual_seed(20)
    a = torch.randn(64, 512, 128, generator=g).half()
    b = torch.randn(64, 128, 512, generator=g).half()
    y = torch.bmm(a.to(DEV), b.to(DEV)).cpu().numpy()
    an, bn = a.numpy(), b.numpy()
    for s in (0, 31, 63):
        aa, ab = O.amax(an[s]), O.amax(bn[s])  # the reference quantises each slice on its own
        rows, cols = _sample(512, 14, s + 21), _sample(512, 62, s + 22)
        qa = O.quant(an[s][rows], aa).astype(np.int64)
        qb = O.quant(np.ascontiguousarray(bn[s][:, cols].T), ab).astype(np.int64)
        want = O.epilogue(qa @ qb.T, aa, ab, np.float16)
        assert_bits_equal(y[s][np.ix_(rows, cols)], want, f"bmm slice {s}")


@pytest.mark.parametrize("C,Fo,H,k,pad,bias", [(256, 64, 56, 1, 0, False), (64, 64, 56, 3, 1, False),
                                               (256, 256, 14, 3, 1, True)])
def test_conv_cfg3_batch64(C, Fo, H, k, pad, bias):
    g = torch.Generator().manual_seed(30 + k)
    x = torch.relu(torch.randn(64, C, H, H, generator=g)).half()
    w = (torch.randn(Fo, C, k, k, generator=g) * math.sqrt(2.0 / (C * k * k))).half()
    b = (torch.randn(Fo, generator=g) * 0.01).half() if bias else None
    y = F.conv2d(x.to(DEV), w.to(DEV), None if b is None else b.to(DEV), padding=pad).cpu().numpy()
    xn, wn = x.numpy(), w.numpy()
    ax, aw = O.amax(xn), O.amax(wn)
    qw = O.quant(wn, aw).astype(np.int64).reshape(Fo, -1)
    OH = H + 2 * pad - k + 1
    pix = [(0, 0, 0), (63, OH - 1, OH - 1), (5, 0, OH - 1), (17, OH - 1, 0)]
    rng = np.random.default_rng(31)
    pix += [(int(rng.integers(64)), int(rng.integers(OH)), int(rng.integers(OH))) for _ in range(12)]
    acc = np.zeros((len(pix), Fo), dtype=np.int64)
    for i, (n, oh, ow) in enumerate(pix):
        xp = np.zeros((C, k, k), dtype=np.float16)
        for r in range(k):
            for s in range(k):
                ih, iw = oh - pad + r, ow - pad + s
                if 0 <= ih < H and 0 <= iw < H:
                    xp[:, r, s] = xn[n, :, ih, iw]
        acc[i] = qw @ O.quant(xp, ax).astype(np.int64).reshape(-1)
    want = O.epilogue(acc, ax, aw, np.float16, bias=None if b is None else b.numpy())
    got = np.stack([y[n, :, oh, ow] for (n, oh, ow) in pix])
    assert_bits_equal(got, want, f"conv {C}->{Fo} k{k} @{H}")


def test_sdpa_bert_size_with_padding_mask():
    """cfg4 attention: q, k, v [32, 12, 512, 64] fp16, additive mask with the last 64
    keys masked; whole (batch, head) slices against the oracle composition."""
    g = torch.Generator().manual_seed(40)
    q, k, v = (torch.randn(32, 12, 512, 64, generator=g).half() for _ in range(3))
    mask = torch.zeros(32, 1, 1, 512, dtype=torch.float16)
    mask[..., -64:] = -10000.0
    out = torch_kunlun.kunlun.scaled_dot_product_attention(q.to(DEV), k.to(DEV), v.to(DEV),
                                                           attn_mask=mask.to(DEV)).cpu()
    for bb, hh in ((0, 0), (13, 7), (31, 11)):
        m3 = mask[bb].expand(1, 512, 512).numpy()
        want = O.sdpa(q[bb, hh][None].numpy(), k[bb, hh][None].numpy(), v[bb, hh][None].numpy(),
                      mask=m3, scale=1.0 / math.sqrt(64))[0]
        err = np.abs(out[bb, hh].float().numpy() - want.astype(np.float32)).max()
        assert err <= 2e-2 * max(1.0, float(v[bb, hh].abs().max())), (bb, hh, err)


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_linear_and_mm_against_torch_cpu_within_the_stated_bound(dtype):
    """Against torch's CPU aten (fp32 arithmetic on the same inputs) the
    quantised path stays within max-abs error 2^-10 * max|A| * max|B| * K, for
    fp16 and for fp32 inputs: the cfg1 linear whole, and an mm."""
    g = torch.Generator().manual_seed(50)
    x = torch.randn(2048, 4096, generator=g).to(dtype)
    w = (torch.randn(4096, 4096, generator=g) * 0.02).to(dtype)
    b = (torch.randn(4096, generator=g) * 0.01).to(dtype)
    got = F.linear(x.to(DEV), w.to(DEV), b.to(DEV)).cpu().float()
    ref = F.linear(x.float(), w.float(), b.float())
    bound = 2 ** -10 * x.abs().max().item() * w.abs().max().item() * 4096
    assert (got - ref).abs().max().item() <= bound
    a, c = torch.randn(300, 1000, generator=g).to(dtype), torch.randn(1000, 200, generator=g).to(dtype)
    got = (a.to(DEV) @ c.to(DEV)).cpu().float()
    ref = a.float() @ c.float()
    assert (got - ref).abs().max().item() <= 2 ** -10 * a.abs().max().item() * c.abs().max().item() * 1000
