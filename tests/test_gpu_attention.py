"""Fused scaled-dot-product attention (tk_sdpa_q16) against the oracle's
restatement of the reference composition (torch_kunlun/kunlun/attention.py:
per-slice quantised q k^T, scale, causal / additive mask, softmax, per-slice
quantised P v) and against the backend's own composed path.

The scores, their roundings and both integer products are exact; softmax is
the one floating-point reduction.  The device's P = T(exp(s - m) * (1/l)) in
binary32 can differ from the oracle's binary64 value by one ulp of T, and
the second product carries that.  Per output element the bound is

    |O_dev - O_oracle| <= Vmax * (2^-9 + S * 2^-24 + S * Pmax / 32767)
                          + 2^-10 * |O| + ulp_T(|O|)

with Vmax = max |v| and Pmax = max P over the slice: sum_j ulp16(P_j) is at
most 2^-10 * sum_j P_j = 2^-10 (plus 2^-24 per subnormal P_j), each of the S
codes of P can round the other way once (Pmax / 32767 each), the slice scale
of P can move by one ulp (the 2^-10 |O| term), and the output rounds once."""
import math

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

torch_kunlun = pytest.importorskip("torch_kunlun")
kunlun = torch_kunlun.kunlun
from oracle import oracle as O  # noqa: E402
from torch_kunlun_b200 import _C  # noqa: E402

DEV = "kunlun"


def rnd(shape, seed, dtype=torch.float16, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(shape, generator=g) * scale).to(dtype)


def oracle_sdpa(q, k, v, mask=None, causal=False, scale=None):
    """q, k, v CPU [B, H, L, E]; mask broadcastable to [B, H, L, S].
    Returns (output [B, H, L, Ev] as fp32, elementwise bound)."""
    B, H, L, E = q.shape
    S, Ev = k.shape[2], v.shape[3]
    m3 = None
    if mask is not None:
        m3 = mask.to(q.dtype).expand(B, H, L, S).reshape(B * H, L, S).numpy()
    vs = v.reshape(B * H, S, Ev).numpy()
    out, p = O.sdpa(q.reshape(B * H, L, E).numpy(), k.reshape(B * H, S, E).numpy(), vs,
                    mask=m3, scale=scale, causal=causal, return_p=True)
    o64 = out.astype(np.float64)
    vmax = np.abs(vs.astype(np.float64)).reshape(B * H, -1).max(1)[:, None, None]
    pmax = np.nan_to_num(p.astype(np.float64)).reshape(B * H, -1).max(1)[:, None, None]
    ulp = (2.0 ** -24 if q.dtype == torch.float16 else 2.0 ** -149) + np.abs(o64) * (
        2.0 ** -10 if q.dtype == torch.float16 else 2.0 ** -23)
    bound = vmax * (2.0 ** -9 + S * 2.0 ** -24 + S * pmax / 32767.0) + 2.0 ** -10 * np.abs(o64) + ulp
    to = lambda a: torch.from_numpy(np.ascontiguousarray(a).astype(np.float32)).reshape(B, H, L, Ev)  # noqa: E731
    return to(out), to(bound)


def check(got, want_and_bound, v=None):
    want, bound = want_and_bound
    err = (got.float() - want).abs()
    bad = err > bound
    assert not bool(bad.any()), (f"{int(bad.sum())} elements beyond the stated bound; "
                                 f"worst excess {float((err - bound).max()):.3g}")


CASES = [
    # B, H, L, S, E, Ev
    (1, 2, 128, 128, 64, 64),
    (2, 3, 100, 77, 40, 24),     # ragged rows, keys and head dims
    (1, 2, 200, 300, 128, 128),  # two limb chunks, two output tiles
    (2, 1, 64, 512, 64, 96),
    (1, 1, 1, 1, 8, 8),
]


@pytest.mark.parametrize("B,H,L,S,E,Ev", CASES)
@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_fused_matches_oracle(B, H, L, S, E, Ev, dtype):
    q, k, v = rnd((B, H, L, E), 1, dtype), rnd((B, H, S, E), 2, dtype), rnd((B, H, S, Ev), 3, dtype)
    out = kunlun.scaled_dot_product_attention(q.to(DEV), k.to(DEV), v.to(DEV)).cpu()
    assert out.shape == (B, H, L, Ev) and out.dtype == dtype
    check(out, oracle_sdpa(q, k, v), v)


def test_fused_bert_size_within_the_stated_bound():
    """BERT-base attention (batch 32, 12 heads, 512 tokens, head dim 64) with
    the additive mask on the last 64 keys, against the oracle composition at
    the bound stated in the module docstring."""
    B, H, L, E = 32, 12, 512, 64
    q, k, v = rnd((B, H, L, E), 31), rnd((B, H, L, E), 32), rnd((B, H, L, E), 33)
    mask = torch.zeros(B, 1, 1, L, dtype=torch.float16)
    mask[..., L - 64:] = -1e4
    out = kunlun.scaled_dot_product_attention(q.to(DEV), k.to(DEV), v.to(DEV), attn_mask=mask.to(DEV)).cpu()
    check(out, oracle_sdpa(q, k, v, mask=mask), v)


@pytest.mark.parametrize("mask_shape", ["2d", "3d_batch", "4d_keys", "4d_full", "bool"])
def test_fused_masks_match_oracle(mask_shape):
    B, H, L, S, E = 2, 3, 96, 160, 64
    q, k, v = rnd((B, H, L, E), 4), rnd((B, H, S, E), 5), rnd((B, H, S, E), 6)
    g = torch.Generator().manual_seed(7)
    if mask_shape == "2d":
        mask = (torch.randn(L, S, generator=g) * 2).half()
    elif mask_shape == "3d_batch":
        mask = (torch.randn(B, L, S, generator=g) * 2).half()
    elif mask_shape == "4d_keys":
        mask = torch.zeros(B, 1, 1, S, dtype=torch.float16)
        mask[..., S - 40:] = -1e4
    elif mask_shape == "4d_full":
        mask = (torch.randn(B, H, L, S, generator=g) * 2).half()
    else:
        mask = torch.rand(L, S, generator=g) < 0.3
    out = kunlun.scaled_dot_product_attention(q.to(DEV), k.to(DEV), v.to(DEV),
                                              attn_mask=mask.to(DEV)).cpu()
    om = mask
    if mask.dtype == torch.bool:
        om = mask.half() * -1e4
    if mask_shape == "3d_batch":
        om = mask.unsqueeze(1)
    check(out, oracle_sdpa(q, k, v, mask=om), v)


def test_fused_causal_scale_and_mask():
    B, H, L, S, E = 1, 4, 130, 130, 64
    q, k, v = rnd((B, H, L, E), 8), rnd((B, H, S, E), 9), rnd((B, H, S, E), 10)
    mask = torch.zeros(B, 1, 1, S, dtype=torch.float16)
    mask[..., :5] = -1e4
    out = kunlun.scaled_dot_product_attention(q.to(DEV), k.to(DEV), v.to(DEV), attn_mask=mask.to(DEV),
                                              is_causal=True, scale=0.3).cpu()
    check(out, oracle_sdpa(q, k, v, mask=mask, causal=True, scale=0.3), v)
    out2 = kunlun.scaled_dot_product_attention(q.to(DEV), k.to(DEV), v.to(DEV), is_causal=True).cpu()
    check(out2, oracle_sdpa(q, k, v, causal=True), v)


def test_fused_equals_composed_path():
    B, H, L, S, E = 2, 4, 256, 256, 64
    q, k, v = rnd((B, H, L, E), 11), rnd((B, H, S, E), 12), rnd((B, H, S, E), 13)
    mask = torch.zeros(B, 1, 1, S, dtype=torch.float16)
    mask[..., S - 32:] = -1e4
    args = (q.to(DEV), k.to(DEV), v.to(DEV), mask.to(DEV), False, None)
    fused = _C.sdpa(*args, fused=True).cpu().float()
    composed = _C.sdpa(*args, fused=False).cpu().float()
    # both are the reference composition; only the softmax sum order differs
    assert (fused - composed).abs().max().item() < 2e-2


@pytest.mark.parametrize("B,H,E,causal,masked", [(2, 3, 64, False, True), (2, 3, 128, False, False),
                                                 (2, 3, 64, True, False), (2, 3, 40, False, True),
                                                 (10, 7, 64, False, True), (9, 8, 128, True, False)])
def test_cluster_kernel_equals_two_kernel_path(B, H, E, causal, masked):
    """Slices of at most 512 queries and keys (fp16) run in one cluster kernel
    that keeps the scores in shared memory; longer slices run the statistics
    and output kernels through HBM.  The two are bit-identical: appending
    copies of query rows 0..127 (and their mask rows) to a 512-query slice
    sends it down the two-kernel path without changing the slice's amax of q
    or its largest probability (a copied row has the same probabilities; with
    a causal mask row 0 already has P = 1), so rows 0..511 must agree bit for
    bit.  70 and 72 slices exceed the clusters that fit on the device at
    once, so each persistent cluster walks several slices."""
    L, S = 512, 448
    q, k, v = rnd((B, H, L, E), 21), rnd((B, H, S, E), 22), rnd((B, H, S, E), 23)
    q2 = torch.cat([q, q[:, :, :128]], dim=2)
    mask = mask2 = None
    if masked:
        mask = (torch.randn(B, 1, L, S, generator=torch.Generator().manual_seed(24)) * 2).half()
        mask[..., S - 64:] = -1e4
        mask2 = torch.cat([mask, mask[:, :, :128]], dim=2)
    one = kunlun.scaled_dot_product_attention(q.to(DEV), k.to(DEV), v.to(DEV),
                                              attn_mask=None if mask is None else mask.to(DEV),
                                              is_causal=causal).cpu()
    two = kunlun.scaled_dot_product_attention(q2.to(DEV), k.to(DEV), v.to(DEV),
                                              attn_mask=None if mask2 is None else mask2.to(DEV),
                                              is_causal=causal).cpu()
    assert torch.equal(one.view(torch.int16), two[:, :, :L].contiguous().view(torch.int16))
    check(one, oracle_sdpa(q, k, v, mask=mask, causal=causal))


def test_fused_reads_strided_head_views():
    """Head-split views of a packed [B, L, 3, H, E] projection give the same
    result as contiguous copies, and the output's heads merge with a view."""
    B, L, H, E = 2, 192, 4, 64
    qkv = rnd((B, L, 3, H, E), 14)
    view = qkv.to(DEV).permute(2, 0, 3, 1, 4)
    out_v = kunlun.scaled_dot_product_attention(view[0], view[1], view[2])
    cont = qkv.permute(2, 0, 3, 1, 4).contiguous()
    out_c = kunlun.scaled_dot_product_attention(cont[0].to(DEV), cont[1].to(DEV), cont[2].to(DEV))
    assert torch.equal(out_v.cpu(), out_c.cpu())
    merged = out_v.transpose(1, 2)
    assert merged.is_contiguous()  # [B, L, H, E] storage: no copy to merge heads
    ref = torch.nn.functional.scaled_dot_product_attention(cont[0].float(), cont[1].float(),
                                                           cont[2].float())
    assert torch.allclose(out_v.cpu().float(), ref, atol=3e-2, rtol=3e-2)


def test_fused_large_magnitudes_and_zero_slice():
    B, H, L, S, E = 1, 2, 64, 64, 32
    q = rnd((B, H, L, E), 15, scale=30.0)
    k = rnd((B, H, S, E), 16, scale=30.0)
    v = rnd((B, H, S, E), 17)
    v[:, 1] = 0.0  # a zero slice: amax 0, quantisation to zero
    out = kunlun.scaled_dot_product_attention(q.to(DEV), k.to(DEV), v.to(DEV)).cpu()
    assert torch.all(out[:, 1] == 0)
    check(out, oracle_sdpa(q, k, v), v)
