"""The BERT-shaped encoder block and the pieces it adds to the dense path:
strided copies (head split / merge), linear with a fused residual, and the
whole block against a torch CPU fp32 composition of the same layers."""
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

torch_kunlun = pytest.importorskip("torch_kunlun")
from torch_kunlun_b200 import encoder, ops  # noqa: E402

DEV = "kunlun"


def rnd(shape, seed, scale=1.0, dtype=torch.float16):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(shape, generator=g) * scale).to(dtype)


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32, torch.int64, torch.uint8])
def test_strided_copies_are_exact(dtype):
    base = (torch.arange(2 * 33 * 3 * 4 * 24) % 251).to(dtype)
    x = base.view(2, 33, 3, 4, 24)
    xd = x.to(DEV)
    cases = [
        lambda t: t.permute(2, 0, 3, 1, 4),           # head split of a packed QKV
        lambda t: t[:, :, 1].transpose(1, 2),         # one of the three, heads first
        lambda t: t.transpose(0, 1)[:, :, :, :, ::2],  # non-unit inner stride
        lambda t: t[:, 5:17, :, :, 8:16],             # vectorisable inner block
        lambda t: t[:1, :1].expand(3, 4, 3, 4, 24),   # broadcast source
    ]
    for f in cases:
        got = f(xd).contiguous().cpu()
        assert torch.equal(got, f(x).contiguous())
    # strided destination
    dst = torch.zeros(33, 2, 3, 4, 24, dtype=dtype, device=DEV)
    dst.permute(1, 0, 2, 3, 4).copy_(xd)
    assert torch.equal(dst.cpu(), x.permute(1, 0, 2, 3, 4).contiguous())


def test_linear_residual_equals_linear_then_add():
    x, w, b = rnd((200, 256), 1), rnd((96, 256), 2, 0.02), rnd((96,), 3, 0.02)
    r = rnd((200, 96), 4)
    xd, wd, bd, rd = x.to(DEV), w.to(DEV), b.to(DEV), r.to(DEV)
    fused = ops.linear(xd, wd, bd, residual=rd).cpu()
    unfused = (F.linear(xd, wd, bd) + rd).cpu()
    assert torch.equal(fused.view(torch.int16), unfused.view(torch.int16))


@pytest.mark.parametrize("dtype,M,K,N,act,bias,res,poison", [
    (torch.float16, 200, 256, 96, "gelu", True, False, None),     # folded into the fp16 epilogue
    (torch.float16, 1030, 768, 3072, "gelu", True, False, None),
    (torch.float16, 64, 128, 48, "none", False, True, None),
    (torch.float16, 64, 128, 40, "relu", True, False, None),      # N % 16 != 0: separate pass
    (torch.float32, 77, 96, 64, "none", True, True, None),        # fp32: separate pass
    (torch.float16, 130, 64, 32, "none", True, False, float("inf")),
    (torch.float16, 130, 64, 32, "none", True, False, float("nan")),
])
def test_linear_amax_out_equals_amax_of_output(dtype, M, K, N, act, bias, res, poison):
    x, w = rnd((M, K), 21, dtype=dtype), rnd((N, K), 22, 0.05, dtype=dtype)
    if poison is not None:
        x[M // 2, 3] = poison
    b = rnd((N,), 23, 0.02, dtype=dtype).to(DEV) if bias else None
    r = rnd((M, N), 24, dtype=dtype).to(DEV) if res else None
    xd, wd = x.to(DEV), w.to(DEV)
    a_out = torch.full((1,), -1.0, dtype=torch.float32, device=DEV)
    y = ops.linear(xd, wd, b, act=act, residual=r, amax_out=a_out)
    y_plain = ops.linear(xd, wd, b, act=act, residual=r)
    bits = lambda t: t.cpu().view(torch.int16 if t.element_size() == 2 else torch.int32)
    assert torch.equal(bits(y), bits(y_plain))
    assert torch.equal(bits(a_out), bits(ops.amax(y)))


def test_ffn_scale_handoff_keeps_values():
    h, w1, b1 = rnd((384, 256), 31), rnd((1024, 256), 32, 0.05), rnd((1024,), 33, 0.02)
    w2, b2 = rnd((256, 1024), 34, 0.03), rnd((256,), 35, 0.02)
    hd, w1d, b1d, w2d, b2d = (t.to(DEV) for t in (h, w1, b1, w2, b2))
    a1 = torch.empty(1, dtype=torch.float32, device=DEV)
    f1 = ops.linear(hd, w1d, b1d, act="gelu", amax_out=a1)
    handed = ops.linear(f1, w2d, b2d, residual=hd, amax_x=a1).cpu()
    own = ops.linear(f1, w2d, b2d, residual=hd).cpu()
    assert torch.equal(handed.view(torch.int16), own.view(torch.int16))


def _reference_block(x, w, mask, heads, eps):
    """torch CPU fp32 composition of the same encoder layers."""
    f = {k: v.float() for k, v in vars(w).items()}
    B, L, H = x.shape
    E = H // heads
    x2 = x.float().reshape(B * L, H)
    qkv = F.linear(x2, f["w_qkv"], f["b_qkv"]).view(B, L, 3, heads, E).permute(2, 0, 3, 1, 4)
    ctx = F.scaled_dot_product_attention(qkv[0], qkv[1], qkv[2],
                                         attn_mask=None if mask is None else mask.float())
    ctx = ctx.transpose(1, 2).reshape(B * L, H)
    h = F.layer_norm(x2 + F.linear(ctx, f["w_o"], f["b_o"]), (H,), f["ln1_w"], f["ln1_b"], eps)
    g = F.gelu(F.linear(h, f["w_1"], f["b_1"]))
    y = F.layer_norm(h + F.linear(g, f["w_2"], f["b_2"]), (H,), f["ln2_w"], f["ln2_b"], eps)
    return y.view(B, L, H)


@pytest.mark.parametrize("B,L,H,heads,Fd,tail", [(2, 128, 256, 4, 1024, 16),
                                                (2, 512, 768, 12, 3072, 64)])
def test_encoder_block_matches_fp32_composition(B, L, H, heads, Fd, tail):
    g = torch.Generator().manual_seed(0)
    x = torch.randn(B, L, H, generator=g).half()
    w = encoder.init_weights(H, Fd, generator=g)
    mask = encoder.padding_mask(B, L, tail)
    y = encoder.encoder_block(x.to(DEV), w.to(DEV), mask.to(DEV), heads=heads).cpu()
    ref = _reference_block(x, w, mask, heads, 1e-12)
    assert y.dtype == torch.float16 and y.shape == (B, L, H)
    # fp16 intermediates (the reference rounds every op's output to fp16) and
    # int16 operand quantisation against an fp32 chain: LN outputs are O(1)
    err = (y.float() - ref).abs()
    assert err.max().item() < 6e-2, err.max().item()
    assert err.mean().item() < 4e-3, err.mean().item()
