"""BERT-base-shaped post-LayerNorm encoder block on the kunlun device.

The block is the reference's dense hot path strung together the way a
transformer encoder uses it: the QKV / output / FFN linears go through the
int16-quantised GEMM (csrc/ops.cpp:210-230, :480-495), attention through the
backend's scaled_dot_product_attention (torch_kunlun/kunlun/attention.py:36-107),
the two post-LayerNorms through layer_norm (csrc/ops_nn.cpp:85-130) and the
FFN activation through gelu (csrc/ops_nn.cpp:132-147).

Fusions keep the reference's values: the bias, the residual add and gelu are
applied in the GEMM epilogue in the reference's order (linear rounds to T,
then the bias add, then the residual add, then gelu, each rounded to T), so
the block's values equal the unfused sequence linear -> add -> add / gelu.
The Q, K and V heads are strided views of the QKV projection (no copies), and
the attention output is read back as [tokens, hidden] through a view.  The
FFN1 GEMM hands max |f1| (the per-tensor scale FFN2 quantises f1 with) out of
its epilogue, so FFN2 does not read f1 an extra time for it.
"""

from __future__ import annotations

from dataclasses import dataclass, fields
from typing import Optional

import torch
import torch.nn.functional as F

from . import ops
from .kunlun.attention import scaled_dot_product_attention


@dataclass
class EncoderWeights:
    w_qkv: torch.Tensor   # [3H, H]: rows 0..H-1 query, H..2H-1 key, 2H.. value
    b_qkv: torch.Tensor   # [3H]
    w_o: torch.Tensor     # [H, H]
    b_o: torch.Tensor     # [H]
    ln1_w: torch.Tensor   # [H]
    ln1_b: torch.Tensor   # [H]
    w_1: torch.Tensor     # [F, H]
    b_1: torch.Tensor     # [F]
    w_2: torch.Tensor     # [H, F]
    b_2: torch.Tensor     # [H]
    ln2_w: torch.Tensor   # [H]
    ln2_b: torch.Tensor   # [H]

    def to(self, *args, **kwargs) -> "EncoderWeights":
        return EncoderWeights(**{f.name: getattr(self, f.name).to(*args, **kwargs)
                                 for f in fields(self)})


def init_weights(hidden: int = 768, ffn: int = 3072, std: float = 0.02,
                 dtype: torch.dtype = torch.float16,
                 generator: Optional[torch.Generator] = None) -> EncoderWeights:
    """Random weights on the CPU: linear weights and biases ~N(0, std),
    LayerNorm gamma 1 and beta 0.  Drawn in fp32 in field order, then cast."""
    def n(*shape):
        return (torch.randn(*shape, generator=generator) * std).to(dtype)
    H, Fd = hidden, ffn
    return EncoderWeights(
        w_qkv=n(3 * H, H), b_qkv=n(3 * H), w_o=n(H, H), b_o=n(H),
        ln1_w=torch.ones(H, dtype=dtype), ln1_b=torch.zeros(H, dtype=dtype),
        w_1=n(Fd, H), b_1=n(Fd), w_2=n(H, Fd), b_2=n(H),
        ln2_w=torch.ones(H, dtype=dtype), ln2_b=torch.zeros(H, dtype=dtype))


def padding_mask(batch: int, seq: int, masked_tail: int, dtype: torch.dtype = torch.float16,
                 value: float = -1.0e4) -> torch.Tensor:
    """Additive attention mask [batch, 1, 1, seq]: `value` on the last
    `masked_tail` key positions of every row, 0 elsewhere."""
    m = torch.zeros(batch, 1, 1, seq, dtype=dtype)
    if masked_tail > 0:
        m[..., seq - masked_tail:] = value
    return m


def encoder_block(x: torch.Tensor, w: EncoderWeights, mask: Optional[torch.Tensor] = None,
                  heads: int = 12, eps: float = 1e-12) -> torch.Tensor:
    """y = LN2(h + FFN(h)), h = LN1(x + Attn(x)) for x [B, L, H] on kunlun."""
    B, L, H = x.shape
    E = H // heads
    x2 = x.reshape(B * L, H)
    qkv = ops.linear(x2, w.w_qkv, w.b_qkv)                        # [B*L, 3H]
    qkv = qkv.view(B, L, 3, heads, E).permute(2, 0, 3, 1, 4)      # [3, B, heads, L, E] view
    ctx = scaled_dot_product_attention(qkv[0], qkv[1], qkv[2], attn_mask=mask)
    ctx = ctx.transpose(1, 2).reshape(B * L, H)
    a = ops.linear(ctx, w.w_o, w.b_o, residual=x2)                # x + attn_out
    h = F.layer_norm(a, (H,), w.ln1_w, w.ln1_b, eps)
    a1 = torch.empty(1, dtype=torch.float32, device=x.device)
    f1 = ops.linear(h, w.w_1, w.b_1, act="gelu", amax_out=a1)     # a1 = max |f1|
    f2 = ops.linear(f1, w.w_2, w.b_2, residual=h, amax_x=a1)      # h + ffn_out
    y = F.layer_norm(f2, (H,), w.ln2_w, w.ln2_b, eps)
    return y.view(B, L, H)


def encoder_block_macs(batch: int, seq: int, hidden: int = 768, ffn: int = 3072) -> int:
    """Multiply-accumulates of one block: QKV, output and FFN linears plus
    the two attention products."""
    T = batch * seq
    return T * hidden * (3 * hidden + hidden + 2 * ffn) + 2 * batch * seq * seq * hidden


__all__ = ["EncoderWeights", "init_weights", "padding_mask", "encoder_block",
           "encoder_block_macs"]
