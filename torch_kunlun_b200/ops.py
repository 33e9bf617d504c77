"""Fused operators of the kunlun backend that have no single aten name.

* ``linear(x, w, b, act)`` -- act(x @ w^T + b) in one quantised GEMM launch;
  the activation is applied to the rounded, bias-added output, i.e. the same
  values the reference produces with linear followed by a separate
  relu / gelu / silu launch (csrc/ops.cpp:480-495, :151-160,
  csrc/ops_nn.cpp:132-147, csrc/ops_extra.cpp:71).
* ``silu_mul(gate, up)`` -- T(silu(gate)) * up, the gated-MLP product, in one
  elementwise pass.
"""

from __future__ import annotations

from typing import Optional

import torch

from . import _C

ACT = {"none": 0, "relu": 1, "gelu": 2, "gelu_tanh": 3, "silu": 4, "silu_gate": 5}


def linear(x: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor] = None,
           act: str = "none", residual: Optional[torch.Tensor] = None,
           amax_x: Optional[torch.Tensor] = None,
           amax_out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """act(x @ w^T + b) [+ residual]: with a residual the epilogue adds it
    after the bias (rounded to T), giving the values of linear followed by a
    separate add (csrc/ops.cpp:480-495 then csrc/ops.cpp:117-149).

    amax_x (1-element fp32) is x's per-tensor scale when the caller already
    has it (skips the pass over x); amax_out (1-element fp32, written)
    receives max |y| — folded into the fp16 epilogue where it applies, one
    pass over y otherwise — so the GEMM that consumes y skips its own pass.
    """
    return _C.linear_act(x, weight, bias, ACT[act], residual, amax_x, amax_out)


def silu_mul(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    return _C.silu_mul(gate, up)


def amax(x: torch.Tensor) -> torch.Tensor:
    """max |x| as a 1-element fp32 tensor on x's device (the per-tensor scale)."""
    return _C.amax(x)


def linear_scaled(x: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor] = None,
                  act: str = "none", amax_x: Optional[torch.Tensor] = None,
                  amax_w: Optional[torch.Tensor] = None,
                  out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``linear`` with given per-tensor scales; row blocks of x with the whole
    x's amax reproduce one unsplit call exactly."""
    return _C.linear_scaled(x, weight, bias, ACT[act], amax_x, amax_w, out)


def silu_mul_amax(gate: torch.Tensor, up: torch.Tensor):
    """(T(silu(gate)) * up, its max |value| as a 1-element fp32 tensor) in
    one pass: the gated activation and the scale the next GEMM quantises it
    with."""
    return _C.silu_mul_amax(gate, up)


def quantize_limbs(x: torch.Tensor, amax: torch.Tensor) -> torch.Tensor:
    """The int16 codes of a 2-D tensor under a given per-tensor scale, as two
    int8 limb planes [2, rows, round_up(cols, 16)] (hi signed, lo unsigned):
    an operand several GEMMs share is quantised once."""
    return _C.quantize_limbs(x, amax)


def linear_from_limbs(a_limbs: torch.Tensor, b_limbs: torch.Tensor, k: int, amax_a: torch.Tensor,
                      amax_b: torch.Tensor, bias: Optional[torch.Tensor] = None, act: str = "none",
                      out: Optional[torch.Tensor] = None, dtype: torch.dtype = torch.float16,
                      gate: Optional[torch.Tensor] = None,
                      amax_out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """act(a b^T + bias) on operands from quantize_limbs: the values of
    linear_scaled(a, b, amax_x=amax_a, amax_w=amax_b) (K <= 32768).

    act="silu_gate" with `gate` [M, N]: T(silu(gate)) * (a b^T + bias), each
    product rounded once -- silu_mul(gate, up) fused into the up projection.
    amax_out (1-element fp32, written) receives max |y| from the epilogue
    (fp16 outputs on the vector path)."""
    return _C.linear_from_limbs(a_limbs, b_limbs, k, amax_a, amax_b, bias, ACT[act], out, dtype, gate, amax_out)


__all__ = ["linear", "silu_mul", "silu_mul_amax", "amax", "linear_scaled", "quantize_limbs",
           "linear_from_limbs", "ACT"]
