"""Tensor-parallel SiLU-gated MLP over the ``bkcl`` collectives.

The Llama-style MLP of the benchmark configs: ``down(silu(gate(x)) * up(x))``
with gate/up weights split by output column across ranks and the down weight
split by input row.  Each rank holds x whole, computes its column shard of
the intermediate activation with no communication, multiplies it by its row
shard of the down weight and produces a full-size partial sum; the partials
are summed by an all-reduce (or reduce-scattered by rows).  Every rank
quantises its own shards with their own per-tensor scales, as separate
per-rank linear calls of the reference would.

Overlap: the down projection is computed in row blocks, each block's
all-reduce running on a communication stream while the next block is
computed.  All blocks use the whole activation's and weight's amax, so the
values equal those of one unsplit call.
"""

from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist

from . import _C, kunlun, ops


def _world(group) -> int:
    return dist.get_world_size(group) if dist.is_available() and dist.is_initialized() else 1


def tp_mlp_forward(x: torch.Tensor, w_gate: torch.Tensor, w_up: torch.Tensor,
                   w_down: torch.Tensor, group=None, reduce: str = "allreduce",
                   chunks: int = 4, comm_stream: Optional[kunlun.Stream] = None) -> torch.Tensor:
    """One rank's part of the tensor-parallel MLP.

    x [T, H]; w_gate, w_up [F/P, H] (this rank's output columns, nn.Linear
    layout); w_down [H, F/P] (this rank's input rows).  Returns the summed
    output [T, H] for ``reduce="allreduce"`` or this rank's rows
    [T/P, H] for ``reduce="reduce_scatter"``.
    """
    T, H = x.shape
    ax = _C.amax(x)  # x is quantised once, with one scale, for both gate and up
    gate = _C.linear_scaled(x, w_gate, None, 0, ax, None)
    up = _C.linear_scaled(x, w_up, None, 0, ax, None)
    h = ops.silu_mul(gate, up)
    del gate, up
    ah, aw = _C.amax(h), _C.amax(w_down)
    world = _world(group)
    if world == 1:
        return _C.linear_scaled(h, w_down, None, 0, ah, aw)
    if reduce == "reduce_scatter":
        if T % world:
            raise ValueError("reduce_scatter needs T divisible by the world size")
        partial = _C.linear_scaled(h, w_down, None, 0, ah, aw)
        out = torch.empty(T // world, H, dtype=x.dtype, device=x.device)
        dist.reduce_scatter_tensor(out, partial, group=group)
        return out
    if reduce != "allreduce":
        raise ValueError(f"unknown reduce mode {reduce!r}")
    out = torch.empty(T, H, dtype=x.dtype, device=x.device)
    comm = comm_stream if comm_stream is not None else kunlun.Stream(x.device)
    compute = kunlun.current_stream(x.device)
    chunks = max(1, min(chunks, T))
    bounds = [(i * T // chunks, (i + 1) * T // chunks) for i in range(chunks)]
    for r0, r1 in bounds:
        _C.linear_scaled(h[r0:r1], w_down, None, 0, ah, aw, out[r0:r1])
        ready = kunlun.Event(device=x.device)
        ready.record(compute)
        with kunlun.stream(comm):
            ready.wait(comm)
            dist.all_reduce(out[r0:r1], group=group)
    out.record_stream(comm)
    compute.wait_stream(comm)
    return out


__all__ = ["tp_mlp_forward"]
