"""Tensor-parallel SiLU-gated MLP over the ``bkcl`` collectives.

The Llama-style MLP of the benchmark configs: ``down(silu(gate(x)) * up(x))``
with gate/up weights split by output column across ranks and the down weight
split by input row.  Each rank holds x whole, computes its column shard of
the intermediate activation with no communication, multiplies it by its row
shard of the down weight and produces a full-size partial sum; the partials
are summed by an all-reduce (or reduce-scattered by rows).  Every rank
quantises its own shards with their own per-tensor scales, as separate
per-rank linear calls of the reference would.  Each operand is quantised
once per step: x once for both the gate and the up GEMM (one scale, so the
same codes), the down weight once for all of its row blocks.  The SiLU gate
runs in the up projection's epilogue (``T(silu(gate)) * up``, each product
rounded once as the separate swish and mul), which also folds the gated
activation's per-tensor scale, so ``up`` is never stored.

Reductions of the partial sums:

- ``"allreduce"``: the down projection is computed in row blocks, each
  block's all-reduce running on a communication stream while the next block
  is computed.  All blocks use the whole activation's and weight's amax, so
  the values equal those of one unsplit call.
- ``"reduce_scatter"``: one GEMM, then the bkcl reduce-scatter by rows.
- ``"peer"``: receive buffers shared through CUDA IPC; the down projection
  runs one row block (one owner's rows) at a time, starting with the next
  rank's rows, and each finished block is copied into slot r of its owner's
  buffer by copy engines over NVLink (four pieces on four streams, so
  several engines share a block) while the next block computes; the
  owner's own block is computed last, straight into its slot.  After a
  one-element all-reduce as a barrier each rank sums its slots in rank order
  in fp32 and rounds once.  Returns this rank's rows, like
  ``"reduce_scatter"``.
- ``"peer_fused"``: the same exchange from one GEMM whose epilogue stores
  every output tile straight into the owner's buffer over NVLink
  (tk_qgemm_scatter_rows).  Same values as ``"peer"``.
"""

from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist

from . import _C, kunlun, ops


def _world(group) -> int:
    return dist.get_world_size(group) if dist.is_available() and dist.is_initialized() else 1


class PeerRowExchange:
    """Receive buffers for one row-parallel output shape, shared by the ranks
    of one node through CUDA IPC.  Rank q's buffer holds one [rows, cols]
    slot per source rank; rank r's GEMM writes slot r of every owner.  Two
    buffers alternate between calls: a rank may run the next call's GEMM
    while another rank still sums the previous call's slots, and the barrier
    of the call in between keeps the call after that from overwriting them."""

    _count = 0

    def __init__(self, rows: int, cols: int, dtype: torch.dtype, device: torch.device, group=None):
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.group = group
        self.rows, self.cols, self.dtype = rows, cols, dtype
        self.device = int(device.index or 0)
        es = torch.tensor([], dtype=dtype).element_size()
        slot_bytes = rows * cols * es
        store = dist.distributed_c10d._get_default_store()
        PeerRowExchange._count += 1  # the same sequence on every rank
        tag = f"tk_peer_rows/{PeerRowExchange._count}/{rows}x{cols}/{dtype}"
        self._owned, self._opened = [], []
        self.dests, self.local = [], []
        for b in range(2):
            ptr, handle = _C.peer_alloc(self.world * slot_bytes, self.device)
            self._owned.append(ptr)
            store.set(f"{tag}/{b}/{self.rank}", handle)
            self.local.append(_C.tensor_at(ptr, [self.world, rows, cols], dtype, self.device))
        for b in range(2):
            bases = []
            for q in range(self.world):
                if q == self.rank:
                    bases.append(self._owned[b])
                else:
                    peer = _C.peer_open(store.get(f"{tag}/{b}/{q}"), self.device)
                    self._opened.append(peer)
                    bases.append(peer)
            self.dests.append([base + self.rank * slot_bytes for base in bases])
        self.flag = torch.zeros(1, dtype=torch.float32, device=device)
        self._next = 0
        dist.barrier(group=group)  # every rank has opened every buffer

    def forward_fused(self, h: torch.Tensor, w: torch.Tensor, ah: torch.Tensor,
                      aw: torch.Tensor) -> torch.Tensor:
        """h [T, F/P] with its scale ah, the whole row-parallel weight w [H, F/P]."""
        b = self._next
        self._next ^= 1
        _C.linear_scatter_rows(h, w, ah, aw, self.dests[b], self.rows)
        # stream-ordered barrier: every rank's GEMM has stored its slots
        dist.all_reduce(self.flag, group=self.group)
        return _C.sum_slots(self.local[b])

    def forward(self, h: torch.Tensor, wl: torch.Tensor, ah: torch.Tensor, aw: torch.Tensor,
                copy_stream: Optional[kunlun.Stream] = None) -> torch.Tensor:
        """h [T, F/P] with its scale ah; wl the down weight's limbs
        (quantize_limbs with aw), shared by every row block."""
        b = self._next
        self._next ^= 1
        R, P, me = self.rows, self.world, self.rank
        compute = kunlun.current_stream(h.device)
        copies = self._copy_streams(h.device, copy_stream)
        if not hasattr(self, "_stage"):
            self._stage = [torch.empty(R, self.cols, dtype=self.dtype, device=h.device) for _ in range(2)]
            self._stage_free = [None, None]
        es = self._stage[0].element_size()
        k = h.shape[1]
        pieces = len(copies)
        row_bytes = self.cols * es
        for i in range(1, P + 1):
            q = (me + i) % P
            rows = _C.quantize_limbs(h[q * R:(q + 1) * R], ah)
            if q == me:
                _C.linear_from_limbs(rows, wl, k, ah, aw, None, 0, self.local[b][me], h.dtype)
                break
            s = i % 2
            if self._stage_free[s] is not None:
                for ev in self._stage_free[s]:
                    compute.wait_event(ev)
            _C.linear_from_limbs(rows, wl, k, ah, aw, None, 0, self._stage[s], h.dtype)
            done = kunlun.Event(device=h.device)
            done.record(compute)
            freed = []
            for j, cs in enumerate(copies):
                r0, r1 = j * R // pieces, (j + 1) * R // pieces
                with kunlun.stream(cs):
                    cs.wait_event(done)
                    _C.copy_bytes(self.dests[b][q] + r0 * row_bytes, self._stage[s].data_ptr() + r0 * row_bytes,
                                  (r1 - r0) * row_bytes)
                    ev = kunlun.Event(device=h.device)
                    ev.record(cs)
                    freed.append(ev)
            self._stage_free[s] = freed
        for cs in copies:
            compute.wait_stream(cs)
        # stream-ordered barrier: every rank's blocks have landed in their slots
        dist.all_reduce(self.flag, group=self.group)
        return _C.sum_slots(self.local[b])

    def _copy_streams(self, device, first=None):
        if not hasattr(self, "_copies"):
            self._copies = [first if first is not None else kunlun.Stream(device)] + \
                [kunlun.Stream(device) for _ in range(3)]
        return self._copies

    def close(self):
        kunlun.synchronize()
        for p in self._opened:
            _C.peer_release(p)
        self._opened = []
        dist.barrier(group=self.group)  # no rank still maps our buffers
        for p in self._owned:
            _C.peer_release(p)
        self._owned = []


_EXCHANGES = {}


def peer_exchange(rows: int, cols: int, dtype: torch.dtype, device: torch.device, group=None) -> PeerRowExchange:
    key = (rows, cols, dtype, int(device.index or 0), id(group))
    ex = _EXCHANGES.get(key)
    if ex is None:
        ex = _EXCHANGES[key] = PeerRowExchange(rows, cols, dtype, device, group)
    return ex


def release_peer_buffers():
    """Unmap and free every exchange buffer (collective: all ranks call it)."""
    for key in sorted(_EXCHANGES, key=str):
        _EXCHANGES[key].close()
    _EXCHANGES.clear()


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
    dt = x.dtype
    # x: one scale and one quantisation for both column-parallel GEMMs
    ax = _C.amax(x)
    xl = _C.quantize_limbs(x, ax)
    awg, awu = _C.amax(w_gate), _C.amax(w_up)
    gate = _C.linear_from_limbs(xl, _C.quantize_limbs(w_gate, awg), H, ax, awg, None, 0, None, dt)
    wul = _C.quantize_limbs(w_up, awu)
    if dt == torch.float16 and gate.shape[1] % 16 == 0:
        # h = T(silu(gate)) * up and its per-tensor scale from the up
        # projection's epilogue: up itself is never stored
        ah = torch.empty(1, dtype=torch.float32, device=x.device)
        h = _C.linear_from_limbs(xl, wul, H, ax, awu, None, ops.ACT["silu_gate"], None, dt, gate, ah)
        del xl, wul, gate
    else:
        up = _C.linear_from_limbs(xl, wul, H, ax, awu, None, 0, None, dt)
        del xl, wul
        h, ah = _C.silu_mul_amax(gate, up)  # the gate and its per-tensor scale, one pass
        del gate, up
    Fl = h.shape[1]
    aw = _C.amax(w_down)
    world = _world(group)
    if reduce == "peer_fused" and world > 1:
        if T % world:
            raise ValueError("peer reduction needs T divisible by the world size")
        return peer_exchange(T // world, H, dt, x.device, group).forward_fused(h, w_down, ah, aw)
    wl = _C.quantize_limbs(w_down, aw)  # once, for every row block of h
    if world == 1:
        return _C.linear_from_limbs(_C.quantize_limbs(h, ah), wl, Fl, ah, aw, None, 0, None, dt)
    if reduce == "peer":
        if T % world:
            raise ValueError("peer reduction needs T divisible by the world size")
        return peer_exchange(T // world, H, dt, x.device, group).forward(h, wl, ah, aw, comm_stream)
    if reduce == "reduce_scatter":
        if T % world:
            raise ValueError("reduce_scatter needs T divisible by the world size")
        partial = _C.linear_from_limbs(_C.quantize_limbs(h, ah), wl, Fl, ah, aw, None, 0, None, dt)
        out = torch.empty(T // world, H, dtype=dt, device=x.device)
        dist.reduce_scatter_tensor(out, partial, group=group)
        return out
    if reduce != "allreduce":
        raise ValueError(f"unknown reduce mode {reduce!r}")
    out = torch.empty(T, H, dtype=dt, device=x.device)
    comm = comm_stream if comm_stream is not None else kunlun.Stream(x.device)
    compute = kunlun.current_stream(x.device)
    chunks = max(1, min(chunks, T))
    bounds = [(i * T // chunks, (i + 1) * T // chunks) for i in range(chunks)]
    for r0, r1 in bounds:
        _C.linear_from_limbs(_C.quantize_limbs(h[r0:r1], ah), wl, Fl, ah, aw, None, 0, out[r0:r1], dt)
        ready = kunlun.Event(device=x.device)
        ready.record(compute)
        with kunlun.stream(comm):
            ready.wait(comm)
            dist.all_reduce(out[r0:r1], group=group)
    out.record_stream(comm)
    compute.wait_stream(comm)
    return out


__all__ = ["tp_mlp_forward", "PeerRowExchange", "peer_exchange", "release_peer_buffers"]
