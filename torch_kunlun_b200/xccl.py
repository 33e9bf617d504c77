"""Single-node collectives and the ``bkcl`` torch.distributed ProcessGroup.

Same surface as the reference's torch_kunlun/xccl.py: raw functions
(``get_unique_id``, ``init_rank``, ``all_reduce``, ``broadcast``,
``all_gather``, ``reduce_scatter``, ``barrier``, ``destroy``) and
``ProcessGroupXCCL`` registered as backend ``"bkcl"`` for device ``kunlun``,
exchanging the communicator id through the c10d store
(torch_kunlun/xccl.py:125-138).

Underneath is NCCL over NVLink/NVSwitch (csrc/host/xccl.cpp).  Unlike the
reference, which follows every collective with a global device synchronise
and returns already-completed Work (torch_kunlun/xccl.py:88-114), work here
is enqueued on the caller's current stream and ``Work`` carries a device
event: ``is_completed()`` queries it without blocking, ``wait()`` makes the
current stream wait for it (the host does not block), ``get_future()``
completes once the event has fired.
"""

from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist

from . import _C

UID_KEY = "kunlun_bkcl_uid"


def get_unique_id() -> bytes:
    return _C.xccl_get_unique_id()


def init_rank(rank: int, nranks: int, unique_id: bytes, device: Optional[int] = None) -> None:
    """Create this process's communicator (one per process, single node)."""
    if device is None:
        device = rank
    _C.xccl_init_rank(int(rank), int(nranks), unique_id, int(device))


def destroy() -> None:
    _C.xccl_destroy()


def rank() -> int:
    return int(_C.xccl_rank())


def nranks() -> int:
    return int(_C.xccl_nranks())


def _device_of(tensor: torch.Tensor) -> int:
    if tensor.device.type != "kunlun":
        raise ValueError("xccl requires a kunlun tensor")
    return int(tensor.device.index or 0)


def all_reduce(tensor: torch.Tensor, op: str = "sum") -> None:
    _C.xccl_all_reduce(tensor, op, _device_of(tensor))


def broadcast(tensor: torch.Tensor, root: int) -> None:
    _C.xccl_broadcast(tensor, int(root), _device_of(tensor))


def all_gather(out: torch.Tensor, tensor: torch.Tensor) -> None:
    _C.xccl_all_gather(out, tensor, _device_of(tensor))


def reduce_scatter(out: torch.Tensor, tensor: torch.Tensor, op: str = "sum") -> None:
    _C.xccl_reduce_scatter(out, tensor, op, _device_of(tensor))


def barrier(device: int = 0) -> None:
    _C.xccl_barrier(int(device))


def op_name(op) -> str:
    """torch.distributed.ReduceOp -> the engine's op string."""
    if op == dist.ReduceOp.SUM:
        return "sum"
    if op == dist.ReduceOp.PRODUCT:
        return "prod"
    if op == dist.ReduceOp.MIN:
        return "min"
    if op == dist.ReduceOp.MAX:
        return "max"
    avg = getattr(dist.ReduceOp, "AVG", None)
    if avg is not None and op == avg:
        return "avg"
    raise NotImplementedError(f"unsupported bkcl reduce op: {op}")


class NcclEngine:
    """The device engine: NCCL collectives on the current kunlun stream."""

    def __init__(self, rank: int, size: int, uid: bytes, device: int):
        init_rank(rank, size, uid, device)
        self.device = device

    @staticmethod
    def unique_id() -> bytes:
        return get_unique_id()

    def all_reduce(self, t, op):
        _C.xccl_all_reduce(t, op, _device_of(t))

    def broadcast(self, t, root):
        _C.xccl_broadcast(t, int(root), _device_of(t))

    def all_gather(self, out, inp):
        _C.xccl_all_gather(out, inp, _device_of(inp))

    def reduce_scatter(self, out, inp, op):
        _C.xccl_reduce_scatter(out, inp, op, _device_of(out))

    def barrier(self):
        _C.xccl_barrier(self.device)

    def record(self):
        """An event recorded on the current stream after the enqueued work."""
        from . import kunlun
        ev = kunlun.Event(device=self.device)
        ev.record()
        return ev

    def shutdown(self):
        destroy()


class _XCCLWork(dist.Work):
    """Work backed by a device event recorded after the collective."""

    def __init__(self, event=None, result=None):
        super().__init__()
        self._event = event
        self._result = result

    def wait(self, timeout=None):
        if self._event is not None:
            self._event.wait()  # the current stream waits; the host does not block
        return True

    def is_completed(self) -> bool:
        return self._event is None or self._event.query()

    def is_success(self) -> bool:
        return True

    def synchronize(self):
        if self._event is not None:
            self._event.synchronize()

    def get_future(self):
        self.synchronize()
        fut = torch.futures.Future()
        fut.set_result(self._result)
        return fut


class ProcessGroupXCCL(dist.ProcessGroup):
    """Single-node ``bkcl`` ProcessGroup (DDP subset: broadcast, allreduce,
    allreduce_coalesced, allgather, _allgather_base, reduce_scatter,
    _reduce_scatter_base, barrier).  Rank r drives device r."""

    engine_factory = NcclEngine

    def __init__(self, store, rank: int, size: int, timeout=None, engine_factory=None):
        if store is None:
            raise ValueError("ProcessGroupXCCL requires a c10d Store")
        # torch 2.11 builds Python ProcessGroup subclasses through the
        # (rank, size) constructor; the store is kept for the id exchange.
        super().__init__(int(rank), int(size))
        self._store = store
        self._rank = int(rank)
        self._size = int(size)
        factory = engine_factory or type(self).engine_factory
        if self._rank == 0:
            uid = factory.unique_id()
            store.set(UID_KEY, uid)
        else:
            uid = store.get(UID_KEY)
        self._engine = factory(self._rank, self._size, uid, self._rank)

    def getBackendName(self) -> str:
        return "bkcl"

    def name(self) -> str:
        return "bkcl"

    def getRank(self) -> int:
        return self._rank

    def getSize(self) -> int:
        return self._size

    def rank(self) -> int:
        return self._rank

    def size(self) -> int:
        return self._size

    def _work(self, result=None):
        return _XCCLWork(self._engine.record(), result)

    def broadcast(self, tensors, opts=None):
        if isinstance(tensors, torch.Tensor):
            tensors = [tensors]
        root = int(getattr(opts, "rootRank", 0) if opts is not None else 0)
        for t in tensors:
            self._engine.broadcast(t, root)
        return self._work(tensors)

    def allreduce(self, tensors, opts=None):
        if isinstance(tensors, torch.Tensor):
            tensors = [tensors]
        op = op_name(getattr(opts, "reduceOp", dist.ReduceOp.SUM) if opts is not None
                     else dist.ReduceOp.SUM)
        for t in tensors:
            self._engine.all_reduce(t, op)
        return self._work(tensors)

    def allreduce_coalesced(self, tensors, opts=None):
        return self.allreduce(tensors, opts)

    def _allgather_base(self, output_buffer, input_buffer, opts=None):
        self._engine.all_gather(output_buffer, input_buffer)
        return self._work(output_buffer)

    def allgather(self, output_tensors, input_tensors, opts=None):
        for out_list, inp in zip(output_tensors, input_tensors):
            if len(out_list) != self._size:
                raise ValueError("all_gather output list must have world_size entries")
            flat = torch.empty(inp.numel() * self._size, dtype=inp.dtype, device=inp.device)
            self._engine.all_gather(flat, inp.contiguous())
            for r, out in enumerate(out_list):
                out.copy_(flat.narrow(0, r * inp.numel(), inp.numel()).view_as(out))
        return self._work(output_tensors)

    def _reduce_scatter_base(self, output, input, opts=None):
        op = op_name(getattr(opts, "reduceOp", dist.ReduceOp.SUM) if opts is not None
                     else dist.ReduceOp.SUM)
        self._engine.reduce_scatter(output, input, op)
        return self._work(output)

    def reduce_scatter(self, output_tensors, input_tensors, opts=None):
        op = op_name(getattr(opts, "reduceOp", dist.ReduceOp.SUM) if opts is not None
                     else dist.ReduceOp.SUM)
        outs = output_tensors if isinstance(output_tensors, (list, tuple)) else [output_tensors]
        ins = input_tensors
        if isinstance(ins, (list, tuple)) and ins and isinstance(ins[0], (list, tuple)):
            for out, in_list in zip(outs, ins):
                flat = torch.cat([t.reshape(-1) for t in in_list]) if len(in_list) > 1 else in_list[0]
                self._engine.reduce_scatter(out, flat.contiguous(), op)
        else:
            self._engine.reduce_scatter(outs[0], ins if isinstance(ins, torch.Tensor) else ins[0], op)
        return self._work(outs)

    def barrier(self, opts=None):
        self._engine.barrier()
        return _XCCLWork(None)

    def shutdown(self):
        self._engine.shutdown()


def _create_process_group(store, rank, size, timeout=None):
    return ProcessGroupXCCL(store, rank, size, timeout)


def register_backend() -> None:
    """Register ``bkcl`` with torch.distributed for the ``kunlun`` device."""
    if "bkcl" in dist.Backend.backend_list:
        return
    dist.Backend.register_backend("bkcl", _create_process_group, devices=["kunlun"])


register_backend()
