"""The bkcl ProcessGroup's host logic on world-size-2 gloo ranks (CPU, no GPU):
unique-id exchange through the c10d store, ReduceOp mapping, collective
dispatch and Work semantics, with a gloo-backed engine standing in for the
NCCL engine (reference torch_kunlun/xccl.py:117-213)."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


class GlooEngine:
    """Engine with the NcclEngine interface, running gloo on CPU tensors."""
    seen_uid = None

    def __init__(self, rank, size, uid, device):
        GlooEngine.seen_uid = uid
        self.rank, self.size = rank, size

    @staticmethod
    def unique_id():
        return b"uid-" + bytes(range(16))

    def all_reduce(self, t, op):
        ops = {"sum": dist.ReduceOp.SUM, "max": dist.ReduceOp.MAX, "min": dist.ReduceOp.MIN,
               "prod": dist.ReduceOp.PRODUCT}
        dist.all_reduce(t, ops[op], group=_GLOO[0])

    def broadcast(self, t, root):
        dist.broadcast(t, root, group=_GLOO[0])

    def all_gather(self, out, inp):
        dist.all_gather_into_tensor(out, inp, group=_GLOO[0])

    def reduce_scatter(self, out, inp, op):
        chunks = list(inp.chunk(self.size))
        red = torch.stack(chunks).clone()
        dist.all_reduce(red, group=_GLOO[0])
        out.copy_(red[self.rank])

    def barrier(self):
        dist.barrier(group=_GLOO[0])

    def record(self):
        return None

    def shutdown(self):
        pass


_GLOO = [None]


def _worker(rank, world, port, q):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        _GLOO[0] = dist.group.WORLD
        from torch_kunlun_b200 import xccl
        store = dist.TCPStore("127.0.0.1", port + 1, world, rank == 0)
        pg = xccl.ProcessGroupXCCL(store, rank, world, engine_factory=GlooEngine)
        assert pg.getBackendName() == "bkcl" and pg.size() == world and pg.rank() == rank
        assert GlooEngine.seen_uid == b"uid-" + bytes(range(16))  # exchanged via the store
        t = torch.full((4,), float(rank + 1))
        w = pg.allreduce([t])
        assert w.wait() and w.is_completed()
        assert torch.equal(t, torch.full((4,), 3.0))
        opts = dist.AllreduceOptions()
        opts.reduceOp = dist.ReduceOp.MAX
        m = torch.tensor([float(rank)])
        pg.allreduce([m], opts).wait()
        assert m.item() == 1.0
        b = torch.tensor([rank * 10.0])
        bo = dist.BroadcastOptions()
        bo.rootRank = 1
        pg.broadcast([b], bo).wait()
        assert b.item() == 10.0
        g = torch.empty(4)
        pg._allgather_base(g, torch.tensor([rank, rank + 0.5])).wait()
        assert torch.equal(g, torch.tensor([0, 0.5, 1, 1.5]))
        rs = torch.empty(2)
        pg._reduce_scatter_base(rs, torch.arange(4, dtype=torch.float32)).wait()
        assert torch.equal(rs, torch.tensor([0.0, 2.0]) + 4 * rank)
        with pytest.raises(NotImplementedError):
            xccl.op_name(dist.ReduceOp.BAND)
        pg.barrier().wait()
        q.put((rank, "ok"))
    except Exception as e:  # pragma: no cover - reported to the parent
        import traceback
        q.put((rank, traceback.format_exc()[-600:]))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def test_bkcl_process_group_logic_on_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert results == {0: "ok", 1: "ok"}, results


def test_bkcl_backend_registered_for_kunlun():
    import torch_kunlun  # noqa: F401
    assert "bkcl" in dist.Backend.backend_list
    assert dist.Backend.default_device_backend_map.get("kunlun") == "bkcl"


def _ddp_worker(rank, world, port, q):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        _GLOO[0] = dist.group.WORLD
        from torch_kunlun_b200 import xccl
        store = dist.TCPStore("127.0.0.1", port + 1, world, rank == 0)
        pg = xccl.ProcessGroupXCCL(store, rank, world, engine_factory=GlooEngine)
        torch.manual_seed(100 + rank)  # different initial weights on every rank
        model = torch.nn.Sequential(torch.nn.Linear(8, 16), torch.nn.ReLU(), torch.nn.Linear(16, 1))
        ddp = torch.nn.parallel.DistributedDataParallel(model, process_group=pg, bucket_cap_mb=0.0001)
        # construction broadcast rank 0's parameters (coalesced broadcast)
        torch.manual_seed(100)
        want0 = torch.nn.Sequential(torch.nn.Linear(8, 16), torch.nn.ReLU(), torch.nn.Linear(16, 1))
        for p, w in zip(model.parameters(), want0.parameters()):
            assert torch.equal(p.detach(), w.detach())
        ref = [p.detach().clone().requires_grad_() for p in model.parameters()]
        opt = torch.optim.SGD(model.parameters(), lr=0.1)
        for step in range(3):
            g = torch.Generator().manual_seed(10 * step + rank)
            x, t = torch.randn(4, 8, generator=g), torch.randn(4, 1, generator=g)
            opt.zero_grad()
            torch.nn.functional.mse_loss(ddp(x), t).backward()
            # every rank's local gradient, gathered, averaged: DDP's result
            for p in ref:
                p.grad = None
            h = torch.relu(x @ ref[0].t() + ref[1])
            torch.nn.functional.mse_loss(h @ ref[2].t() + ref[3], t).backward()
            for p, r in zip(model.parameters(), ref):
                parts = [torch.empty_like(r.grad) for _ in range(world)]
                dist.all_gather(parts, r.grad, group=_GLOO[0])
                want = sum(parts) / world
                assert torch.allclose(p.grad, want, atol=1e-6, rtol=1e-5), (step, p.grad, want)
            opt.step()
            with torch.no_grad():
                for p, r in zip(model.parameters(), ref):
                    r.copy_(p)
        flat = torch.cat([p.detach().reshape(-1) for p in model.parameters()])
        every = [torch.empty_like(flat) for _ in range(world)]
        dist.all_gather(every, flat, group=_GLOO[0])
        assert all(torch.equal(every[0], e) for e in every)
        q.put((rank, "ok"))
    except Exception:  # pragma: no cover - reported to the parent
        import traceback
        q.put((rank, traceback.format_exc()[-1500:]))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def test_ddp_over_the_bkcl_process_group_on_two_gloo_ranks():
    """DistributedDataParallel driving ProcessGroupXCCL (reference
    torch_kunlun/xccl.py:158-213): the coalesced parameter broadcast at
    construction, per-bucket gradient allreduce through Work futures, and
    identical parameters on every rank after the optimizer steps."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_ddp_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=180) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert results == {0: "ok", 1: "ok"}, results
