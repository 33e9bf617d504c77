"""DistributedDataParallel over the ``bkcl`` ProcessGroup on two GPUs
(reference torch_kunlun/xccl.py:117-213: the DDP subset broadcast /
allreduce / allreduce_coalesced / all_gather with Work objects).

Each rank trains an fp16 MLP on its own batch.  Checked on the device:
- DDP's construction broadcast leaves every rank with rank 0's parameters
  (coalesced broadcast, which needs ``cat`` on the kunlun device);
- each gradient equals fp16(fp16(g_0 / 2) + fp16(g_1 / 2)) bit for bit, g_r being
  rank r's local gradient from the same quantised backward: the reducer's
  multiply-into-bucket (``mul.out`` with a wrapped scalar) and one NCCL sum;
- the parameters stay bit-identical across ranks after the SGD steps, with
  and without ``gradient_as_bucket_view`` (which divides in place, ``div_``)."""
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

torch_kunlun = pytest.importorskip("torch_kunlun")


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _mlp(seed, dev):
    torch.manual_seed(seed)
    return torch.nn.Sequential(torch.nn.Linear(32, 64), torch.nn.ReLU(),
                               torch.nn.Linear(64, 8)).half().to(dev)


def _rank_main(rank, world, port, as_view, q):
    import datetime
    import traceback
    try:
        import torch.distributed as dist
        import torch_kunlun as tk
        tk.kunlun.set_device(rank)
        dist.init_process_group("bkcl", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                                world_size=world, timeout=datetime.timedelta(seconds=60))
        dev = torch.device("kunlun", rank)
        model = _mlp(100 + rank, dev)  # different initial weights on every rank
        ddp = torch.nn.parallel.DistributedDataParallel(model, gradient_as_bucket_view=as_view)
        want0 = _mlp(100, "cpu")
        for p, w in zip(model.parameters(), want0.parameters()):
            assert torch.equal(p.detach().cpu(), w.detach().cpu()), "construction broadcast"
        ref = _mlp(0, dev)  # local (non-DDP) copy for the per-rank gradients
        opt = torch.optim.SGD(model.parameters(), lr=0.05, foreach=False)
        for step in range(3):
            with torch.no_grad():
                for r, p in zip(ref.parameters(), model.parameters()):
                    r.copy_(p)
            g = torch.Generator().manual_seed(10 * step + rank)
            x = torch.randn(16, 32, generator=g).half().to(dev)
            t = torch.randn(16, 8, generator=g).half().to(dev)
            opt.zero_grad()
            torch.nn.functional.mse_loss(ddp(x), t).backward()
            ref.zero_grad()
            torch.nn.functional.mse_loss(ref(x), t).backward()
            for p, r in zip(model.parameters(), ref.parameters()):
                local = r.grad.reshape(-1).contiguous()
                every = torch.empty(world * local.numel(), dtype=local.dtype, device=dev)
                dist.all_gather_into_tensor(every, local)
                parts = every.cpu().float().reshape(world, -1)
                halves = (parts * (1.0 / world)).half().float()
                want = halves.sum(0).half() if world == 2 else None
                got = p.grad.reshape(-1).cpu()
                if want is not None:
                    np.testing.assert_array_equal(got.view(torch.int16).numpy(),
                                                  want.view(torch.int16).numpy(),
                                                  err_msg=f"step {step} gradient")
            opt.step()
        flat = torch.cat([p.detach().reshape(-1) for p in model.parameters()])
        every = torch.empty(world * flat.numel(), dtype=flat.dtype, device=dev)
        dist.all_gather_into_tensor(every, flat)
        e = every.cpu().view(torch.int16).reshape(world, -1)
        assert all(torch.equal(e[0], e[i]) for i in range(world)), "parameters diverged"
        dist.barrier()
        del ddp
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except Exception:
        q.put((rank, traceback.format_exc()[-2000:]))


@pytest.mark.skipif(torch_kunlun.kunlun.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("as_view", [False, True])
def test_ddp_training_over_bkcl_on_two_gpus(as_view):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, as_view, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = {}
    for _ in procs:
        r, msg = q.get(timeout=300)
        results[r] = msg
    for p in procs:
        p.join(timeout=60)
    assert results == {0: "ok", 1: "ok"}, results
