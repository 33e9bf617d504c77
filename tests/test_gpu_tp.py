"""Tensor-parallel MLP and the bkcl collectives on the kunlun device.

Single GPU: the row-blocked down projection with the whole activation's scale
equals one unsplit call bit for bit, the TP forward at world size 1 equals
the plain composition, and the last GEMM matches the oracle.  Two GPUs
(skipped with fewer): the bkcl ProcessGroup's collectives on NCCL, and the
TP MLP all-reduce / reduce-scatter against each rank's own partial sums."""
import socket

import numpy as np

import pytest
import torch

pytestmark = pytest.mark.gpu

torch_kunlun = pytest.importorskip("torch_kunlun")
from oracle import oracle as O  # noqa: E402
from tests._qgemm_helpers import assert_bits_equal  # noqa: E402
from torch_kunlun_b200 import ops, tp  # noqa: E402

DEV = "kunlun"


def rnd(shape, seed, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(shape, generator=g) * scale).half()


def test_row_blocks_with_shared_scales_equal_one_call():
    x, w = rnd((300, 256), 1).to(DEV), rnd((96, 256), 2, 0.02).to(DEV)
    full = torch.nn.functional.linear(x, w)
    ax, aw = ops.amax(x), ops.amax(w)
    out = torch.empty(300, 96, dtype=torch.float16, device=DEV)
    for r0, r1 in [(0, 77), (77, 128), (128, 300)]:
        ops.linear_scaled(x[r0:r1], w, amax_x=ax, amax_w=aw, out=out[r0:r1])
    assert torch.equal(out.cpu().view(torch.int16), full.cpu().view(torch.int16))
    assert ops.amax(x).cpu().item() == float(O.amax(x.cpu().numpy()))


@pytest.mark.parametrize("M,K,N,bias", [(300, 256, 384, False), (130, 768, 96, True),
                                        (256, 2048, 320, False), (64, 4096, 160, True)])
def test_silu_gate_epilogue_equals_separate_gate(M, K, N, bias):
    """silu_mul(gate, up) fused into the up projection's epilogue: the same
    bits, and max |h| from the epilogue equals the separate pass's (128x128
    tiles for K < 2048, 128x160 above)."""
    x, wg, wu = rnd((M, K), 11).to(DEV), rnd((N, K), 12, 0.05).to(DEV), rnd((N, K), 13, 0.05).to(DEV)
    b = rnd((N,), 14, 0.1).to(DEV) if bias else None
    ax, awg, awu = ops.amax(x), ops.amax(wg), ops.amax(wu)
    xl, wgl, wul = ops.quantize_limbs(x, ax), ops.quantize_limbs(wg, awg), ops.quantize_limbs(wu, awu)
    gate = ops.linear_from_limbs(xl, wgl, K, ax, awg)
    up = ops.linear_from_limbs(xl, wul, K, ax, awu, bias=b)
    h_ref, ah_ref = ops.silu_mul_amax(gate, up)
    ah = torch.full((1,), -1.0, dtype=torch.float32, device=DEV)
    h = ops.linear_from_limbs(xl, wul, K, ax, awu, bias=b, act="silu_gate", gate=gate, amax_out=ah)
    assert torch.equal(h.cpu().view(torch.int16), h_ref.cpu().view(torch.int16))
    assert torch.equal(ah.cpu().view(torch.int32), ah_ref.cpu().view(torch.int32))


def test_silu_gate_epilogue_rejects_unsupported_forms():
    x, w = rnd((64, 256), 15).to(DEV), rnd((40, 256), 16, 0.05).to(DEV)  # N % 16 != 0
    ax, aw = ops.amax(x), ops.amax(w)
    xl, wl = ops.quantize_limbs(x, ax), ops.quantize_limbs(w, aw)
    gate = torch.zeros(64, 40, dtype=torch.float16, device=DEV)
    with pytest.raises(RuntimeError):
        ops.linear_from_limbs(xl, wl, 256, ax, aw, act="silu_gate", gate=gate)
    with pytest.raises(RuntimeError):  # the gate operand is required
        ops.linear_from_limbs(xl, wl, 256, ax, aw, act="silu_gate")


def test_tp_mlp_world1_matches_composition_and_oracle():
    T, H, F = 256, 128, 384
    x = rnd((T, H), 3).to(DEV)
    wg, wu = rnd((F, H), 4, 0.02).to(DEV), rnd((F, H), 5, 0.02).to(DEV)
    wd = rnd((H, F), 6, 0.02).to(DEV)
    y = tp.tp_mlp_forward(x, wg, wu, wd)
    gate = torch.nn.functional.linear(x, wg)
    up = torch.nn.functional.linear(x, wu)
    h = ops.silu_mul(gate, up)
    ref = torch.nn.functional.linear(h, wd)
    assert torch.equal(y.cpu().view(torch.int16), ref.cpu().view(torch.int16))
    # gate/up and the down projection are bit-exact against the oracle; the
    # SiLU gate is checked at fp16 tolerance
    assert_bits_equal(gate.cpu().numpy(), O.linear(x.cpu().numpy(), wg.cpu().numpy()), "gate")
    g64, u64 = gate.cpu().double(), up.cpu().double()
    silu_ref = (g64 / (1 + torch.exp(-g64))).half().double() * u64
    assert torch.allclose(h.cpu().double(), silu_ref, atol=1e-3, rtol=2e-3)
    assert_bits_equal(y.cpu().numpy(), O.linear(h.cpu().numpy(), wd.cpu().numpy()), "down")


def test_fused_silu_gate_amax_and_limb_gemms_equal_the_plain_ops():
    """The TP step's building blocks: silu_mul_amax equals silu_mul then amax
    (bit for bit, NaN-free); a GEMM on operands quantised once by
    quantize_limbs equals linear_scaled with the same scales, also on a row
    block written into a slice of a larger output."""
    g, u = rnd((300, 520), 20), rnd((300, 520), 21)
    gd, ud = g.to(DEV), u.to(DEV)
    h, ah = ops.silu_mul_amax(gd, ud)
    assert torch.equal(h.cpu().view(torch.int16), ops.silu_mul(gd, ud).cpu().view(torch.int16))
    assert ah.cpu().item() == ops.amax(h).cpu().item()
    gh, uh = rnd((301, 520), 22), rnd((301, 520), 23)  # odd count: the element-wise path
    h2, ah2 = ops.silu_mul_amax(gh.to(DEV), uh.to(DEV))
    assert ah2.cpu().item() == float(np.abs(h2.cpu().float().numpy()).max())
    w = rnd((200, 520), 24, 0.02).to(DEV)
    aw = ops.amax(w)
    hl, wl = ops.quantize_limbs(h, ah), ops.quantize_limbs(w, aw)
    got = ops.linear_from_limbs(hl, wl, 520, ah, aw)
    want = ops.linear_scaled(h, w, amax_x=ah, amax_w=aw)
    assert torch.equal(got.cpu().view(torch.int16), want.cpu().view(torch.int16))
    out = torch.zeros(400, 200, dtype=torch.float16, device=DEV)
    ops.linear_from_limbs(ops.quantize_limbs(h[100:250], ah), wl, 520, ah, aw, out=out[50:200])
    assert torch.equal(out[50:200].cpu().view(torch.int16), want[100:250].cpu().view(torch.int16))
    assert_bits_equal(got.cpu().numpy(), O.linear(h.cpu().numpy(), w.cpu().numpy()), "from limbs")


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank_main(rank, world, port, q):
    import datetime
    import traceback
    try:
        import torch.distributed as dist
        import torch_kunlun as tk  # noqa: F401
        tk.kunlun.set_device(rank)
        dist.init_process_group("bkcl", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                                world_size=world, timeout=datetime.timedelta(seconds=60))
        dev = torch.device("kunlun", rank)
        t = torch.full((1000,), float(rank + 1), dtype=torch.float16, device=dev)
        dist.all_reduce(t)
        assert torch.all(t.cpu() == sum(range(1, world + 1)))
        b = torch.full((16,), float(rank * 7), dtype=torch.float32, device=dev)
        dist.broadcast(b, src=1)
        assert torch.all(b.cpu() == 7.0)
        g = torch.empty(4 * world, dtype=torch.float32, device=dev)
        dist.all_gather_into_tensor(g, torch.full((4,), float(rank), device=dev))
        assert torch.equal(g.cpu(), torch.arange(world).repeat_interleave(4).float())
        rs = torch.empty(8, dtype=torch.float32, device=dev)
        dist.reduce_scatter_tensor(rs, torch.arange(8 * world, dtype=torch.float32).to(dev))
        assert torch.equal(rs.cpu(), (torch.arange(8) + 8 * rank).float() * world)
        # tensor-parallel MLP: the same full weights on every rank, sharded
        T, H, F = 512, 256, 1024
        x = rnd((T, H), 10).to(dev)
        wg, wu, wd = rnd((F, H), 11, 0.02), rnd((F, H), 12, 0.02), rnd((H, F), 13, 0.02)
        f0, f1 = rank * F // world, (rank + 1) * F // world
        wgs, wus = wg[f0:f1].contiguous().to(dev), wu[f0:f1].contiguous().to(dev)
        wds = wd[:, f0:f1].contiguous().to(dev)
        # this rank's partial, computed locally without communication
        ax = ops.amax(x)
        h = ops.silu_mul(ops.linear_scaled(x, wgs, amax_x=ax), ops.linear_scaled(x, wus, amax_x=ax))
        partial = torch.nn.functional.linear(h, wds)
        parts = torch.empty(world * T, H, dtype=torch.float16, device=dev)
        dist.all_gather_into_tensor(parts, partial)
        p = parts.cpu().float().reshape(world, T, H)
        want = p.sum(0)
        y = tp.tp_mlp_forward(x, wgs, wus, wds, reduce="allreduce", chunks=4)
        assert torch.allclose(y.cpu().float(), want, atol=1e-3, rtol=2 ** -9)
        ys = tp.tp_mlp_forward(x, wgs, wus, wds, reduce="reduce_scatter")
        rows = want[rank * T // world:(rank + 1) * T // world]
        assert torch.allclose(ys.cpu().float(), rows, atol=1e-3, rtol=2 ** -9)
        # peer reduction: every rank's partial stored into the owner's buffer by
        # the GEMM epilogue over NVLink, summed in rank order in fp32, one rounding
        mine = p[:, rank * T // world:(rank + 1) * T // world]
        acc = torch.zeros_like(mine[0])
        for r in range(world):
            acc = acc + mine[r]
        want_peer = acc.half()
        for mode in ("peer", "peer_fused", "peer"):  # both alternating buffers, and reuse
            yp = tp.tp_mlp_forward(x, wgs, wus, wds, reduce=mode)
            assert torch.equal(yp.cpu().view(torch.int16), want_peer.view(torch.int16)), mode
        if world == 2:  # one add of two binary16 values: NCCL's sum rounds the same way
            assert torch.equal(yp.cpu().view(torch.int16), ys.cpu().view(torch.int16))
        tp.release_peer_buffers()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except Exception:
        q.put((rank, traceback.format_exc()[-1500:]))


@pytest.mark.skipif(torch_kunlun.kunlun.device_count() < 2, reason="needs 2 GPUs")
def test_bkcl_collectives_and_tp_mlp_on_two_gpus():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = {}
    for _ in procs:
        r, msg = q.get(timeout=300)
        results[r] = msg
    for p in procs:
        p.join(timeout=60)
    assert results == {0: "ok", 1: "ok"}, results
