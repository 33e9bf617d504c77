"""The reference's 1-D and broadcast matmul cases (tests/test_extra_ops.py:
216-245: (4,)x(4,), (4,)x(4,3), (2,3,4)x(4,), (2,1,3,4)x(5,4,2) and an einsum,
forward and backward) on the device.  The reference stages these through the
CPU (csrc/linalg_extra.cpp:232-236); here they run in a child process with
KUNLUN_CPU_FALLBACK=error, so any host staging or CPU fallback fails the
test, and every value is compared bit for bit with the oracle's quantised
products (each operand of each product one per-tensor scale, as torch's
decomposition onto dot / mv / mm / bmm hands them to the backend)."""
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CHILD = r"""
import sys
sys.path.insert(0, ROOT)
import numpy as np
import torch
import torch_kunlun  # noqa: F401
from oracle import oracle as O

def bits(a):
    return np.ascontiguousarray(np.asarray(a, dtype=np.float16)).view(np.uint16)

def same(got, want, what):
    g, w = bits(got), bits(want)
    assert g.shape == w.shape, (what, g.shape, w.shape)
    assert np.array_equal(g, w), (what, np.asarray(got), np.asarray(want))

def run(a, b, fn):
    ak = a.to("kunlun").requires_grad_()
    bk = b.to("kunlun").requires_grad_()
    c = fn(ak, bk)
    c.backward(torch.ones(c.shape, dtype=c.dtype).to("kunlun"))
    torch_kunlun.kunlun.synchronize()
    return c.detach().cpu().numpy(), ak.grad.cpu().numpy(), bk.grad.cpu().numpy()

def f16sum(parts, axis):
    # the backend's sum: fp32 accumulation, one rounding (exact here: a few fp16 terms)
    return parts.astype(np.float64).sum(axis).astype(np.float16)

g = torch.Generator().manual_seed(0)
rn = lambda *s: torch.randn(*s, generator=g).half()
ones = lambda *s: np.ones(s, dtype=np.float16)

# (4,) x (4,): dot; grads are other * 1
a, b = rn(4), rn(4)
c, ga, gb = run(a, b, torch.matmul)
an, bn = a.numpy(), b.numpy()
same(c, O.mm(an[None], bn[:, None])[0, 0], "dot")
same(ga, bn, "dot grad a")
same(gb, an, "dot grad b")

# (4,) x (4,3): unsqueeze(0).mm(b).squeeze_(0)
a, b = rn(4), rn(4, 3)
c, ga, gb = run(a, b, torch.matmul)
an, bn = a.numpy(), b.numpy()
same(c, O.mm(an[None], bn)[0], "vec @ mat")
same(ga, O.mm(ones(1, 3), np.ascontiguousarray(bn.T))[0], "vec @ mat grad a")
same(gb, O.mm(an[:, None], ones(1, 3)), "vec @ mat grad b")

# (2,3,4) x (4,): folded to (6,4).mv(b); mv's grads: grad outer b, a^T mv grad
a, b = rn(2, 3, 4), rn(4)
c, ga, gb = run(a, b, torch.matmul)
an, bn = a.numpy(), b.numpy()
a2 = an.reshape(6, 4)
same(c, O.mm(a2, bn[:, None])[:, 0].reshape(2, 3), "batched mat @ vec")
same(ga, np.broadcast_to(bn, (2, 3, 4)), "batched mat @ vec grad a")
same(gb, O.mm(np.ascontiguousarray(a2.T), ones(6, 1))[:, 0], "batched mat @ vec grad b")

# (2,1,3,4) x (5,4,2): batch dims broadcast to (2,5) -> bmm over 10 slices
a, b = rn(2, 1, 3, 4), rn(5, 4, 2)
c, ga, gb = run(a, b, torch.matmul)
an, bn = a.numpy(), b.numpy()
A = np.broadcast_to(an, (2, 5, 3, 4)).reshape(10, 3, 4)
B = np.broadcast_to(bn, (2, 5, 4, 2)).reshape(10, 4, 2)
same(c, O.bmm(np.ascontiguousarray(A), np.ascontiguousarray(B)).reshape(2, 5, 3, 2), "broadcast bmm")
gA = O.bmm(ones(10, 3, 2), np.ascontiguousarray(np.swapaxes(B, 1, 2))).reshape(2, 5, 3, 4)
same(ga, f16sum(gA, 1)[:, None], "broadcast bmm grad a")
gB = O.bmm(np.ascontiguousarray(np.swapaxes(A, 1, 2)), ones(10, 3, 2)).reshape(2, 5, 4, 2)
same(gb, f16sum(gB, 0), "broadcast bmm grad b")

# einsum ij,jk->ik: mm
a, b = rn(2, 3), rn(3, 4)
c, ga, gb = run(a, b, lambda x, y: torch.einsum("ij,jk->ik", x, y))
an, bn = a.numpy(), b.numpy()
same(c, O.mm(an, bn), "einsum")
same(ga, O.mm(ones(2, 4), np.ascontiguousarray(bn.T)), "einsum grad a")
same(gb, O.mm(np.ascontiguousarray(an.T), ones(2, 4)), "einsum grad b")
print("ok")
""".replace("ROOT", repr(ROOT))


def test_reference_1d_and_broadcast_matmul_stay_on_device_bit_exact():
    env = dict(os.environ, KUNLUN_CPU_FALLBACK="error")
    r = subprocess.run([sys.executable, "-c", CHILD], env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0 and r.stdout.strip().endswith("ok"), r.stdout[-3000:] + r.stderr[-3000:]
