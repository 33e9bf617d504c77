"""CPU tests of the oracle: IEEE helpers, known-answer cases, and the exact
float64 GEMM shortcut against the scalar int64 loop."""
import numpy as np
import pytest

from oracle import oracle as O


def test_f64_to_f16_matches_numpy_rounding():
    rng = np.random.default_rng(1)
    vals = np.concatenate([
        rng.standard_normal(20000) * 10.0 ** rng.integers(-9, 6, 20000),
        np.array([0.0, -0.0, 65504.0, 65519.99, 65520.0, 1e10, -1e10, 2.0 ** -24,
                  2.0 ** -25, 2.0 ** -25 * 1.0000001, 3 * 2.0 ** -26, 6.1e-5,
                  np.inf, -np.inf, 1.0 + 2.0 ** -11, 1.0 + 3 * 2.0 ** -11,
                  2049.0, 2051.0, -2.0 ** -14 * 0.999]),
    ])
    # Halfway cases between adjacent fp16 values (exact in float64).
    h = rng.integers(0, 0x7BFF, 5000).astype(np.uint16).view(np.float16).astype(np.float64)
    h2 = (rng.integers(0, 0x7BFF, 5000).astype(np.uint16) + 1).view(np.float16).astype(np.float64)
    vals = np.concatenate([vals, (h + np.nextafter(h, np.inf)) / 2, h2])
    ours = np.array([O.f64_to_f16_bits(v) for v in vals], dtype=np.uint16)
    ref = vals.astype(np.float16).view(np.uint16)
    assert np.array_equal(ours, ref)


def test_limbs_recombine():
    q = np.arange(-32767, 32768, dtype=np.int16)
    hi, lo = O.limbs(q)
    assert hi.min() == -128 and hi.max() == 127 and lo.min() == 0 and lo.max() == 255
    assert np.array_equal(hi.astype(np.int32) * 256 + lo.astype(np.int32), q.astype(np.int32))


def test_quant_known_answers():
    x = np.array([1.0, -1.0, 0.5, 0.0, 1.0 / 65534.0, 3.0 / 65534.0], dtype=np.float32)
    q = O.quant(x)
    assert q[0] == 32767 and q[1] == -32767 and q[3] == 0
    assert q[2] == 16384  # 0.5 * 32767 = 16383.5 -> ties to even
    assert q[4] == 0      # 0.49999... -> 0 ; exact half rounds to even
    assert q[5] == 2      # 1.5 -> 2
    assert np.all(O.quant(np.zeros(8, np.float16)) == 0)


def test_amax_nan_dominates_and_zero():
    x = np.array([1.0, np.nan, -3.0], dtype=np.float32)
    assert np.isnan(O.amax(x))
    assert O.amax(np.array([-0.0, 0.0], np.float32)) == 0.0
    assert O.amax(np.array([-7.5, 2.0], np.float16)) == np.float32(7.5)


def test_fc_fp32_probe_value():
    # Row [1e-5, 1] times column [1, 1e5]: the small term is lost to the
    # per-tensor int16 scale and the result is exactly 1e5 in fp32.
    x = np.array([[1e-5, 1.0]], dtype=np.float32)
    w = np.array([[1.0], [1e5]], dtype=np.float32)
    y, acc, ax, aw = O.fc(x, w, w_trans=False)
    assert acc[0, 0] == 32767 * 32767
    assert y[0, 0] == np.float32(1e5)


def test_fc_all_equal_and_single_element():
    K = 37
    x = np.full((3, K), 0.75, np.float16)
    w = np.full((5, K), -2.0, np.float16)
    y, acc, _, _ = O.fc(x, w, w_trans=True)
    assert np.all(acc == -K * 32767 * 32767)
    assert np.all(y == np.float16(-0.75 * 2.0 * K))
    x = np.zeros((4, 4), np.float16); x[2, 1] = 3.0
    w = np.zeros((4, 4), np.float16); w[1, 3] = -0.5
    y = O.mm(x, w)
    expect = np.zeros((4, 4), np.float16); expect[2, 3] = -1.5
    assert np.array_equal(y, expect)


def test_fc_zero_operand_and_nonfinite():
    x = np.random.default_rng(0).standard_normal((4, 8)).astype(np.float16)
    assert np.all(O.linear(x, np.zeros((3, 8), np.float16)) == 0)
    w = np.ones((3, 8), np.float16); w[0, 0] = np.inf
    assert np.all(np.isnan(O.linear(x, w)))


def test_exact_shortcut_matches_scalar_loop():
    rng = np.random.default_rng(2)
    for (M, K, N) in [(1, 1, 1), (7, 129, 5), (33, 300, 17)]:
        qa = rng.integers(-32767, 32768, (M, K)).astype(np.int16)
        qb = rng.integers(-32767, 32768, (K, N)).astype(np.int16)
        qa[0, :] = 32767; qb[:, 0] = 32767  # extreme accumulations
        assert np.array_equal(O.gemm_i16_exact(qa, qb), O.gemm_i16_scalar(qa, qb))


def test_fc_matches_torch_cpu_within_reference_tolerance():
    # tests/test_numeric_semantics.py:49-57 of the reference: fp16 mm rel-L2 < 5e-3.
    rng = np.random.default_rng(0)
    x = rng.standard_normal((64, 128)).astype(np.float16)
    w = rng.standard_normal((128, 64)).astype(np.float16)
    exact = x.astype(np.float64) @ w.astype(np.float64)
    out = O.mm(x, w).astype(np.float64)
    rel = np.linalg.norm(out - exact) / np.linalg.norm(exact)
    assert rel < 5e-3


def test_epilogue_order_bias_after_rounding():
    acc = np.array([[12345678901]], dtype=np.int64)
    y0 = O.epilogue(acc, 1.0, 1.0, np.float16)
    yb = O.epilogue(acc, 1.0, 1.0, np.float16, bias=np.array([0.3], np.float16))
    step = np.float16(np.float32(y0[0, 0]) + np.float32(np.float16(0.3)))
    assert yb[0, 0] == step


def test_conv_fast_matches_scalar():
    rng = np.random.default_rng(3)
    x = np.maximum(rng.standard_normal((2, 6, 9, 7)), 0).astype(np.float16)
    for (F, KH, stride, pad, dil, groups) in [(4, 3, (1, 1), (1, 1), (1, 1), 1),
                                              (6, 3, (2, 1), (0, 2), (1, 2), 3),
                                              (6, 1, (1, 1), (0, 0), (1, 1), 6)]:
        w = rng.standard_normal((F, 6 // groups, KH, KH)).astype(np.float16)
        qx, qw = O.quant(x), O.quant(w)
        a = O.conv2d_acc(qx, qw, stride, pad, dil, groups, scalar=False)
        b = O.conv2d_acc(qx, qw, stride, pad, dil, groups, scalar=True)
        assert np.array_equal(a, b)


def test_nd_and_transposed_conv_accumulators_match_exact_float64_convs():
    """The oracle's N-d gather and its scatter definition of the transposed
    convolution against torch's CPU float64 convolutions of the same integer
    codes (exact: every partial sum is an integer below 2^53)."""
    import torch
    import torch.nn.functional as F
    rng = np.random.default_rng(7)
    x = rng.standard_normal((2, 4, 5, 6, 7)).astype(np.float16)
    w = rng.standard_normal((6, 2, 2, 3, 2)).astype(np.float16)
    qx, qw = O.quant(x), O.quant(w)
    want = F.conv3d(torch.tensor(qx, dtype=torch.float64), torch.tensor(qw, dtype=torch.float64),
                    stride=(1, 2, 1), padding=(1, 0, 1), dilation=(2, 1, 1), groups=2).numpy()
    assert np.array_equal(O.convnd_acc(qx, qw, (1, 2, 1), (1, 0, 1), (2, 1, 1), 2), want.astype(np.int64))
    x2 = rng.standard_normal((2, 4, 7, 6)).astype(np.float16)
    q2 = O.quant(x2)
    w2 = O.quant(rng.standard_normal((6, 2, 3, 3)).astype(np.float16))
    assert np.array_equal(O.convnd_acc(q2, w2, (2, 1), (1, 1), (1, 2), 2),
                          O.conv2d_acc(q2, w2, (2, 1), (1, 1), (1, 2), 2))
    wt = O.quant(rng.standard_normal((4, 3, 3, 3)).astype(np.float16))
    for s, p, op, d in [((2, 2), (1, 1), (1, 1), (1, 1)), ((2, 3), (2, 0), (0, 2), (2, 1))]:
        want = F.conv_transpose2d(torch.tensor(q2, dtype=torch.float64), torch.tensor(wt, dtype=torch.float64),
                                  stride=s, padding=p, output_padding=op, groups=2, dilation=d).numpy()
        assert np.array_equal(O.conv_transpose_acc(q2, wt, s, p, op, d, 2), want.astype(np.int64))
    x1 = rng.standard_normal((2, 3, 9)).astype(np.float16)
    w1 = rng.standard_normal((4, 3, 3)).astype(np.float16)
    y1 = O.conv1d(x1, w1, None, 2, 1, 1, 1)
    y2 = O.conv2d(x1[:, :, None, :], w1[:, :, None, :], None, (1, 2), (0, 1), (1, 1), 1)[:, :, 0, :]
    assert np.array_equal(y1.view(np.uint16), y2.view(np.uint16))


def test_sampled_recomputation_equals_the_whole_oracle():
    """The full-size GPU tests check sampled outputs: scales of the whole
    operands, codes of the sampled rows / receptive fields only, exact int64
    dots, the oracle epilogue.  On a small case that equals the whole
    oracle's output at the same positions."""
    rng = np.random.default_rng(3)
    x = rng.standard_normal((40, 72)).astype(np.float16)
    w = (rng.standard_normal((50, 72)) * 0.02).astype(np.float16)
    b = (rng.standard_normal(50) * 0.01).astype(np.float16)
    full = O.linear(x, w, b)
    ax, aw = O.amax(x), O.amax(w)
    rows, cols = np.array([0, 7, 39]), np.array([0, 3, 20, 49])
    acc = O.quant(x[rows], ax).astype(np.int64) @ O.quant(w[cols], aw).astype(np.int64).T
    got = O.epilogue(acc, ax, aw, np.float16, bias=b[cols])
    assert np.array_equal(got.view(np.uint16), full[np.ix_(rows, cols)].view(np.uint16))
    xc = np.maximum(rng.standard_normal((2, 5, 7, 7)), 0).astype(np.float16)
    wc = (rng.standard_normal((4, 5, 3, 3)) * 0.3).astype(np.float16)
    fullc = O.conv2d(xc, wc, None, (1, 1), (1, 1), (1, 1), 1)
    axc, awc = O.amax(xc), O.amax(wc)
    qw = O.quant(wc, awc).astype(np.int64).reshape(4, -1)
    for n, oh, ow in [(0, 0, 0), (1, 6, 6), (1, 3, 0)]:
        xp = np.zeros((5, 3, 3), dtype=np.float16)
        for r in range(3):
            for s in range(3):
                ih, iw = oh - 1 + r, ow - 1 + s
                if 0 <= ih < 7 and 0 <= iw < 7:
                    xp[:, r, s] = xc[n, :, ih, iw]
        acc = (qw @ O.quant(xp, axc).astype(np.int64).reshape(-1))[None]
        got = O.epilogue(acc, axc, awc, np.float16)[0]
        assert np.array_equal(got.view(np.uint16), fullc[n, :, oh, ow].view(np.uint16))


def test_conv_weight_grad_accumulators_match_loops_and_float64_convs():
    """The oracle's weight-gradient accumulators against a scalar loop over the
    definition (2-D, strided, padded, dilated, grouped) and against torch's
    CPU float64 conv weight gradients of the same integer codes (exact)."""
    import torch
    rng = np.random.default_rng(11)
    x = rng.standard_normal((2, 4, 7, 6)).astype(np.float16)
    stride, pad, dil, groups = (2, 1), (1, 2), (1, 2), 2
    w_shape = (6, 2, 3, 2)
    OH = (7 + 2 - 2 - 1) // 2 + 1
    OW = (6 + 4 - 2 - 1) // 1 + 1
    g = rng.standard_normal((2, 6, OH, OW)).astype(np.float16)
    qx, qg = O.quant(x).astype(np.int64), O.quant(g).astype(np.int64)
    acc = O.conv_weight_grad_acc(qx, qg, w_shape, stride, pad, dil, groups)
    want = np.zeros(w_shape, dtype=np.int64)
    for f in range(6):
        grp = f // 3
        for c in range(2):
            for r in range(3):
                for s in range(2):
                    t = 0
                    for n in range(2):
                        for oh in range(OH):
                            for ow in range(OW):
                                ih, iw = oh * stride[0] - pad[0] + r * dil[0], ow * stride[1] - pad[1] + s * dil[1]
                                if 0 <= ih < 7 and 0 <= iw < 6:
                                    t += qg[n, f, oh, ow] * qx[n, grp * 2 + c, ih, iw]
                    want[f, c, r, s] = t
    assert np.array_equal(acc, want)
    tw = torch.nn.grad.conv2d_weight(torch.tensor(qx, dtype=torch.float64), w_shape,
                                     torch.tensor(qg, dtype=torch.float64), stride, pad, dil, groups)
    assert np.array_equal(acc, tw.numpy().astype(np.int64))
    x3 = rng.standard_normal((2, 3, 4, 5, 6)).astype(np.float16)
    g3 = rng.standard_normal((2, 4, 2, 5, 6)).astype(np.float16)
    q3, qg3 = O.quant(x3), O.quant(g3)
    acc3 = O.conv_weight_grad_acc(q3, qg3, (4, 3, 3, 1, 3), (2, 1, 1), (1, 0, 1), (1, 1, 1), 1)
    tw3 = torch.nn.grad.conv3d_weight(torch.tensor(q3, dtype=torch.float64), (4, 3, 3, 1, 3),
                                      torch.tensor(qg3, dtype=torch.float64), (2, 1, 1), (1, 0, 1), (1, 1, 1), 1)
    assert np.array_equal(acc3, tw3.numpy().astype(np.int64))
