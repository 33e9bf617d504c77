"""conv2d on the kunlun device against the oracle's exact restatement of the
reference's quantised conv (csrc/ops.cpp:237-285): one max-abs int16 scale for
the whole input and one for the whole weight, exact integer MAC, T(acc * s),
then the bias added and rounded.  These cases exercise the implicit-GEMM
tensor-core path (groups 1, stride 1: shifted TMA windows over NHWC limb
rows), including ragged channel groups, filter tiles, wide rows split into
several pixel tiles, dilation and fp32; results must be bit-identical."""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu

torch_kunlun = pytest.importorskip("torch_kunlun")
from oracle import oracle as O  # noqa: E402
from tests._qgemm_helpers import assert_bits_equal  # noqa: E402

DEV = "kunlun"


def rnd(shape, seed, scale=1.0, dtype=torch.float16):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(shape, generator=g) * scale).to(dtype)


CASES = [
    # N, C, H, W, F, k, pad, dil, bias, dtype
    (2, 64, 12, 12, 64, 3, 1, 1, False, torch.float16),
    (1, 70, 9, 11, 33, 3, 1, 1, True, torch.float16),      # ragged channel group, F < 64
    (2, 32, 5, 140, 200, 1, 0, 1, True, torch.float16),    # row wider than one pixel tile, 2 filter tiles
    (1, 128, 14, 14, 130, 3, 1, 1, True, torch.float16),   # BN=128 tiles with a ragged second tile
    (1, 16, 10, 10, 24, 3, 2, 2, False, torch.float16),    # dilation 2
    (2, 8, 7, 7, 16, 5, 2, 1, True, torch.float32),        # fp32
    (1, 3, 17, 17, 8, 7, 3, 1, True, torch.float16),       # RGB stem-like
    # 1x1 with the input quantised inside the kernel (fp16, <= 64 filters, <= 256
    # channels, plane a multiple of 8 pixels):
    (2, 256, 56, 56, 64, 1, 0, 1, False, torch.float16),   # the ResNet-50 stage shape, ragged last pixel tile
    (3, 100, 9, 8, 40, 1, 0, 1, True, torch.float16),      # ragged channel group (zero-filled), bias
    (1, 192, 16, 16, 64, 1, 0, 1, True, torch.float16),    # three channel groups
    # 1x1 cases that keep the limb pass: plane not a multiple of 8, 320 channels
    (2, 64, 7, 9, 8, 1, 0, 1, False, torch.float16),
    (1, 320, 8, 8, 64, 1, 0, 1, True, torch.float16),
]


def test_1x1_in_kernel_quantisation_non_finite():
    """A NaN or an infinity in the input makes its scale non-finite: every
    output is NaN, on the path that quantises the input inside the 1x1 kernel
    too."""
    for bad in (float("nan"), float("inf"), -float("inf")):
        x = torch.relu(rnd((2, 128, 16, 16), 43))
        x[1, 127, 15, 15] = bad
        w = rnd((32, 128, 1, 1), 44, scale=0.1)
        y = torch.nn.functional.conv2d(x.to(DEV), w.to(DEV)).cpu()
        assert bool(torch.isnan(y).all()), bad


@pytest.mark.parametrize("case", CASES)
def test_implicit_gemm_conv_bit_exact(case):
    N, C, H, W, F, k, pad, dil, has_b, dt = case
    x = torch.relu(rnd((N, C, H, W), 40, dtype=dt))
    w = rnd((F, C, k, k), 41, scale=math.sqrt(2.0 / (C * k * k)), dtype=dt)
    b = rnd((F,), 42, scale=0.01, dtype=dt) if has_b else None
    y = torch.nn.functional.conv2d(x.to(DEV), w.to(DEV), None if b is None else b.to(DEV),
                                   padding=pad, dilation=dil).cpu()
    want = O.conv2d(x.numpy(), w.numpy(), None if b is None else b.numpy(), (1, 1), (pad, pad),
                    (dil, dil), 1)
    assert y.shape == want.shape
    assert_bits_equal(y.numpy(), want, f"conv2d {case}")


def test_resnet_stage_shapes_match_fp32_reference():
    """The benchmark's ResNet-50 stage convs (batch 2 here) against torch's
    fp32 CPU conv within the fp16 quantised bound."""
    for (C, F, H, k, pad, bias) in [(256, 64, 56, 1, 0, False), (64, 64, 56, 3, 1, False),
                                    (256, 256, 14, 3, 1, True)]:
        x = torch.relu(rnd((2, C, H, H), 43))
        w = rnd((F, C, k, k), 44, scale=math.sqrt(2.0 / (C * k * k)))
        b = rnd((F,), 45, scale=0.01) if bias else None
        y = torch.nn.functional.conv2d(x.to(DEV), w.to(DEV), None if b is None else b.to(DEV),
                                       padding=pad).cpu().float()
        ref = torch.nn.functional.conv2d(x.float(), w.float(), None if b is None else b.float(),
                                         padding=pad)
        bound = 2 ** -10 * x.abs().max().item() * w.abs().max().item() * C * k * k
        assert (y - ref).abs().max().item() <= bound


DW_CASES = [
    # N, C, mult, H, W, k, stride, pad, dil, bias, dtype
    (2, 512, 1, 7, 7, 3, 1, 1, 1, False, torch.float16),   # the ResNet/MobileNet-style stage shape
    (1, 6, 2, 9, 11, 3, 2, 1, 1, True, torch.float16),     # channel multiplier 2, stride 2
    (1, 4, 1, 40, 40, 5, 1, 4, 2, True, torch.float32),    # plane above the shared-memory size
    (3, 5, 1, 8, 8, 3, 1, 0, 1, True, torch.float32),
    (1, 3, 1, 50, 50, 3, 1, 1, 1, False, torch.float16),   # plane too large for the staged kernels
    (2, 8, 2, 40, 40, 3, 1, 1, 1, True, torch.float16),    # multiplier 2 on planes above 1024
    # the row kernel (multiplier 1, unit stride and dilation, KW in 3/5/7):
    (64, 512, 1, 7, 7, 3, 1, 1, 1, True, torch.float16),   # the benchmark shape, with bias
    (2, 16, 1, 9, 13, 3, 1, 1, 1, False, torch.float32),   # rows longer than one 8-output window
    (3, 5, 1, 20, 17, 5, 1, 2, 1, True, torch.float16),    # 5x5, ragged plane count per block
    (1, 7, 1, 11, 11, 7, 1, 3, 1, True, torch.float16),    # 7x7
    (2, 3, 1, 1, 40, 3, 1, 1, 1, False, torch.float16),    # one-row planes, padding wider than the row
    (2, 6, 1, 5, 5, 3, 1, 2, 1, True, torch.float32),      # padding 2: outputs beyond the input
    # more blocks than fit on the device in one wave: the two-pass path (amax
    # launch, then the row kernel) instead of the partials + scaled kernels
    (64, 512, 1, 14, 14, 3, 1, 1, 1, True, torch.float16),
]


def test_depthwise_scaled_path_propagates_non_finite():
    """A NaN or an infinity anywhere in the input makes the input scale
    non-finite, so every output is NaN (the library's convention), through
    the path whose convolution kernel folds the partial maxima of the amax
    kernel before it."""
    for bad in (float("nan"), float("inf")):
        x = torch.relu(rnd((4, 32, 7, 7), 49))
        x[3, 31, 6, 6] = bad
        w = rnd((32, 1, 3, 3), 50)
        y = torch.nn.functional.conv2d(x.to(DEV), w.to(DEV), padding=1, groups=32).cpu()
        assert bool(torch.isnan(y).all()), bad
    x = torch.relu(rnd((4, 32, 7, 7), 51))
    w = rnd((32, 1, 3, 3), 52)
    w[17, 0, 1, 1] = float("nan")
    y = torch.nn.functional.conv2d(x.to(DEV), w.to(DEV), padding=1, groups=32).cpu()
    assert bool(torch.isnan(y).all())


@pytest.mark.parametrize("case", DW_CASES)
def test_depthwise_conv_bit_exact(case):
    N, C, mult, H, W, k, s, pad, dil, has_b, dt = case
    F = C * mult
    x = torch.relu(rnd((N, C, H, W), 46, dtype=dt))
    w = rnd((F, 1, k, k), 47, scale=math.sqrt(2.0 / (k * k)), dtype=dt)
    b = rnd((F,), 48, scale=0.01, dtype=dt) if has_b else None
    y = torch.nn.functional.conv2d(x.to(DEV), w.to(DEV), None if b is None else b.to(DEV), stride=s,
                                   padding=pad, dilation=dil, groups=C).cpu()
    want = O.conv2d(x.numpy(), w.numpy(), None if b is None else b.numpy(), (s, s), (pad, pad),
                    (dil, dil), C)
    assert_bits_equal(y.numpy(), want, f"depthwise {case}")
