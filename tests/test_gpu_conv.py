"""Conv kernel parity: the CUDA path through the C ABI against the CPU oracle.

FP32 path (default, TB_MATH_FP32): bit-exact -- the order-exact kernel (and the direct kernel for
short reductions) keeps the reference's k order and one FMA per k.  The elementwise metric
(|a-b| / max(|b|, 1e-3 rms) per map) is reported and is 0.
The tiled FP32 kernels (TB_MATH_FP32_TILED: k tiles in (kh, kw, c) order, split-K) reorder the
sum and are held to max|a-b|/max|b| <= 1e-4 per map."""
import numpy as np
import pytest
import torch

from conftest import FP32_TOL, assert_bit_exact, logistic_ulps, worst_map_err
from oracle import oracle as O
from tensorium_b200 import MATH_FP32_TILED, synth
from tensorium_b200.layers import TConvolutionalLayer, TNNetState

pytestmark = pytest.mark.gpu


def run_layer(ctx, x, w, b, F, k, s, p, act, bn=None, residual=None, dil=1, math_mode=-1, in_bs=0):
    B, C, H, W = x.shape
    L = TConvolutionalLayer(B, H, W, C, F, 1, k, s, s, dil, p, act, bn is not None).bind(ctx)
    L.weights, L.biases = w, b
    if bn is not None:
        L.scales, L.rolling_mean, L.rolling_variance = bn
    xd = torch.from_numpy(x).to(ctx.torch_device)
    rd = None if residual is None else torch.from_numpy(residual).to(ctx.torch_device)
    y = L.forward(TNNetState(xd), residual=rd, math_mode=math_mode)
    return y.cpu().numpy()


def rand_case(seed, B, C, H, F, k):
    rng = np.random.default_rng(seed)
    x = rng.uniform(0, 1, (B, C, H, H)).astype(np.float32)
    w = (rng.standard_normal((F, C * k * k)) * np.sqrt(2.0 / (C * k * k))).astype(np.float32)
    b = rng.standard_normal(F).astype(np.float32) * 0.1
    return x, w, b


CASES = [  # (B, C, H, F, k, s, p, dil) -- every mode of the order-exact kernel and the direct kernel
    (1, 3, 416, 32, 3, 1, 1, 1),     # config 0 shape (direct kernel)
    (2, 32, 52, 64, 3, 2, 1, 1),     # 3x3 stride 2
    (2, 64, 26, 32, 1, 1, 0, 1),     # 1x1 vectorised (OHW % 4 == 0), 32 filters
    (3, 128, 13, 256, 3, 1, 1, 1),   # 3x3, OHW odd
    (1, 512, 13, 1024, 3, 1, 1, 1),  # K = 4608
    (2, 256, 13, 255, 1, 1, 0, 1),   # 1x1 gather (OHW % 4 != 0), M = 255
    (1, 20, 17, 40, 3, 1, 2, 2),     # dilation 2, C not a multiple of the stage's channels
    (4, 1, 28, 32, 5, 1, 2, 1),      # MNIST conv1 (direct)
    (2, 32, 14, 64, 5, 1, 2, 1),     # MNIST conv2 (generic window)
    (1, 100, 9, 130, 5, 2, 2, 1),    # ragged everything, generic window
    (2, 33, 11, 20, 1, 2, 0, 1),     # strided 1x1, odd channels
    (1, 7, 10, 9, 3, 1, 0, 1),       # 3x3 without padding, C < 16 (CRS-packed weights)
]


@pytest.mark.parametrize("B,C,H,F,k,s,p,dil", CASES)
def test_conv_bit_exact(ctx, B, C, H, F, k, s, p, dil):
    x, w, b = rand_case(B * 1000 + C + F, B, C, H, F, k)
    for act in (9, 4):
        y = run_layer(ctx, x, w, b, F, k, s, p, act, dil=dil)
        ref = O.conv2d(x, w, b, F, k, s, p, act, dilation=dil)
        assert_bit_exact(y, ref, B * F, (B, C, H, F, k, s, act))


@pytest.mark.parametrize("tile", [0, 1, 2, 3, 4, 5, 10, 15, 17, 100, 101, 110, 111])
def test_every_exact_tile(ctx, tile, monkeypatch):
    """Each configuration of the order-exact kernel (TB_EXACT_FORCE pins it: tile = index % 5,
    stage-depth variant = index / 5, 100 / 101 the warp-specialised kernel with 64 / 128 pixels;
    a configuration a layer cannot take falls back to an admissible one) on the 3x3, 1x1 vector,
    1x1 gather and generic-window modes, each twice."""
    monkeypatch.setenv("TB_EXACT_FORCE", str(tile))
    for i, (B, C, H, F, k, s, p) in enumerate([(2, 32, 26, 64, 3, 2, 1), (1, 64, 20, 128, 3, 1, 1),
                                               (2, 64, 12, 96, 1, 1, 0), (2, 48, 13, 40, 1, 1, 0),
                                               (1, 24, 12, 70, 5, 1, 2), (1, 20, 9, 30, 3, 1, 1)]):
        x, w, b = rand_case(100 + i, B, C, H, F, k)
        ref = O.conv2d(x, w, b, F, k, s, p, 9)
        y1 = run_layer(ctx, x, w, b, F, k, s, p, 9)
        y2 = run_layer(ctx, x, w, b, F, k, s, p, 9)
        assert_bit_exact(y1, ref, B * F, (tile, i))
        assert np.array_equal(y1, y2)


def test_config0_unfused_batchnorm(ctx):
    """conv 3->32 3x3 + batchnorm (unfused, as TConvolutionalLayer.forward
    runs it) + leaky, on 3x416x416: bit-exact."""
    s = synth.config0_spec()[0]
    x = synth.input_images(0, "cfg0", 1, (3, 416, 416))
    bn = (s["scales"], s["mean"], s["var"])
    y = run_layer(ctx, x, s["weights"], s["biases"], 32, 3, 1, 1, 9, bn=bn)
    ref = O.conv2d(x, s["weights"], s["biases"], 32, 3, 1, 1, 9, bn=bn)
    assert_bit_exact(y, ref, 32, "config 0")


def test_unfused_batchnorm_exact_kernel(ctx):
    x, w, b = rand_case(17, 2, 64, 20, 96, 3)
    rng = np.random.default_rng(18)
    bn = (rng.uniform(0.5, 1.5, 96).astype(np.float32), (rng.standard_normal(96) * 0.1).astype(np.float32),
          rng.uniform(0.5, 1.5, 96).astype(np.float32))
    y = run_layer(ctx, x, w, b, 96, 3, 1, 1, 9, bn=bn)
    ref = O.conv2d(x, w, b, 96, 3, 1, 1, 9, bn=bn)
    assert_bit_exact(y, ref, 2 * 96, "unfused batchnorm")


def test_residual_epilogue(ctx):
    rng = np.random.default_rng(7)
    x = rng.uniform(0, 1, (2, 64, 26, 26)).astype(np.float32)
    w = (rng.standard_normal((128, 64 * 9)) * 0.05).astype(np.float32)
    b = np.zeros(128, np.float32)
    r = rng.standard_normal((2, 128, 26, 26)).astype(np.float32)
    y = run_layer(ctx, x, w, b, 128, 3, 1, 1, 9, residual=r)
    ref = O.shortcut(O.conv2d(x, w, b, 128, 3, 1, 1, 9), r)
    assert_bit_exact(y, ref, 2 * 128, "residual")


PIECEWISE = (1, 2, 3, 4, 5, 7, 8, 9, 13, 14)   # relu relu6 relie linear ramp plse revleaky leaky hardtan lhtan
TRANSCENDENTAL = (0, 6, 10, 11, 15)           # logistic tanh elu loggy selu (double exp: libm vs CUDA)


def test_all_activations(ctx):
    rng = np.random.default_rng(8)
    x = rng.standard_normal((1, 8, 12, 12)).astype(np.float32)
    w = rng.standard_normal((16, 72)).astype(np.float32) * 0.3
    b = np.zeros(16, np.float32)
    for act in PIECEWISE:
        y = run_layer(ctx, x, w, b, 16, 3, 1, 1, act)
        assert_bit_exact(y, O.conv2d(x, w, b, 16, 3, 1, 1, act), 16, act)
    for act in TRANSCENDENTAL:
        y = run_layer(ctx, x, w, b, 16, 3, 1, 1, act)
        ref = O.conv2d(x, w, b, 16, 3, 1, 1, act)
        assert logistic_ulps(y[ref != 0], ref[ref != 0]) <= 2.0, act
        assert np.array_equal(y[ref == 0], ref[ref == 0]), act


@pytest.mark.parametrize("cfg", ["128,128,1", "64,128,1", "64,64,1", "32,256,1", "128,128,3", "64,128,5",
                                 "64,64,2", "32,256,4", "128,128,1,1", "128,128,3,1"])
def test_tiled_kernel_every_tile_and_split(ctx, cfg, monkeypatch):
    """TB_MATH_FP32_TILED: each CTA tile and split-K count (pinned through TB_CONV_FORCE), on a
    strided RSC layer, a stride-1 RSC layer, a CRS layer and a vectorised 1x1 layer; each twice,
    so the split-K arrival counters are seen to reset.  A fourth field 1 selects the TMA-fed
    kernel.  The summation is reordered: max|a-b|/max|b| <= 1e-4 per map."""
    monkeypatch.setenv("TB_CONV_FORCE", cfg)
    rng = np.random.default_rng(11)
    for (B, C, H, F, k, s, p) in [(2, 32, 26, 64, 3, 2, 1), (1, 64, 20, 128, 3, 1, 1), (1, 3, 21, 16, 3, 1, 1),
                                  (2, 64, 12, 96, 1, 1, 0)]:
        x = rng.uniform(0, 1, (B, C, H, H)).astype(np.float32)
        w = (rng.standard_normal((F, C * k * k)) * 0.1).astype(np.float32)
        b = rng.standard_normal(F).astype(np.float32) * 0.1
        ref = O.conv2d(x, w, b, F, k, s, p, 9)
        y1 = run_layer(ctx, x, w, b, F, k, s, p, 9, math_mode=MATH_FP32_TILED)
        y2 = run_layer(ctx, x, w, b, F, k, s, p, 9, math_mode=MATH_FP32_TILED)
        assert np.array_equal(y1, y2)
        assert worst_map_err(y1, ref, B * F) <= FP32_TOL, (cfg, C)


DIRECT_CASES = [  # (B, C, H, F, k, s, p, dil): reductions of <= 32 on the direct kernel
    (2, 3, 416, 32, 3, 1, 1, 1),     # YOLOv3 layer 0 / config 0
    (2, 3, 33, 16, 3, 2, 1, 1),      # stride 2, odd size
    (8, 1, 28, 32, 5, 1, 2, 1),      # MNIST conv1
    (1, 2, 20, 100, 3, 1, 2, 2),     # dilation 2, F not a multiple of 8
    (3, 4, 9, 128, 2, 1, 0, 1),      # even kernel, no padding, F = 128
]


@pytest.mark.parametrize("B,C,H,F,k,s,p,dil", DIRECT_CASES)
def test_direct_kernel_is_bit_exact(ctx, B, C, H, F, k, s, p, dil):
    """The direct kernel runs the reference's dot product (one FMA per k, ascending, from 0) and
    epilogue in the same order, so it equals the oracle bit for bit."""
    x, w, b = rand_case(B * 100 + C * 10 + F, B, C, H, F, k)
    for act in (9, 4):
        y = run_layer(ctx, x, w, b, F, k, s, p, act, dil=dil)
        assert_bit_exact(y, O.conv2d(x, w, b, F, k, s, p, act, dilation=dil), B * F, act)


def test_tiled_kernel_on_a_direct_layer(ctx, monkeypatch):
    rng = np.random.default_rng(3)
    x = rng.uniform(0, 1, (2, 3, 64, 64)).astype(np.float32)
    w = (rng.standard_normal((32, 27)) * 0.3).astype(np.float32)
    b = rng.standard_normal(32).astype(np.float32) * 0.1
    bn = (np.ones(32, np.float32), (rng.standard_normal(32) * 0.1).astype(np.float32),
          rng.uniform(0.5, 1.5, 32).astype(np.float32))
    monkeypatch.setenv("TB_CONV_FORCE", "32,256,1")
    g = run_layer(ctx, x, w, b, 32, 3, 1, 1, 9, bn=bn, math_mode=MATH_FP32_TILED)
    ref = O.conv2d(x, w, b, 32, 3, 1, 1, 9, bn=bn)
    assert worst_map_err(g, ref, 64) <= FP32_TOL
