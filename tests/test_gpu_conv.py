"""Conv kernel parity: the CUDA path through the C ABI against the CPU oracle (FP32 path, max
relative error per activation map <= 1e-4 with a 0.1%-of-rms floor; see conftest)."""
import numpy as np
import pytest
import torch

from conftest import FP32_TOL, worst_map_err
from oracle import oracle as O
from tensorium_b200 import synth
from tensorium_b200.layers import TConvolutionalLayer, TNNetState

pytestmark = pytest.mark.gpu


def run_layer(ctx, x, w, b, F, k, s, p, act, bn=None, residual=None, dil=1):
    B, C, H, W = x.shape
    L = TConvolutionalLayer(B, H, W, C, F, 1, k, s, s, dil, p, act, bn is not None).bind(ctx)
    L.weights, L.biases = w, b
    if bn is not None:
        L.scales, L.rolling_mean, L.rolling_variance = bn
    xd = torch.from_numpy(x).to(ctx.torch_device)
    rd = None if residual is None else torch.from_numpy(residual).to(ctx.torch_device)
    y = L.forward(TNNetState(xd), residual=rd)
    return y.cpu().numpy()


CASES = [  # (B, C, H, F, k, s, p, dil)  -- every kernel mode / tile config / split-K
    (1, 3, 416, 32, 3, 1, 1, 1),     # config 0 shape (CRS, 32x256 tile)
    (2, 3, 33, 16, 3, 2, 1, 1),      # CRS, stride 2, odd size
    (2, 32, 52, 64, 3, 2, 1, 1),     # RSC, 64x128
    (2, 64, 26, 32, 1, 1, 0, 1),     # 1x1 vectorised, 32x256
    (3, 128, 13, 256, 3, 1, 1, 1),   # RSC, OHW odd, split-K
    (1, 512, 13, 1024, 3, 1, 1, 1),  # big K, split-K, 64x64
    (2, 256, 13, 255, 1, 1, 0, 1),   # 1x1 scalar path (OHW % 4 != 0), M = 255
    (1, 20, 17, 40, 3, 1, 2, 2),     # dilation 2, C not a multiple of 16
    (4, 1, 28, 32, 5, 1, 2, 1),      # MNIST conv1
    (1, 100, 9, 130, 5, 2, 2, 1),    # ragged everything
]


@pytest.mark.parametrize("B,C,H,F,k,s,p,dil", CASES)
def test_conv_matches_oracle(ctx, B, C, H, F, k, s, p, dil):
    rng = np.random.default_rng(B * 1000 + C + F)
    x = rng.uniform(0, 1, (B, C, H, H)).astype(np.float32)
    w = (rng.standard_normal((F, C * k * k)) * np.sqrt(2.0 / (C * k * k))).astype(np.float32)
    b = rng.standard_normal(F).astype(np.float32) * 0.1
    for act in (9, 4):
        y = run_layer(ctx, x, w, b, F, k, s, p, act, dil=dil)
        ref = O.conv2d(x, w, b, F, k, s, p, act, dilation=dil)
        assert y.shape == ref.shape
        assert worst_map_err(y, ref, B * F) <= FP32_TOL


def test_config0_unfused_batchnorm(ctx):
    """conv 3->32 3x3 + batchnorm (unfused, as TConvolutionalLayer.forward
    runs it) + leaky, on 3x416x416."""
    s = synth.config0_spec()[0]
    x = synth.input_images(0, "cfg0", 1, (3, 416, 416))
    bn = (s["scales"], s["mean"], s["var"])
    y = run_layer(ctx, x, s["weights"], s["biases"], 32, 3, 1, 1, 9, bn=bn)
    ref = O.conv2d(x, s["weights"], s["biases"], 32, 3, 1, 1, 9, bn=bn)
    assert worst_map_err(y, ref, 32) <= FP32_TOL


def test_residual_epilogue(ctx):
    rng = np.random.default_rng(7)
    x = rng.uniform(0, 1, (2, 64, 26, 26)).astype(np.float32)
    w = (rng.standard_normal((128, 64 * 9)) * 0.05).astype(np.float32)
    b = np.zeros(128, np.float32)
    r = rng.standard_normal((2, 128, 26, 26)).astype(np.float32)
    y = run_layer(ctx, x, w, b, 128, 3, 1, 1, 9, residual=r)
    ref = O.shortcut(O.conv2d(x, w, b, 128, 3, 1, 1, 9), r)
    assert worst_map_err(y, ref, 2 * 128) <= FP32_TOL


def test_all_activations(ctx):
    rng = np.random.default_rng(8)
    x = rng.standard_normal((1, 8, 12, 12)).astype(np.float32)
    w = rng.standard_normal((16, 72)).astype(np.float32) * 0.3
    b = np.zeros(16, np.float32)
    for act in (0, 1, 2, 3, 4, 5, 6, 7, 8, 9, 10, 11, 13, 14, 15):
        y = run_layer(ctx, x, w, b, 16, 3, 1, 1, act)
        ref = O.conv2d(x, w, b, 16, 3, 1, 1, act)
        assert worst_map_err(y, ref, 16) <= FP32_TOL, act


@pytest.mark.parametrize("cfg", ["128,128,1", "64,128,1", "64,64,1", "32,256,1", "128,128,3", "64,128,5",
                                 "64,64,2", "32,256,4", "128,128,1,1", "128,128,3,1"])
def test_every_tile_and_split_configuration(ctx, cfg, monkeypatch):
    """Each CTA tile and split-K count (pinned through the TB_CONV_FORCE test hook), on a
    strided RSC layer, a stride-1 RSC layer, a CRS layer and a vectorised 1x1 layer; each twice,
    so the split-K arrival counters are seen to reset.  A fourth field 1 selects the TMA-fed
    kernel (RSC and 1x1 layers; the CRS layer keeps the gather kernel)."""
    monkeypatch.setenv("TB_CONV_FORCE", cfg)
    rng = np.random.default_rng(11)
    for (B, C, H, F, k, s, p) in [(2, 32, 26, 64, 3, 2, 1), (1, 64, 20, 128, 3, 1, 1), (1, 3, 21, 16, 3, 1, 1),
                                  (2, 64, 12, 96, 1, 1, 0)]:
        x = rng.uniform(0, 1, (B, C, H, H)).astype(np.float32)
        w = (rng.standard_normal((F, C * k * k)) * 0.1).astype(np.float32)
        b = rng.standard_normal(F).astype(np.float32) * 0.1
        ref = O.conv2d(x, w, b, F, k, s, p, 9)
        y1 = run_layer(ctx, x, w, b, F, k, s, p, 9)
        y2 = run_layer(ctx, x, w, b, F, k, s, p, 9)
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
    epilogue in the same order, so it equals the oracle bit for bit; the GEMM kernel on the same
    layer (pinned with TB_CONV_FORCE) agrees within the FP32 tolerance."""
    rng = np.random.default_rng(B * 100 + C * 10 + F)
    x = rng.uniform(0, 1, (B, C, H, H)).astype(np.float32)
    w = (rng.standard_normal((F, C * k * k)) * np.sqrt(2.0 / (C * k * k))).astype(np.float32)
    b = rng.standard_normal(F).astype(np.float32) * 0.1
    for act in (9, 4, 0):
        y = run_layer(ctx, x, w, b, F, k, s, p, act, dil=dil)
        ref = O.conv2d(x, w, b, F, k, s, p, act, dilation=dil)
        assert np.array_equal(y, ref), (act, np.abs(y - ref).max())


def test_direct_kernel_against_gemm_kernel(ctx, monkeypatch):
    rng = np.random.default_rng(3)
    x = rng.uniform(0, 1, (2, 3, 64, 64)).astype(np.float32)
    w = (rng.standard_normal((32, 27)) * 0.3).astype(np.float32)
    b = rng.standard_normal(32).astype(np.float32) * 0.1
    bn = (np.ones(32, np.float32), (rng.standard_normal(32) * 0.1).astype(np.float32),
          rng.uniform(0.5, 1.5, 32).astype(np.float32))
    y = run_layer(ctx, x, w, b, 32, 3, 1, 1, 9, bn=bn)
    monkeypatch.setenv("TB_CONV_FORCE", "32,256,1")
    g = run_layer(ctx, x, w, b, 32, 3, 1, 1, 9, bn=bn)
    ref = O.conv2d(x, w, b, 32, 3, 1, 1, 9, bn=bn)
    assert worst_map_err(y, ref, 64) <= FP32_TOL and worst_map_err(g, ref, 64) <= FP32_TOL
