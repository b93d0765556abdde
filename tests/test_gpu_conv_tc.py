"""TF32 tensor-core conv path (tcgen05 / TMEM mainloop) through the C ABI against the CPU oracle.

The reference has no tensor-core path; the bar for it is the one the BASELINE north star states
for TF32/BF16: relative L2 error <= 1e-2 (here per activation map, stricter than on the final head
only), and the same top-k boxes on whole networks.  TF32 keeps 10 of fp32's 23 mantissa bits, so a
map's error is ~1e-3 of its magnitude; an operand-layout error shows up as O(1)."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from tensorium_b200 import MATH_TF32
from tensorium_b200.layers import TConvolutionalLayer, TNNetState

pytestmark = pytest.mark.gpu

TF32_TOL = 1e-2  # relative L2 per activation map


def rel_l2_maps(a, b, maps):
    a = np.asarray(a, np.float64).reshape(maps, -1)
    b = np.asarray(b, np.float64).reshape(maps, -1)
    assert np.all(np.isfinite(a))
    num = np.sqrt(((a - b) ** 2).sum(axis=1))
    den = np.maximum(np.sqrt((b ** 2).sum(axis=1)), 1e-30)
    return float((num / den).max())


def run_layer(ctx, x, w, b, F, k, s, p, act, bn=None, residual=None, math_mode=MATH_TF32, dil=1):
    B, C, H, W = x.shape
    L = TConvolutionalLayer(B, H, W, C, F, 1, k, s, s, dil, p, act, bn is not None).bind(ctx)
    L.weights, L.biases = w, b
    if bn is not None:
        L.scales, L.rolling_mean, L.rolling_variance = bn
    xd = torch.from_numpy(x).to(ctx.torch_device)
    rd = None if residual is None else torch.from_numpy(residual).to(ctx.torch_device)
    y = L.forward(TNNetState(xd), residual=rd, math_mode=math_mode)
    return y.cpu().numpy()


CASES = [  # (B, C, H, F, k, s, p, dil): C % 32 == 0, the shapes the tcgen05 path takes
    (1, 32, 52, 64, 3, 1, 1, 1),      # YOLOv3 stage-1 shape, one k tile per tap
    (3, 64, 28, 96, 1, 1, 0, 1),      # 1x1, W % 4 == 0: A read from x in place; tiles span images
    (2, 256, 13, 255, 1, 1, 0, 1),    # 1x1 head shape: F = 255, W % 4 != 0 (replica), ragged tiles
    (3, 128, 13, 256, 3, 1, 1, 1),    # 3x3, odd spatial size, padded pixel grid
    (1, 512, 13, 1024, 3, 1, 1, 1),   # big K (144 k tiles), wide filter tiles
    (2, 96, 30, 40, 3, 1, 1, 1),      # F < 32 multiple (ragged filter tile), W = 30
    (2, 32, 52, 64, 3, 2, 1, 1),      # stride 2 (YOLOv3 downsampling): two row phases
    (1, 64, 27, 48, 3, 2, 1, 1),      # stride 2, odd input size
    (1, 32, 20, 32, 3, 1, 2, 2),      # dilation 2
    (2, 32, 17, 64, 5, 1, 2, 1),      # 5x5
    (2, 3, 64, 32, 3, 1, 1, 1),       # YOLOv3 layer-0 shape (3 channels): im2col rows, K = 27 -> 32
    (4, 1, 28, 32, 5, 1, 2, 1),       # MNIST conv1 (1 channel, 5x5)
    (1, 20, 17, 40, 3, 1, 2, 2),      # 20 channels (RSC packing, Cpad 32), dilation 2: im2col rows
    (2, 64, 13, 96, 1, 1, 0, 1),      # 1x1 with H*W % 4 != 0: one-tap replica
    (2, 64, 26, 48, 1, 1, 0, 1),      # 1x1 in place, H*W % 32 != 0: bounds-checked last group
]


@pytest.mark.parametrize("B,C,H,F,k,s,p,dil", CASES)
def test_tc_conv_matches_oracle(ctx, B, C, H, F, k, s, p, dil):
    rng = np.random.default_rng(B * 1000 + C + F + 7)
    x = rng.uniform(0, 1, (B, C, H, H)).astype(np.float32)
    w = (rng.standard_normal((F, C * k * k)) * np.sqrt(2.0 / (C * k * k))).astype(np.float32)
    b = rng.standard_normal(F).astype(np.float32) * 0.1
    for act in (9, 4):  # linear, leaky
        y = run_layer(ctx, x, w, b, F, k, s, p, act, dil=dil)
        ref = O.conv2d(x, w, b, F, k, s, p, act, dilation=dil)
        assert y.shape == ref.shape
        e = rel_l2_maps(y, ref, B * F)
        assert e <= TF32_TOL, e
        assert e > 0.0  # the tensor-core path ran (TF32 rounding is visible)


def test_tc_conv_batchnorm_and_residual(ctx):
    rng = np.random.default_rng(11)
    x = rng.uniform(0, 1, (2, 64, 26, 26)).astype(np.float32)
    w = (rng.standard_normal((128, 64 * 9)) * 0.05).astype(np.float32)
    b = np.zeros(128, np.float32)
    bn = (np.ones(128, np.float32), (rng.standard_normal(128) * 0.1).astype(np.float32),
          rng.uniform(0.5, 1.5, 128).astype(np.float32))
    r = rng.standard_normal((2, 128, 26, 26)).astype(np.float32)
    y = run_layer(ctx, x, w, b, 128, 3, 1, 1, 9, bn=bn, residual=r)
    ref = O.shortcut(O.conv2d(x, w, b, 128, 3, 1, 1, 9, bn=bn), r)
    assert rel_l2_maps(y, ref, 2 * 128) <= TF32_TOL


def test_tc_unsupported_shape_uses_fp32_kernel(ctx):
    """A conv with one output pixel per image (a connected layer) is not on the tensor-core path:
    TF32 mode gives the FP32 kernel's result."""
    rng = np.random.default_rng(12)
    x = rng.uniform(0, 1, (16, 64, 1, 1)).astype(np.float32)
    w = (rng.standard_normal((32, 64)) * 0.1).astype(np.float32)
    b = np.zeros(32, np.float32)
    a = run_layer(ctx, x, w, b, 32, 1, 1, 0, 9)
    f = run_layer(ctx, x, w, b, 32, 1, 1, 0, 9, math_mode=0)
    assert np.array_equal(a, f)


def test_yolov3_tf32_heads_and_boxes(ctx):
    """Whole YOLOv3-416 on the TF32 path (69 of 75 convs on tensor cores), batch 2, against the
    FP32 oracle: relative L2 <= 1e-2 on each head conv (per image), and the same detection index
    set (objectness > 0.45) apart from candidates whose logit lies inside the tolerance band."""
    from tensorium_b200 import synth
    from tensorium_b200.net import TNNet
    specs = synth.yolov3_specs()
    shape = (3, 416, 416)
    x = synth.input_images(3, "yolov3", 2, shape)
    heads, raws = [82, 94, 106], [81, 93, 105]
    ref = O.run_network(specs, x, keep=heads + raws)
    net = TNNet(ctx, specs, 2, shape, fusion=False, math_mode=MATH_TF32)
    net.forward(torch.from_numpy(x).to(ctx.torch_device), use_graph=False)
    thresh = 0.45
    logit = np.log(thresh / (1 - thresh))
    for h, r in zip(heads, raws):
        raw = net.output(r).cpu().numpy().reshape(2, -1)
        e = rel_l2_maps(raw, ref[r].reshape(2, -1), 2)
        print(f"head conv {r}: relative L2 {e:.2e}")
        assert e <= TF32_TOL, (r, e)
        got = net.output(h).cpu().numpy().reshape(2, 3, 85, -1)
        g = got.shape[-1]
        go, ro = got[:, :, 4], ref[h].reshape(2, 3, 85, g)[:, :, 4]
        xo = ref[r].reshape(2, 3, 85, g)[:, :, 4]
        band = TF32_TOL * np.sqrt((ref[r].reshape(2, 3, 85, g)[:, :, 4] ** 2).mean(axis=2, keepdims=True))
        sure = np.abs(xo - logit) > 4 * band
        assert np.array_equal((go > thresh)[sure], (ro > thresh)[sure]), h
    net.close()


PAIR_CASES = [  # (B, C, H, F, k, s, p) under a forced tile shape
    (1, 32, 52, 64, 3, 1, 1),      # 3x3 replica
    (3, 64, 28, 96, 1, 1, 0),      # in place, pair tiles straddling images
    (2, 256, 13, 255, 1, 1, 0),    # ragged filters (255) and pixels
    (2, 32, 52, 64, 3, 2, 1),      # stride 2
    (2, 3, 40, 32, 3, 1, 1),       # im2col rows
    (1, 256, 13, 160, 3, 1, 1),    # 72 k tiles: split-K units of uneven tiles
]


@pytest.mark.parametrize("shape", ["64,2", "128,2", "256,2", "256,1", "32,1", "128,1,2", "256,1,3", "64,1,4"])
def test_tc_conv_every_tile_shape(ctx, shape, monkeypatch):
    """Each (filters per tile, CTAs per tile[, K splits]) shape of the tensor-core kernel, pinned
    through the TB_TC_FORCE test hook: 2 CTAs = a pair on two SMs (cta_group::2, M = 256); splits =
    split-K units whose partial tiles the last arriving unit sums in split order.  Each case runs
    twice: identical results (deterministic split-K, counters reset)."""
    monkeypatch.setenv("TB_TC_FORCE", shape)
    rng = np.random.default_rng(21)
    for (B, C, H, F, k, s, p) in PAIR_CASES:
        x = rng.uniform(0, 1, (B, C, H, H)).astype(np.float32)
        w = (rng.standard_normal((F, C * k * k)) * np.sqrt(2.0 / (C * k * k))).astype(np.float32)
        b = rng.standard_normal(F).astype(np.float32) * 0.1
        y1 = run_layer(ctx, x, w, b, F, k, s, p, 4)
        y2 = run_layer(ctx, x, w, b, F, k, s, p, 4)
        assert np.array_equal(y1, y2), (shape, C)
        ref = O.conv2d(x, w, b, F, k, s, p, 4)
        e = rel_l2_maps(y1, ref, B * F)
        assert 0.0 < e <= TF32_TOL, (shape, C, e)


def test_yolov3_tf32_nhwc_plan(ctx):
    """The fused TF32 YOLOv3 runs its activations NHWC (every conv on the NHWC tensor-core kernel,
    A operand by TMA im2col): intermediate maps and the three yolo outputs within the TF32 bar of
    the FP32 oracle, the same detection index sets away from the threshold band, and graph replay
    equal to eager."""
    import ctypes as C_
    from tensorium_b200 import synth
    from tensorium_b200._lib import lib
    from tensorium_b200.net import TNNet
    specs = synth.yolov3_specs()
    shape = (3, 416, 416)
    x = synth.input_images(3, "yolov3", 2, shape)
    heads, raws, inner = [82, 94, 106], [81, 93, 105], [1, 36, 61, 85, 97]
    ref = O.run_network(specs, x, keep=heads + raws + inner)
    net = TNNet(ctx, specs, 2, shape, math_mode=MATH_TF32)
    ps = C_.c_int64()
    lib.tb_net_layer_layout(net.handle, 36, C_.byref(ps))
    assert ps.value == 384  # NHWC, a 256-channel slice of the 384-channel route 97 buffer
    xd = torch.from_numpy(x).to(ctx.torch_device)
    net.forward(xd, use_graph=False)
    for i in inner:  # per image, as the heads
        e = rel_l2_maps(net.output(i).cpu().numpy(), ref[i], 2)
        assert e <= TF32_TOL, (i, e)
    eager = [net.output(h).clone() for h in heads]
    thresh = 0.45
    logit = np.log(thresh / (1 - thresh))
    for h, r, got in zip(heads, raws, eager):
        got = got.cpu().numpy()
        e = rel_l2_maps(got, ref[h], 2)
        assert e <= TF32_TOL, (h, e)
        g = got.shape[-1] // 255
        go, ro = got.reshape(2, 3, 85, g)[:, :, 4], ref[h].reshape(2, 3, 85, g)[:, :, 4]
        xo = ref[r].reshape(2, 3, 85, g)[:, :, 4]
        band = TF32_TOL * np.sqrt((xo ** 2).mean(axis=2, keepdims=True))
        sure = np.abs(xo - logit) > 4 * band
        assert np.array_equal((go > thresh)[sure], (ro > thresh)[sure]), h
    net.forward(xd, use_graph=True)
    for h, e in zip(heads, eager):
        assert torch.equal(net.output(h), e)
    net.close()
