"""The staged-once 3x3 stride-1 conv kernel (k_conv_slide, configurations 120-136 of the order-exact
FP32 conv: 128x128, 128x64, 64x128, 64x64 filters x positions, with a register window over
one staged copy (120-123), four shifted copies (124-127), relaxed register caps (128-130) and
smaller thread tiles (131-136)) against the CPU oracle, bit for bit.

Its position space pads every image row to a pitch Wp (Wp mod 4 = 0, 1 or 2 give different
compile-time window offsets) and every image by one junk row, so the cases cover each pitch class
(W = 13 -> Wp 14, W = 26 -> 28, W = 52 -> 53), non-square images, tiles that straddle images, ragged
filter counts, an input that is a channel slice of a wider tensor (a zero-copy route), the residual
and unfused-batchnorm epilogues, and two calls in a row."""
import ctypes as C

import numpy as np
import pytest
import torch

from conftest import assert_bit_exact
from oracle import oracle as O
from tensorium_b200._lib import ConvDesc, check, lib
from tensorium_b200.context import ptr

pytestmark = pytest.mark.gpu

TILES = list(range(120, 137))


def _conv(ctx, x, w, b, F, act=9, x_bs=0, residual=None, bn=None):
    """tb_conv2d_fwd through the C ABI on an input whose images are x_bs floats apart."""
    B, Cin, H, W = x.shape if x_bs == 0 else (x.shape[0], w.shape[1] // 9, x.shape[2], x.shape[3])
    d = ConvDesc(B, Cin, H, W, F, 3, 3, 1, 1, 1, 1, 1, 1, act, x_bs, 0, 0)
    dev = ctx.torch_device
    n = C.c_int64()
    check(lib.tb_conv_packed_weights_count(C.byref(d), C.byref(n)))
    raw = torch.from_numpy(np.ascontiguousarray(w)).to(dev)
    packed = torch.empty(n.value, dtype=torch.float32, device=dev)
    check(lib.tb_conv_pack_weights(ctx.handle, C.byref(d), ptr(raw), ptr(packed)))
    xd = torch.from_numpy(np.ascontiguousarray(x)).to(dev)
    bd = torch.from_numpy(b).to(dev)
    y = torch.full((B, F, H, W), float("nan"), device=dev)
    rd = None if residual is None else torch.from_numpy(residual).to(dev)
    bnd = [None, None, None] if bn is None else [torch.from_numpy(a).to(dev) for a in bn]
    check(lib.tb_conv2d_fwd(ctx.handle, C.byref(d), ptr(xd), ptr(packed), ptr(bd),
                            *[ptr(t) if t is not None else None for t in bnd],
                            ptr(rd) if rd is not None else None, ptr(y), -1))
    torch.cuda.synchronize()
    return y.cpu().numpy()


def _case(seed, B, Cin, H, W, F):
    rng = np.random.default_rng(seed)
    x = rng.uniform(-1, 1, (B, Cin, H, W)).astype(np.float32)
    w = (rng.standard_normal((F, Cin * 9)) * np.sqrt(2.0 / (Cin * 9))).astype(np.float32)
    b = (rng.standard_normal(F) * 0.1).astype(np.float32)
    return x, w, b


SHAPES = [  # (B, C, H, W, F)
    (8, 64, 13, 13, 128),   # Wp 14: tiles straddle images
    (2, 32, 26, 26, 64),    # Wp 28
    (2, 16, 52, 52, 40),    # Wp 53, ragged filters
    (3, 8, 7, 7, 130),      # tiny images, F beyond one tile row
    (1, 12, 20, 33, 24),    # non-square, Wp 34
    (2, 4, 9, 5, 70),       # one stage, narrow rows
]


@pytest.mark.parametrize("tile", TILES)
def test_slide_bit_exact(ctx, tile, monkeypatch):
    monkeypatch.setenv("TB_EXACT_FORCE", str(tile))
    for i, (B, Cin, H, W, F) in enumerate(SHAPES):
        x, w, b = _case(300 + i, B, Cin, H, W, F)
        ref = O.conv2d(x, w, b, F, 3, 1, 1, 9)
        y1 = _conv(ctx, x, w, b, F)
        y2 = _conv(ctx, x, w, b, F)
        assert_bit_exact(y1, ref, B * F, (tile, i))
        assert np.array_equal(y1, y2)


@pytest.mark.parametrize("tile", [120, 123, 124, 127, 131, 133])
def test_slide_channel_slice_input(ctx, tile, monkeypatch):
    """The input is channels [0, C) of a tensor with 3C channels per image (in_batch_stride)."""
    monkeypatch.setenv("TB_EXACT_FORCE", str(tile))
    B, Cin, H, F = 3, 16, 26, 48
    rng = np.random.default_rng(9)
    wide = rng.uniform(-1, 1, (B, 3 * Cin, H, H)).astype(np.float32)
    w = (rng.standard_normal((F, Cin * 9)) * 0.1).astype(np.float32)
    b = np.zeros(F, np.float32)
    y = _conv(ctx, wide, w, b, F, x_bs=3 * Cin * H * H)
    ref = O.conv2d(np.ascontiguousarray(wide[:, :Cin]), w, b, F, 3, 1, 1, 9)
    assert_bit_exact(y, ref, B * F, "slice")


@pytest.mark.parametrize("tile", [121, 122, 125, 126, 132, 136])
def test_slide_residual_and_batchnorm(ctx, tile, monkeypatch):
    monkeypatch.setenv("TB_EXACT_FORCE", str(tile))
    B, Cin, H, F = 2, 32, 13, 64
    x, w, b = _case(11, B, Cin, H, H, F)
    rng = np.random.default_rng(12)
    r = rng.standard_normal((B, F, H, H)).astype(np.float32)
    y = _conv(ctx, x, w, b, F, residual=r)
    assert_bit_exact(y, O.shortcut(O.conv2d(x, w, b, F, 3, 1, 1, 9), r), B * F, "residual")
    bn = (rng.uniform(0.5, 1.5, F).astype(np.float32), (rng.standard_normal(F) * 0.1).astype(np.float32),
          rng.uniform(0.5, 1.5, F).astype(np.float32))
    y = _conv(ctx, x, w, b, F, bn=bn)
    assert_bit_exact(y, O.conv2d(x, w, b, F, 3, 1, 1, 9, bn=bn), B * F, "batchnorm")
