"""TF32 tensor-core conv on NHWC activations (A operand by TMA im2col) through the C ABI against
the CPU oracle: relative L2 <= 1e-2 per activation map (the TF32 bar), for every output layout
(NHWC, NHWC into a channel slice, NCHW), residual, stride, dilation, kernel size and ragged
channel / filter counts."""
import ctypes as C

import numpy as np
import pytest
import torch

from oracle import oracle as O
from tensorium_b200._lib import ConvDesc, check, lib
from tensorium_b200.context import ptr

pytestmark = pytest.mark.gpu

TF32_TOL = 1e-2


def rel_l2_maps(a, b, maps):
    a = np.asarray(a, np.float64).reshape(maps, -1)
    b = np.asarray(b, np.float64).reshape(maps, -1)
    assert np.all(np.isfinite(a))
    num = np.sqrt(((a - b) ** 2).sum(axis=1))
    den = np.maximum(np.sqrt((b ** 2).sum(axis=1)), 1e-30)
    return float((num / den).max())


def run_nhwc(ctx, x, w, b, F, k, s, p, act, dil=1, residual=None, out="nhwc", y_extra=0):
    """x: NCHW numpy; runs the NHWC kernel on its NHWC copy; returns the output as NCHW numpy."""
    B, Cc, H, W = x.shape
    OH = (H + 2 * p - dil * (k - 1) - 1) // s + 1
    OW = (W + 2 * p - dil * (k - 1) - 1) // s + 1
    dev = ctx.torch_device
    xn = torch.from_numpy(np.ascontiguousarray(x.transpose(0, 2, 3, 1))).to(dev)
    d = ConvDesc(B, Cc, H, W, F, k, k, s, s, p, p, dil, dil, act, 0, F * OH * OW, 0)
    cnt = C.c_int64()
    check(lib.tb_conv_nhwc_packed_count(C.byref(d), C.byref(cnt)))
    wd = torch.from_numpy(np.ascontiguousarray(w)).to(dev)
    wp = torch.empty(cnt.value, device=dev)
    check(lib.tb_conv_pack_weights_nhwc(ctx.handle, C.byref(d), ptr(wd), ptr(wp)))
    bd = torch.from_numpy(b).to(dev)
    rd, rps = None, 0
    if residual is not None:
        rd = torch.from_numpy(np.ascontiguousarray(residual.transpose(0, 2, 3, 1))).to(dev)
        rps = F
    if out == "nchw":
        y = torch.full((B, F, OH, OW), float("nan"), device=dev)
        check(lib.tb_conv2d_fwd_nhwc(ctx.handle, C.byref(d), ptr(xn), Cc, ptr(wp), ptr(bd), None, 0, ptr(y), 0))
        return y.cpu().numpy()
    yps = F + y_extra
    ybuf = torch.full((B, OH, OW, yps), -7.0, device=dev)
    yv = ybuf[..., y_extra:]  # the output sits at channel offset y_extra of a wider buffer
    check(lib.tb_conv2d_fwd_nhwc(ctx.handle, C.byref(d), ptr(xn), Cc, ptr(wp), ptr(bd),
                                 ptr(rd) if rd is not None else None, rps, yv.data_ptr(), yps))
    if y_extra:
        assert torch.all(ybuf[..., :y_extra] == -7.0)
    return yv.permute(0, 3, 1, 2).cpu().numpy()


CASES = [  # (B, C, H, F, k, s, p, dil)
    (4, 64, 26, 128, 3, 1, 1, 1),     # 3x3, BN = 128
    (2, 128, 52, 256, 3, 1, 1, 1),    # YOLOv3 52x52 stage shape, BN = 256
    (2, 32, 104, 64, 3, 2, 1, 1),     # stride 2 (downsampling), C = 32
    (8, 512, 13, 1024, 3, 1, 1, 1),   # 13x13: tiles span images, long K
    (4, 256, 26, 128, 1, 1, 0, 1),    # 1x1
    (3, 48, 30, 40, 3, 1, 1, 1),      # C = 48 (zero-filled to 64), F = 40 (BN = 64, ragged)
    (2, 64, 33, 96, 5, 1, 2, 1),      # 5x5, odd size
    (2, 64, 40, 64, 3, 1, 2, 2),      # dilation 2
    (2, 96, 27, 80, 3, 2, 1, 1),      # stride 2, odd input
]


@pytest.mark.parametrize("B,C,H,F,k,s,p,dil", CASES)
def test_nhwc_conv_matches_oracle(ctx, B, C, H, F, k, s, p, dil):
    rng = np.random.default_rng(B * 7 + C + F)
    x = rng.uniform(0, 1, (B, C, H, H)).astype(np.float32)
    w = (rng.standard_normal((F, C * k * k)) * np.sqrt(2.0 / (C * k * k))).astype(np.float32)
    b = rng.standard_normal(F).astype(np.float32) * 0.1
    ref = O.conv2d(x, w, b, F, k, s, p, 9, dilation=dil)
    y = run_nhwc(ctx, x, w, b, F, k, s, p, 9, dil=dil)
    assert y.shape == ref.shape
    e = rel_l2_maps(y, ref, B * F)
    assert 0.0 < e <= TF32_TOL, e


def test_nhwc_output_layouts_and_residual(ctx):
    rng = np.random.default_rng(5)
    B, Cc, H, F = 2, 64, 26, 96
    x = rng.uniform(0, 1, (B, Cc, H, H)).astype(np.float32)
    w = (rng.standard_normal((F, Cc * 9)) * 0.05).astype(np.float32)
    b = rng.standard_normal(F).astype(np.float32) * 0.1
    ref = O.conv2d(x, w, b, F, 3, 1, 1, 9)
    # NCHW output (the yolo head layout)
    assert rel_l2_maps(run_nhwc(ctx, x, w, b, F, 3, 1, 1, 9, out="nchw"), ref, B * F) <= TF32_TOL
    # output in a channel slice of a wider NHWC buffer (a zero-copy route)
    assert rel_l2_maps(run_nhwc(ctx, x, w, b, F, 3, 1, 1, 9, y_extra=32), ref, B * F) <= TF32_TOL
    # residual (shortcut) added after the activation
    r = rng.standard_normal((B, F, H, H)).astype(np.float32)
    y = run_nhwc(ctx, x, w, b, F, 3, 1, 1, 9, residual=r)
    assert rel_l2_maps(y, O.shortcut(ref, r), B * F) <= TF32_TOL


def test_nhwc_rejects_what_it_cannot_take(ctx):
    d = ConvDesc(1, 8, 8, 8, 8, 3, 3, 1, 1, 1, 1, 1, 1, 4, 0, 0, 0)  # 2 KB input: under 128 KB
    x = torch.zeros(1024, device=ctx.torch_device)
    rc = lib.tb_conv2d_fwd_nhwc(ctx.handle, C.byref(d), ptr(x), 8, ptr(x), None, None, 0, ptr(x), 8)
    assert rc < 0


@pytest.mark.parametrize("shape", ["32,1", "32,3", "64,1", "128,1", "256,1", "256,3", "128,2", "64,4", "256,8",
                                   "128,1,2", "256,1,2"])
def test_nhwc_every_tile_shape(ctx, shape, monkeypatch):
    """Each (filters per tile, K splits, CTAs per tile) shape, pinned through the TB_NHWC_FORCE test
    hook; the tiles past the last whole wave are split, and a split tile is summed by its last
    arriving unit in split order, so two runs are identical. The CTA-pair shapes (cta_group::2, 256 pixels per tile) meet geometries whose last
    tile leaves the odd CTA's pixels wholly past the end and filters past F in the odd CTA's half."""
    monkeypatch.setenv("TB_NHWC_FORCE", shape)
    ctx.reserve(256 << 20)  # room for the split-K partial tiles
    rng = np.random.default_rng(31)
    # (8, 64, 52, 72): more tiles than SMs, so split shapes store whole waves and split the rest
    for (B, Cc, H, F, k, s, p) in [(2, 128, 26, 256, 3, 1, 1), (8, 512, 13, 160, 3, 1, 1), (2, 64, 52, 96, 1, 1, 0),
                                   (2, 64, 40, 72, 3, 2, 1), (8, 64, 52, 72, 3, 1, 1)]:
        x = rng.uniform(0, 1, (B, Cc, H, H)).astype(np.float32)
        w = (rng.standard_normal((F, Cc * k * k)) * np.sqrt(2.0 / (Cc * k * k))).astype(np.float32)
        b = rng.standard_normal(F).astype(np.float32) * 0.1
        r = rng.standard_normal((B, F, (H + 2 * p - k) // s + 1, (H + 2 * p - k) // s + 1)).astype(np.float32)
        y1 = run_nhwc(ctx, x, w, b, F, k, s, p, 9, residual=r)
        y2 = run_nhwc(ctx, x, w, b, F, k, s, p, 9, residual=r)
        assert np.array_equal(y1, y2), (shape, Cc)
        ref = O.shortcut(O.conv2d(x, w, b, F, k, s, p, 9), r)
        e = rel_l2_maps(y1, ref, B * F)
        assert 0.0 < e <= TF32_TOL, (shape, Cc, e)
