"""Memory-bound layers, XNOR conv and detection extraction: CUDA path vs the CPU oracle.
Bit-exact where the reference path is integer, an index or a pure copy."""
import ctypes as C

import numpy as np
import pytest
import torch

from conftest import assert_bit_exact
from oracle import oracle as O
from tensorium_b200._lib import check, lib
from tensorium_b200.context import ptr
from tensorium_b200 import synth
from tensorium_b200.layers import (TAddLayer, TAvgPoolLayer, TConcatLayer, TConnectedLayer, TMaxPoolLayer,
                                   TNNetState, TSoftmaxLayer, TUpSampleLayer, TXNORConvolutionLayer,
                                   TYoloLayer, get_detections)

pytestmark = pytest.mark.gpu


def dev(ctx, a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(ctx.torch_device)


@pytest.mark.parametrize("B,C,H,W,k,s,p", [(2, 8, 28, 28, 2, 2, 0), (3, 5, 7, 9, 2, 2, 0),
                                           (1, 4, 13, 13, 3, 1, 2), (2, 3, 10, 10, 3, 2, 1),
                                           (1, 2, 6, 6, 5, 1, 4)])
def test_maxpool_bit_exact_with_indexes(ctx, B, C, H, W, k, s, p):
    rng = np.random.default_rng(H * 10 + k)
    x = rng.integers(-3, 4, (B, C, H, W)).astype(np.float32)  # many ties
    L = TMaxPoolLayer(B, H, W, C, k, s, s, p).bind(ctx)
    idx = torch.empty((B, C, L.outH, L.outW), dtype=torch.int64, device=ctx.torch_device)
    y = L.forward(TNNetState(dev(ctx, x)), indexes=idx)
    ry, ridx = O.maxpool(x, k, s, p, want_index=True)
    assert np.array_equal(y.cpu().numpy(), ry)
    assert np.array_equal(idx.cpu().numpy(), ridx)


@pytest.mark.parametrize("B,C,H,W,s", [(2, 256, 13, 13, 2), (1, 3, 5, 7, 3), (2, 4, 6, 8, 2)])
def test_upsample_bit_exact(ctx, B, C, H, W, s):
    x = np.random.default_rng(1).standard_normal((B, C, H, W)).astype(np.float32)
    y = TUpSampleLayer(B, W, H, C, s).bind(ctx).forward(TNNetState(dev(ctx, x)))
    assert np.array_equal(y.cpu().numpy(), O.upsample(x, s))


def test_upsample_into_route_slice(ctx):
    B, C, H, W = 2, 4, 3, 4
    x = np.random.default_rng(2).standard_normal((B, C, H, W)).astype(np.float32)
    big = torch.zeros((B, 3 * C, 2 * H, 2 * W), device=ctx.torch_device)
    TUpSampleLayer(B, W, H, C, 2).bind(ctx).forward(TNNetState(dev(ctx, x)), out=big[:, C:], out_batch_stride=3 * C * 4 * H * W)
    got = big.cpu().numpy()
    assert np.array_equal(got[:, C:2 * C], O.upsample(x, 2))
    assert not got[:, :C].any() and not got[:, 2 * C:].any()


def test_route_per_sample_and_reference_concat(ctx):
    rng = np.random.default_rng(3)
    a = rng.standard_normal((3, 5, 4, 4)).astype(np.float32)
    b = rng.standard_normal((3, 2, 4, 4)).astype(np.float32)
    R = TConcatLayer(3, [0, 1], [a[0].size, b[0].size], per_sample=True).bind(ctx)
    y = R.forward_tensors([dev(ctx, a), dev(ctx, b)]).cpu().numpy()
    assert np.array_equal(y, np.concatenate([a, b], axis=1).reshape(3, -1))
    R.per_sample = False
    y2 = R.forward_tensors([dev(ctx, a), dev(ctx, b)]).cpu().numpy().ravel()
    assert np.array_equal(y2, O.concat([a, b]))  # TTensor.concat: whole tensors back to back


def test_shortcut_bit_exact(ctx):
    rng = np.random.default_rng(4)
    for n in (4096, 1001):
        a = rng.standard_normal(n).astype(np.float32)
        b = rng.standard_normal(n).astype(np.float32)
        for act in (4, 9):
            y = TAddLayer(1, [0], act).bind(ctx).forward_tensors(dev(ctx, a), dev(ctx, b))
            assert np.array_equal(y.cpu().numpy(), O.shortcut(a, b, act))


@pytest.mark.parametrize("scale_xy", [1.0, 1.05])
def test_yolo_forward(ctx, scale_xy):
    rng = np.random.default_rng(5)
    x = (rng.standard_normal((2, 255, 13, 13)) * 4).astype(np.float32)
    Y = TYoloLayer(2, 13, 13, 3, 9, [6, 7, 8], 80, scaleXY=scale_xy).bind(ctx)
    y = Y.forward(TNNetState(dev(ctx, x))).cpu().numpy()
    ref = O.yolo(x, 3, 80, scale_xy)
    assert np.max(np.abs(y - ref)) <= 2 ** -23 * 2  # logistic in double on both sides


def test_softmax_avgpool_connected(ctx):
    rng = np.random.default_rng(6)
    x = rng.standard_normal((64, 10)).astype(np.float32)
    y = TSoftmaxLayer(64, 10).bind(ctx).forward(TNNetState(dev(ctx, x))).cpu().numpy()
    assert np.max(np.abs(y - O.softmax(x))) <= 1e-7
    z = rng.standard_normal((8, 10, 4, 4)).astype(np.float32)
    a = TAvgPoolLayer(8, 4, 4, 10).bind(ctx).forward(TNNetState(dev(ctx, z))).cpu().numpy()
    assert np.array_equal(a, O.avgpool(z))
    xi = rng.uniform(0, 1, (256, 3136)).astype(np.float32)
    w = (rng.standard_normal((1024, 3136)) * 0.02).astype(np.float32)
    b = rng.standard_normal(1024).astype(np.float32) * 0.1
    fc = TConnectedLayer(256, 1, 3136, 1024, "relu", w, b).bind(ctx)
    yf = fc.forward(TNNetState(dev(ctx, xi))).cpu().numpy()
    assert_bit_exact(yf, O.connected(xi, w, b, 1), 256, "connected (sdot_avx2 order)")


@pytest.mark.parametrize("C,S,B", [(128, 13, 2), (256, 26, 1), (64, 7, 3), (40, 9, 2)])
@pytest.mark.parametrize("pad_mode", [0, 1])
def test_xnor_bit_exact(ctx, C, S, B, pad_mode):
    rng = np.random.default_rng(C + S)
    x = rng.standard_normal((B, C, S, S)).astype(np.float32)
    w = rng.standard_normal((C, C * 9)).astype(np.float32)
    L = TXNORConvolutionLayer(B, S, S, C, C, 3, 1, 1, "linear", pad_mode)
    L.upload(ctx, w)
    cnt = torch.empty((B, C, S, S), dtype=torch.int32, device=ctx.torch_device)
    y = L.forward(TNNetState(dev(ctx, x)), counts=cnt).cpu().numpy()
    mean = O.xnor_mean(w)
    assert np.array_equal(L.mean.cpu().numpy(), mean)
    rc, ry = O.xnor_conv(x, w, mean, C, 3, 1, 1, pad_mode)
    assert np.array_equal(cnt.cpu().numpy(), rc)
    assert np.array_equal(y, ry)


def test_detections_match_oracle_order_and_values(ctx):
    rng = np.random.default_rng(9)
    heads, outs, host = [], [], []
    for (g, mask) in ((13, [6, 7, 8]), (26, [3, 4, 5])):
        raw = (rng.standard_normal((2, 255, g, g)) * 2).astype(np.float32)
        act = O.yolo(raw, 3, 80)
        heads.append(TYoloLayer(2, g, g, 3, 9, mask, 80).bind(ctx))
        outs.append(dev(ctx, act))
        host.append((act, g, mask))
    recs, probs, counts = get_detections(ctx, heads, outs, 2, 640, 480, 416, 416, 0.45, relative=False,
                                         letter=True, capacity=8192)
    for b in range(2):
        exp_boxes, exp_meta, exp_probs, total = [], [], [], 0
        for hi, (act, g, mask) in enumerate(host):
            cnt, bx, meta, pr = O.yolo_detections(act, b, 3, 80, g, g, mask, synth.YOLO_ANCHORS, 640, 480,
                                                  416, 416, 0.45, relative=False, letter=True)
            total += cnt
            exp_boxes.append(bx)
            exp_meta.append(np.c_[np.full(len(meta), hi), meta[:, :2]])
            exp_probs.append(pr)
        assert counts[b] == total
        r = recs[b, :total]
        got_meta = np.c_[r["head"], r["index"], r["anchor"]]
        assert np.array_equal(got_meta, np.concatenate(exp_meta))  # index set and order bit-exact
        got_box = np.c_[r["x"], r["y"], r["w"], r["h"], r["objectness"]]
        np.testing.assert_allclose(got_box, np.concatenate(exp_boxes), rtol=1e-6, atol=1e-6)
        assert np.array_equal(probs[b, :total], np.concatenate(exp_probs))


@pytest.mark.parametrize("C", [128, 256, 512, 1024])
@pytest.mark.parametrize("S", [52, 26, 13])
def test_xnor_config4_batch64(ctx, C, S):
    """BASELINE config 4 at its full size: C_in = C_out = C, 3x3 s1 p1, S x S, batch 64.  The
    serial oracle checks images 0, 31 and 63 of the batch-64 launch bit for bit (popcounts and
    scaled outputs, the reference's bit-0 padding)."""
    B = 64
    rng = np.random.default_rng(1000 + C + S)
    w = rng.standard_normal((C, C * 9)).astype(np.float32)
    g = torch.Generator(device=ctx.torch_device).manual_seed(C * 100 + S)
    x = torch.randn((B, C, S, S), generator=g, device=ctx.torch_device)
    L = TXNORConvolutionLayer(B, S, S, C, C, 3, 1, 1, "linear", 0)
    L.upload(ctx, w)
    cnt = torch.empty((B, C, S, S), dtype=torch.int32, device=ctx.torch_device)
    y = L.forward(TNNetState(x), counts=cnt)
    mean = O.xnor_mean(w)
    for b in (0, 31, 63):
        rc, ry = O.xnor_conv(x[b:b + 1].cpu().numpy(), w, mean, C, 3, 1, 1, 0)
        assert np.array_equal(cnt[b:b + 1].cpu().numpy(), rc), b
        assert np.array_equal(y[b:b + 1].cpu().numpy(), ry), b
