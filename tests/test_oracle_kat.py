"""Known-answer tests of the CPU oracle against hand-derived results.

The reference ships no tests or golden vectors and cannot be compiled here (FreePascal), so
these hand-checkable cases are what pins the restatement (parity unpinned against the reference
itself)."""
import numpy as np
import pytest

from oracle import oracle as O

LEAKY, LINEAR, LOGISTIC, RELU = 9, 4, 0, 1


def naive_conv(x, w, stride, pad, dil=1):
    x = x.astype(np.float64)
    B, C, H, W = x.shape
    F = w.shape[0]
    k = int(round((w.shape[1] / C) ** 0.5))
    w = w.reshape(F, C, k, k).astype(np.float64)
    oh = (H + 2 * pad - (dil * (k - 1) + 1)) // stride + 1
    ow = (W + 2 * pad - (dil * (k - 1) + 1)) // stride + 1
    xp = np.zeros((B, C, H + 2 * pad, W + 2 * pad))
    xp[:, :, pad:pad + H, pad:pad + W] = x
    y = np.zeros((B, F, oh, ow))
    for r in range(k):
        for s in range(k):
            patch = xp[:, :, r * dil: r * dil + stride * (oh - 1) + 1: stride,
                       s * dil: s * dil + stride * (ow - 1) + 1: stride]
            y += np.einsum("bchw,fc->bfhw", patch, w[:, :, r, s])
    return y


@pytest.mark.parametrize("C,F,H,k,s,p,d", [(3, 8, 9, 3, 1, 1, 1), (5, 4, 10, 3, 2, 1, 1),
                                          (16, 7, 6, 1, 1, 0, 1), (2, 3, 11, 5, 1, 2, 1),
                                          (3, 2, 12, 3, 1, 2, 2), (4, 5, 7, 1, 2, 0, 1)])
def test_conv_matches_float64_convolution(C, F, H, k, s, p, d):
    rng = np.random.default_rng(C * 100 + H)
    x = rng.standard_normal((2, C, H, H)).astype(np.float32)
    w = rng.standard_normal((F, C * k * k)).astype(np.float32)
    y = O.conv2d(x, w, None, F, k, s, p, LINEAR, dilation=d)
    ref = naive_conv(x, w, s, p, d)
    assert y.shape == ref.shape
    assert np.max(np.abs(y - ref)) <= 1e-5 * max(1.0, np.max(np.abs(ref)))


def test_identity_kernel_reproduces_input():
    rng = np.random.default_rng(0)
    x = rng.standard_normal((1, 3, 7, 9)).astype(np.float32)
    w = np.zeros((3, 27), np.float32)
    for c in range(3):
        w[c, c * 9 + 4] = 1.0  # centre tap of channel c
    y = O.conv2d(x, w, None, 3, 3, 1, 1, LINEAR)
    assert np.array_equal(y, x)


def test_bias_bn_and_leaky_follow_the_reference_formulas():
    rng = np.random.default_rng(2)
    x = rng.standard_normal((1, 2, 5, 5)).astype(np.float32)
    w = np.zeros((2, 2), np.float32)
    w[0, 0] = 1.0
    w[1, 1] = 1.0  # 1x1 identity: the epilogue sees x itself
    b = np.array([0.25, -0.5], np.float32)
    sc = np.array([1.5, 0.75], np.float32)
    mu = np.array([0.1, -0.2], np.float32)
    var = np.array([0.8, 1.3], np.float32)
    y = O.conv2d(x, w, b, 2, 1, 1, 0, LEAKY, bn=(sc, mu, var))
    sd = np.sqrt(var.astype(np.float64)).astype(np.float32)
    t = ((x - mu[None, :, None, None]) / sd[None, :, None, None]).astype(np.float32)
    t = (t * sc[None, :, None, None]).astype(np.float32) + b[None, :, None, None]
    expect = np.where(t < 0, t * np.float32(0.1), t)
    assert np.array_equal(y, expect)


def test_activation_forms():
    x = np.array([-3.0, -0.5, -0.0, 0.0, 0.5, 7.0], np.float32)
    assert np.array_equal(O.activate(x, LEAKY), np.where(x < 0, x * np.float32(0.1), x))
    lg = (1.0 / (1.0 + np.exp(-x.astype(np.float64)))).astype(np.float32)
    assert np.array_equal(O.activate(x, LOGISTIC), lg)
    assert np.array_equal(O.activate(x, RELU), np.maximum(x, 0) * (x > 0))
    assert np.array_equal(O.activate(x, LINEAR), x)


def test_maxpool_planted_maxima_ties_and_indexes():
    x = np.zeros((1, 2, 4, 4), np.float32)
    x[0, 0, 1, 0] = 5.0
    x[0, 1] = 1.0  # all equal: the first element of each window wins
    y, idx = O.maxpool(x, 2, 2, 0, want_index=True)
    assert y[0, 0, 0, 0] == 5.0 and idx[0, 0, 0, 0] == 4  # flat index 1*4+0
    assert idx[0, 1, 1, 1] == 16 + 2 * 4 + 2
    # padding 1 with size 2 stride 1: offsets -padding div 2 = 0 -> windows reach past the edge
    y2, idx2 = O.maxpool(-np.ones((1, 1, 2, 2), np.float32), 2, 1, 1, want_index=True)
    assert y2.shape == (1, 1, 2, 2) and np.all(y2 == -1) and idx2[0, 0, 1, 1] == 3


def test_upsample_concat_shortcut_are_exact_copies():
    rng = np.random.default_rng(3)
    x = rng.standard_normal((2, 3, 2, 3)).astype(np.float32)
    u = O.upsample(x, 2)
    assert np.array_equal(u, x.repeat(2, axis=2).repeat(2, axis=3))
    a, b = x, rng.standard_normal(x.shape).astype(np.float32)
    assert np.array_equal(O.concat([a, b]), np.concatenate([a.ravel(), b.ravel()]))
    assert np.array_equal(O.shortcut(a, b), a + b)


def test_yolo_activates_all_entries_but_w_h():
    rng = np.random.default_rng(4)
    n, classes = 3, 2
    x = rng.standard_normal((1, n * (classes + 5), 2, 2)).astype(np.float32)
    y = O.yolo(x, n, classes)
    for a in range(n):
        for e in range(classes + 5):
            c = a * (classes + 5) + e
            if e in (2, 3):
                assert np.array_equal(y[0, c], x[0, c])
            else:
                assert np.array_equal(y[0, c], O.activate(x[0, c], LOGISTIC))


def test_detections_decode_one_planted_box():
    n, classes, h, w = 3, 2, 2, 2
    out = np.zeros((1, n * (classes + 5), h, w), np.float32)
    a, row, col = 1, 1, 0
    base = a * (classes + 5)
    out[0, base + 0, row, col] = 0.25
    out[0, base + 1, row, col] = 0.5
    out[0, base + 2, row, col] = 0.0  # exp(0) = 1
    out[0, base + 3, row, col] = np.log(2.0)
    out[0, base + 4, row, col] = 0.9
    out[0, base + 5 + 1, row, col] = 0.8
    anchors = np.arange(18, dtype=np.float32) + 1
    mask = [3, 4, 5]
    cnt, boxes, meta, probs = O.yolo_detections(out, 0, n, classes, h, w, mask, anchors, 416, 416, 416, 416, 0.5)
    assert cnt == 1
    assert tuple(meta[0][:2]) == (row * w + col, a)
    np.testing.assert_allclose(boxes[0], [0.125, 0.75, anchors[8] / 416, 2 * anchors[9] / 416, 0.9], rtol=1e-6)
    assert probs[0, 0] == 0 and probs[0, 1] == np.float32(0.9) * np.float32(0.8)


def test_softmax_and_avgpool():
    rng = np.random.default_rng(5)
    x = rng.standard_normal((3, 10)).astype(np.float32)
    s = O.softmax(x)
    np.testing.assert_allclose(s.sum(1), 1.0, rtol=1e-6)
    np.testing.assert_allclose(s, np.exp(x) / np.exp(x).sum(1, keepdims=True), rtol=1e-6)
    y = rng.standard_normal((2, 3, 4, 4)).astype(np.float32)
    np.testing.assert_allclose(O.avgpool(y), y.mean((2, 3)), rtol=1e-6, atol=1e-7)


def test_xnor_all_plus_one_counts():
    C, F, H = 32, 4, 5
    x = np.ones((1, C, H, H), np.float32)
    w = np.ones((F, C * 9), np.float32)
    mean = O.xnor_mean(w)
    assert np.all(mean == 1.0)
    cnt, y = O.xnor_conv(x, w, mean, F, 3, 1, 1, pad_mode=0)
    K = C * 9
    assert cnt[0, 0, 2, 2] == K  # interior: every bit matches
    assert cnt[0, 0, 0, 0] == K - 2 * 5 * C  # corner: 5 padded taps are bit 0 = mismatch
    assert cnt[0, 0, 0, 2] == K - 2 * 3 * C
    cnt1, _ = O.xnor_conv(x, w, mean, F, 3, 1, 1, pad_mode=1)
    assert cnt1[0, 0, 0, 0] == 4 * C and cnt1[0, 0, 2, 2] == K


def test_xnor_zero_pad_mode_equals_sign_convolution():
    rng = np.random.default_rng(6)
    C, F, H = 40, 6, 6
    x = rng.standard_normal((2, C, H, H)).astype(np.float32)
    w = rng.standard_normal((F, C * 9)).astype(np.float32)
    mean = O.xnor_mean(w)
    np.testing.assert_allclose(mean, np.abs(w).mean(1), rtol=1e-6)
    cnt, y = O.xnor_conv(x, w, mean, F, 3, 1, 1, pad_mode=1)
    ref = naive_conv(np.where(x > 0, 1.0, -1.0).astype(np.float32), np.where(w > 0, 1.0, -1.0).astype(np.float32), 1, 1)
    assert np.array_equal(cnt, ref.astype(np.int32))
    assert np.array_equal(y, cnt.astype(np.float32) * mean[None, :, None, None])


def test_nms_sort_known_answers():
    """TDetectionsHelper.doNMSSort restated: per class, the higher-probability box of an
    overlapping pair keeps its probability, the other's is zeroed; disjoint boxes and other
    classes are untouched; objectness-0 records take no part."""
    boxes = np.array([[0.50, 0.50, 0.20, 0.20],   # 0
                      [0.52, 0.50, 0.20, 0.20],   # 1 overlaps 0 (IoU ~0.82)
                      [0.10, 0.10, 0.05, 0.05],   # 2 disjoint
                      [0.51, 0.50, 0.20, 0.20]],  # 3 overlaps 0 and 1, objectness 0
                     np.float32)
    obj = np.array([0.9, 0.8, 0.7, 0.0], np.float32)
    probs = np.array([[0.6, 0.0], [0.7, 0.3], [0.5, 0.4], [0.0, 0.0]], np.float32)
    out, order = O.nms_sort(boxes, obj, probs, 0.45)
    assert np.array_equal(out, np.array([[0.0, 0.0], [0.7, 0.3], [0.5, 0.4], [0.0, 0.0]], np.float32))
    assert order[-1] == 3  # the objectness-0 record went to the end
    # above the IoU threshold nothing is suppressed
    out2, _ = O.nms_sort(boxes, obj, probs, 0.9)
    assert np.array_equal(out2, probs)
