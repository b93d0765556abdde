"""Class-wise NMS on the GPU (tb_yolo_nms, TDetectionsHelper.doNMSSort) against the oracle's
restatement of the reference (bit-exact when the probabilities of a class are distinct), and
against the stated tie rule (equal probabilities taken in detection order) when they are not."""
import ctypes as C

import numpy as np
import pytest
import torch

from oracle import oracle as O
from tensorium_b200.layers import DET_DTYPE, nms_sort

pytestmark = pytest.mark.gpu


def iou32(a, b):
    """box_iou in float32, the operation order of source/ntypes.pas:1059-1108 (b: many boxes)."""
    f = np.float32
    h = f(0.5)
    with np.errstate(all="ignore"):  # random-weight YOLO boxes can be inf / NaN; both sides agree
        return _iou32(a, b, f, h)


def _iou32(a, b, f, h):

    def overlap(x1, w1, x2, w2):
        l1, l2 = f(x1 - w1 * h), (x2 - w2 * h).astype(f)
        r1, r2 = f(x1 + w1 * h), (x2 + w2 * h).astype(f)
        return (np.minimum(r1, r2) - np.maximum(l1, l2)).astype(f)

    w = overlap(a[0], a[2], b[:, 0], b[:, 2])
    hh = overlap(a[1], a[3], b[:, 1], b[:, 3])
    i = np.where((w < 0) | (hh < 0), f(0), (w * hh).astype(f)).astype(f)
    u = ((f(a[2] * a[3]) + (b[:, 2] * b[:, 3]).astype(f)).astype(f) - i).astype(f)
    with np.errstate(divide="ignore", invalid="ignore"):
        r = np.where((i == 0) | (u == 0), f(0), (i / u).astype(f))
    return r.astype(f)


def nms_index_ties(boxes, obj, probs, thresh):
    """The reference's greedy suppression with equal probabilities taken in detection order."""
    probs = probs.copy()
    n, classes = probs.shape
    for k in range(classes):
        cand = [j for j in range(n) if obj[j] != 0 and probs[j, k] != 0]
        cand.sort(key=lambda j: (-probs[j, k], j))
        cand = np.array(cand, np.int64)
        supp = np.zeros(len(cand), bool)
        for i in range(len(cand) - 1):
            if supp[i]:
                continue
            ov = iou32(boxes[cand[i]], boxes[cand[i + 1:]]) > np.float32(thresh)
            supp[i + 1:] |= ov
        probs[cand[supp], k] = 0
    return probs


def to_device(ctx, boxes, obj, probs, capacity):
    n, classes = probs.shape
    rec = np.zeros(capacity, DET_DTYPE)
    rec["x"], rec["y"], rec["w"], rec["h"] = (np.pad(boxes[:, i], (0, capacity - n)) for i in range(4))
    rec["objectness"] = np.pad(obj, (0, capacity - n))
    d = torch.from_numpy(rec.view(np.uint8).copy()).to(ctx.torch_device)
    p = torch.zeros((capacity, classes), dtype=torch.float32)
    p[:n] = torch.from_numpy(probs)
    return d, p.to(ctx.torch_device)


def clustered(rng, n, classes, distinct):
    centers = rng.uniform(0.1, 0.9, (max(1, n // 6), 2))
    c = centers[rng.integers(0, len(centers), n)] + rng.normal(0, 0.02, (n, 2))
    wh = rng.uniform(0.05, 0.2, (n, 2))
    boxes = np.concatenate([c, wh], 1).astype(np.float32)
    obj = rng.uniform(0.5, 1.0, n).astype(np.float32)
    obj[rng.random(n) < 0.05] = 0.0
    if distinct:
        probs = rng.permutation(n * classes).reshape(n, classes).astype(np.float32) / (n * classes) + 0.01
    else:
        probs = rng.choice(np.array([0.25, 0.5, 0.75, 1.0], np.float32), (n, classes))
    probs[rng.random((n, classes)) < 0.6] = 0.0
    probs[obj == 0] = 0.0
    return boxes, obj, probs.astype(np.float32)


@pytest.mark.parametrize("n,classes", [(2, 1), (37, 3), (300, 8), (1500, 4)])
def test_nms_matches_reference_on_distinct_probabilities(ctx, n, classes):
    rng = np.random.default_rng(n + classes)
    boxes, obj, probs = clustered(rng, n, classes, distinct=True)
    ref, _ = O.nms_sort(boxes, obj, probs, 0.45)
    d, p = to_device(ctx, boxes, obj, probs, n + 5)
    nms_sort(ctx, d, p, [n], n + 5, classes, 0.45)
    got = p.cpu().numpy()[:n]
    assert np.array_equal(got, ref)
    assert (ref == 0).sum() > (probs == 0).sum() or n < 10  # something was suppressed


def test_nms_tie_rule_and_batch(ctx):
    """Tied probabilities (common when YOLO's logistic saturates), two images at once."""
    rng = np.random.default_rng(5)
    cap, classes = 700, 5
    imgs = [clustered(rng, 640, classes, distinct=False), clustered(rng, 311, classes, distinct=False)]
    ds, ps = zip(*[to_device(ctx, b, o, p, cap) for b, o, p in imgs])
    d, p = torch.cat(ds), torch.cat(ps)
    nms_sort(ctx, d, p, [640, 311], cap, classes, 0.5)
    got = p.cpu().numpy().reshape(2, cap, classes)
    for i, (b, o, pr) in enumerate(imgs):
        n = len(b)
        assert np.array_equal(got[i, :n], nms_index_ties(b, o, pr, 0.5)), i
        # where the class probabilities of overlapping boxes are not tied, the reference agrees
        ref, _ = O.nms_sort(b, o, pr, 0.5)
        assert (got[i, :n] == ref).mean() > 0.9


def test_yolov3_detections_then_nms(ctx):
    from tensorium_b200 import synth
    from tensorium_b200.net import TNNet
    specs = synth.yolov3_specs()
    x = synth.input_images(3, "yolov3", 1, (3, 416, 416))
    net = TNNet(ctx, specs, 1, (3, 416, 416))
    net.predict(x, layers=[106])
    recs, probs, counts = net.detections(416, 416, 0.45, capacity=8192)
    recs2, probs2, counts2 = net.detections(416, 416, 0.45, capacity=8192, nms=0.45)
    n = int(min(counts[0], 8192))
    assert counts2[0] == counts[0] and n > 0
    r = recs[0, :n]
    boxes = np.stack([r["x"], r["y"], r["w"], r["h"]], 1)
    want = nms_index_ties(boxes, r["objectness"], probs[0, :n], 0.45)
    assert np.array_equal(probs2[0, :n], want)
    net.close()
