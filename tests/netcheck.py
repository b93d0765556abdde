"""Helpers of the whole-network parity tests: a batchnorm-calibrated YOLOv3 and the detection
comparison against the oracle.  Test infrastructure (imports the oracle)."""
from __future__ import annotations

import copy
import functools

import numpy as np

from oracle import oracle as O
from tensorium_b200 import synth

HEADS, RAWS = [82, 94, 106], [81, 93, 105]
MASKS = {82: [6, 7, 8], 94: [3, 4, 5], 106: [0, 1, 2]}


@functools.lru_cache(maxsize=None)
def calibrated_yolov3_specs(seed: int = 3, calib_shape=(3, 128, 128)):
    """YOLOv3 with He-init weights whose batchnorm statistics are set from a forward pass: the
    running mean / variance of every batch-normalised conv are the per-channel mean / variance of
    its raw output on one synthetic calibration image (the oracle's conv, layer by layer).  The
    activations then stay O(1) through all 75 convs, so the yolo logistic outputs and objectness
    are not saturated (with the BASELINE statistics they reach ~1e5 and saturate to 0 / 1)."""
    specs = copy.deepcopy(synth.yolov3_specs(seed))
    x = synth.input_images(99, "calibration", 1, calib_shape)
    outs = {}

    def get(j):
        return outs[j]

    prev = x
    for i, s in enumerate(specs):
        if s["type"] == "conv" and s.get("batch_normalize"):
            raw = O.conv2d(prev, s["weights"], np.zeros(s["filters"], np.float32), s["filters"], s["size"],
                           s["stride"], s["pad"], 4)
            r = raw.reshape(raw.shape[1], -1).astype(np.float64)
            s["mean"] = r.mean(axis=1).astype(np.float32)
            s["var"] = np.maximum(r.var(axis=1), 1e-2).astype(np.float32)
            s["scales"] = np.ones(s["filters"], np.float32)
            s["biases"] = np.zeros(s["filters"], np.float32)
        outs[i] = O.run_layer(specs, i, prev, get)
        prev = outs[i]
    return specs


def oracle_detections(ref_heads, batch, thresh, img=(416, 416), net=(416, 416)):
    """Per image: (meta [head, index, anchor], boxes [x, y, w, h, objectness], probs) from the
    oracle's getDetections over the three heads, in the reference order."""
    res = []
    for b in range(batch):
        metas, boxes, probs = [], [], []
        for hi, h in enumerate(HEADS):
            out = ref_heads[h]
            g = int(round(np.sqrt(out.reshape(batch, -1).shape[1] // 255)))
            cnt, bx, meta, pr = O.yolo_detections(out.reshape(batch, 255, g, g), b, 3, 80, g, g, MASKS[h],
                                                  synth.YOLO_ANCHORS, img[0], img[1], net[0], net[1], thresh,
                                                  relative=True, letter=False)
            metas.append(np.c_[np.full(len(meta), hi), meta[:, :2]] if cnt else np.zeros((0, 3), np.int64))
            boxes.append(bx.reshape(-1, 5))
            probs.append(pr.reshape(-1, 80))
        res.append((np.concatenate(metas), np.concatenate(boxes), np.concatenate(probs)))
    return res


def assert_same_detections(net, ref_heads, batch, thresh=0.45):
    """GPU detection extraction on the network's heads against the oracle's on its heads: the
    same index set in the same order, boxes and probabilities within 1e-6."""
    recs, probs, counts = net.detections(416, 416, thresh, capacity=16384)
    exp = oracle_detections(ref_heads, batch, thresh)
    total = 0
    for b in range(batch):
        meta, bx, pr = exp[b]
        assert counts[b] == len(meta), (b, counts[b], len(meta))
        r = recs[b, :counts[b]]
        assert np.array_equal(np.c_[r["head"], r["index"], r["anchor"]], meta), b
        np.testing.assert_allclose(np.c_[r["x"], r["y"], r["w"], r["h"], r["objectness"]], bx, rtol=1e-6, atol=1e-6)
        np.testing.assert_allclose(probs[b, :counts[b]], pr, rtol=1e-6, atol=1e-7)
        total += len(meta)
    return total
