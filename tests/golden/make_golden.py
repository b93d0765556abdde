"""Generate the golden fixtures in this directory from the CPU oracle (oracle/oracle.cpp, the
restatement of the reference's CPU path; the FreePascal reference itself cannot be run here, so
these pin the oracle against regressions and give the GPU tests fixed expected outputs).

    python tests/golden/make_golden.py

Every input is made by tensorium_b200.synth from a fixed seed."""
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))

from oracle import oracle as O  # noqa: E402
from tensorium_b200 import synth  # noqa: E402


def tiny_yolo_specs(seed=7, classes=3):
    """A small darknet net with every YOLOv3 layer kind: strided convs, 1x1/3x3 convs with BN,
    a shortcut, a single-input route, an upsample, a two-input route and two yolo heads."""
    A = synth.ACT
    nout = 3 * (classes + 5)
    L = [synth.conv_spec(seed, "t0", 3, 8, 3, 1, 1, A["leaky"], True),
         synth.conv_spec(seed, "t1", 8, 16, 3, 2, 1, A["leaky"], True),
         synth.conv_spec(seed, "t2", 16, 8, 1, 1, 0, A["leaky"], True),
         synth.conv_spec(seed, "t3", 8, 16, 3, 1, 1, A["leaky"], True),
         {"type": "shortcut", "from": -3, "activation": A["linear"]},
         synth.conv_spec(seed, "t5", 16, 32, 3, 2, 1, A["leaky"], True),
         synth.conv_spec(seed, "t6", 32, nout, 1, 1, 0, A["linear"], False),
         {"type": "yolo", "classes": classes, "mask": [3, 4, 5], "anchors": synth.YOLO_ANCHORS.copy(), "scale_xy": 1.0},
         {"type": "route", "layers": [-3]},
         synth.conv_spec(seed, "t9", 32, 16, 1, 1, 0, A["leaky"], True),
         {"type": "upsample", "stride": 2, "scale": 1.0},
         {"type": "route", "layers": [-1, 4]},
         synth.conv_spec(seed, "t12", 32, nout, 1, 1, 0, A["linear"], False),
         {"type": "yolo", "classes": classes, "mask": [0, 1, 2], "anchors": synth.YOLO_ANCHORS.copy(), "scale_xy": 1.0}]
    return L


def main():
    out = {}
    # conv: config-0 shape at reduced size, CRS path, unfused BN + leaky
    s = synth.config0_spec()[0]
    x = synth.input_images(0, "g.cfg0", 1, (3, 24, 24))
    out["conv_bn_x"], out["conv_bn_w"] = x, s["weights"]
    out["conv_bn_bn"] = np.stack([s["scales"], s["mean"], s["var"]])
    out["conv_bn_y"] = O.conv2d(x, s["weights"], s["biases"], 32, 3, 1, 1, 9, bn=(s["scales"], s["mean"], s["var"]))
    # conv: RSC path, stride 2, bias, leaky
    x2 = synth.input_images(1, "g.rsc", 2, (32, 14, 14))
    w2 = synth.normal(1, "g.rsc.w", (24, 32 * 9), 0, 0.08)
    b2 = synth.normal(1, "g.rsc.b", (24,), 0, 0.1)
    out["conv_rsc_x"], out["conv_rsc_w"], out["conv_rsc_b"] = x2, w2, b2
    out["conv_rsc_y"] = O.conv2d(x2, w2, b2, 24, 3, 2, 1, 9)
    # maxpool with argmax (ties)
    xm = np.floor(synth.uniform(2, "g.mp", (2, 3, 9, 9)) * 4).astype(np.float32)
    out["maxpool_x"] = xm
    out["maxpool_y"], out["maxpool_idx"] = O.maxpool(xm, 3, 2, 1, want_index=True)
    # xnor counts (bit-exact integer path)
    xx = synth.normal(3, "g.xnor.x", (1, 64, 7, 7))
    wx = synth.normal(3, "g.xnor.w", (16, 64 * 9))
    mean = O.xnor_mean(wx)
    out["xnor_x"], out["xnor_w"], out["xnor_mean"] = xx, wx, mean
    out["xnor_counts"], out["xnor_y"] = O.xnor_conv(xx, wx, mean, 16, 3, 1, 1, 0)
    # tiny yolo net, every layer, and its detections
    specs = tiny_yolo_specs()
    xn = synth.input_images(4, "g.tiny", 2, (3, 32, 32))
    outs = O.run_network(specs, xn)
    out["net_x"] = xn
    for i, v in outs.items():
        out[f"net_{i}"] = v
    cnt, boxes, meta, probs = O.yolo_detections(outs[13].reshape(2, 24, 16, 16), 0, 3, 3, 16, 16, [0, 1, 2],
                                                synth.YOLO_ANCHORS, 640, 480, 32, 32, 0.5, relative=False, letter=True)
    out["det_count"], out["det_boxes"], out["det_meta"], out["det_probs"] = np.int64(cnt), boxes, meta, probs
    np.savez_compressed(HERE / "golden_v1.npz", **out)
    print("wrote", HERE / "golden_v1.npz", sum(v.nbytes for v in out.values()), "bytes raw")


if __name__ == "__main__":
    main()
