"""Committed golden fixtures (tests/golden/golden_v1.npz, made by tests/golden/make_golden.py):
the oracle must reproduce them bit for bit (CPU), and the CUDA path must match them within the
FP32 tolerance, bit-exactly for the integer / index / copy parts (GPU)."""
import importlib.util
from pathlib import Path

import numpy as np
import pytest

from conftest import assert_bit_exact, assert_yolo_parity
from oracle import oracle as O
from tensorium_b200 import synth

G = np.load(Path(__file__).parent / "golden" / "golden_v1.npz")


def _tiny_specs():
    spec = importlib.util.spec_from_file_location("make_golden", Path(__file__).parent / "golden" / "make_golden.py")
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    return m.tiny_yolo_specs()


def test_oracle_reproduces_golden_layers():
    s = synth.config0_spec()[0]
    bn = tuple(G["conv_bn_bn"])
    assert np.array_equal(O.conv2d(G["conv_bn_x"], G["conv_bn_w"], s["biases"], 32, 3, 1, 1, 9, bn=bn), G["conv_bn_y"])
    assert np.array_equal(O.conv2d(G["conv_rsc_x"], G["conv_rsc_w"], G["conv_rsc_b"], 24, 3, 2, 1, 9), G["conv_rsc_y"])
    y, idx = O.maxpool(G["maxpool_x"], 3, 2, 1, want_index=True)
    assert np.array_equal(y, G["maxpool_y"]) and np.array_equal(idx, G["maxpool_idx"])
    cnt, yx = O.xnor_conv(G["xnor_x"], G["xnor_w"], G["xnor_mean"], 16, 3, 1, 1, 0)
    assert np.array_equal(cnt, G["xnor_counts"]) and np.array_equal(yx, G["xnor_y"])
    assert np.array_equal(O.xnor_mean(G["xnor_w"]), G["xnor_mean"])


def test_oracle_reproduces_golden_network():
    specs = _tiny_specs()
    outs = O.run_network(specs, G["net_x"])
    for i, v in outs.items():
        assert np.array_equal(v, G[f"net_{i}"]), i
    cnt, boxes, meta, probs = O.yolo_detections(outs[13].reshape(2, 24, 16, 16), 0, 3, 3, 16, 16, [0, 1, 2],
                                                synth.YOLO_ANCHORS, 640, 480, 32, 32, 0.5, relative=False, letter=True)
    assert cnt == int(G["det_count"]) and np.array_equal(meta, G["det_meta"])
    assert np.array_equal(boxes, G["det_boxes"]) and np.array_equal(probs, G["det_probs"])


@pytest.mark.gpu
def test_gpu_matches_golden_network(ctx):
    from tensorium_b200.net import TNNet
    specs = _tiny_specs()
    shapes = synth.layer_shapes(specs, (3, 32, 32))
    net = TNNet(ctx, specs, 2, (3, 32, 32), fusion=False)
    import torch
    net.forward(torch.from_numpy(G["net_x"]).to(ctx.torch_device), use_graph=False)
    for i, s in enumerate(specs):
        got = net.output(i).cpu().numpy()
        ref = G[f"net_{i}"]
        if s["type"] == "yolo":
            assert_yolo_parity(got.reshape(ref.shape), ref, 3, 3, i)
        else:
            assert_bit_exact(got.reshape(ref.shape), ref, 2 * shapes[i][0], i)
    recs, probs, counts = net.detections(640, 480, 0.5, relative=False, letter=True, capacity=4096)
    # heads: the last yolo layer only in the golden record (image 0)
    heads, outs = net.yolo_heads()
    from tensorium_b200.layers import get_detections
    r2, p2, c2 = get_detections(ctx, heads[1:], outs[1:], 2, 640, 480, 32, 32, 0.5, False, True, 4096)
    k = int(G["det_count"])
    assert c2[0] == k
    got_meta = np.c_[r2[0, :k]["index"], r2[0, :k]["anchor"]]
    assert np.array_equal(got_meta, G["det_meta"][:, :2])
