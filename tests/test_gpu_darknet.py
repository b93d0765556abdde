"""Networks loaded from darknet .cfg / .weights files (tb_darknet_load) on the GPU.

A net loaded from the files that oracle/darknet.py writes for a layer specification runs the
same kernels on the same arrays as the net built from the specification, so its outputs must be
identical bit for bit; the YOLOv3 heads are also checked against the CPU oracle (the FP32 path is
order-exact: w/h entries identical, logistic entries within 1 ulp)."""
import numpy as np
import pytest
import torch

from conftest import assert_bit_exact, assert_yolo_parity
from oracle import darknet as D
from oracle import oracle as O
from tensorium_b200 import synth
from tensorium_b200.net import TNNet

pytestmark = pytest.mark.gpu


def files(tmp_path, specs, shape, batch):
    c, w = tmp_path / "m.cfg", tmp_path / "m.weights"
    D.write(specs, shape, c, w, batch)
    return c, w


def test_yolov3_from_darknet_files(ctx, tmp_path):
    specs = synth.yolov3_specs()
    shape = (3, 416, 416)
    cfg, wts = files(tmp_path, specs, shape, 2)
    net = TNNet.from_darknet(ctx, cfg, wts)
    assert net.batch == 2 and net.input_shape == shape and net.yolo_layers == [82, 94, 106]
    ref_net = TNNet(ctx, specs, 2, shape)
    x = synth.input_images(3, "yolov3", 2, shape)
    heads = [82, 94, 106]
    got = net.predict(x, layers=heads)
    want = ref_net.predict(x, layers=heads)
    for g, w in zip(got, want):
        assert np.array_equal(g, w)
    ref = O.run_network(specs, x, keep=heads + [81, 93, 105])
    for h, g in zip(heads, got):
        assert_yolo_parity(g.reshape(ref[h].shape), ref[h], 3, 80, h)
    a = net.detections(416, 416, 0.45, capacity=16384, nms=0.45)
    b = ref_net.detections(416, 416, 0.45, capacity=16384, nms=0.45)
    assert np.array_equal(a[2], b[2])
    for i, n in enumerate(a[2]):
        assert np.array_equal(a[0][i, :n].view(np.uint8), b[0][i, :n].view(np.uint8))
        assert np.array_equal(a[1][i, :n], b[1][i, :n])
    net.close()
    ref_net.close()


def test_mnist_from_darknet_files(ctx, tmp_path):
    """Connected weights stored transposed (major > 1000) load to the same network."""
    specs = synth.mnist_specs()
    shape = (1, 28, 28)
    c, w = tmp_path / "m.cfg", tmp_path / "m.weights"
    c.write_text(D.cfg_text(specs, shape, 64))
    w.write_bytes(D.weights_bytes(specs, major=1001, minor=0))
    net = TNNet.from_darknet(ctx, c, w)
    x = synth.input_images(1, "mnist", 64, shape)
    ref = O.run_network(specs, x, keep=[4, 5, 6])
    out = net.predict(x, layers=[4, 5, 6])
    for got, i in zip(out[:2], (4, 5)):
        assert_bit_exact(got.reshape(ref[i].shape), ref[i], 64, i)
    assert np.abs(out[2] - ref[6]).max() <= 1e-7
    net.close()


def test_host_only_net_cannot_run(tmp_path):
    specs = synth.config0_spec()
    c, w = files(tmp_path, specs, (3, 416, 416), 1)
    net = TNNet.from_darknet(None, c, w)
    with pytest.raises(Exception):
        net.forward(torch.zeros((1, 3, 416, 416), device="cuda"))
    net.close()
