"""The BF16-split tensor-core path (TB_MATH_BF16_SPLIT): YOLOv3 on tcgen05 kind::f16 MMAs whose
operands carry every fp32 value as a bf16 pair (hi + lo), against the FP32 oracle.

The north star's bar for a tensor-core path is relative L2 <= 1e-2 on the final heads with the
same top-k boxes.  Plain TF32 meets it on the random-weight net but not on a batchnorm-calibrated
one (its error compounds through 75 well-conditioned layers to ~1.5e-2, see test_gpu_net); the
split operands keep ~16 mantissa bits, so both nets stay orders of magnitude inside the bar."""
import ctypes as C

import numpy as np
import pytest
import torch

from netcheck import HEADS, calibrated_yolov3_specs, oracle_detections
from oracle import oracle as O
from tensorium_b200 import MATH_BF16_SPLIT, synth
from tensorium_b200._lib import lib
from tensorium_b200.net import TNNet

pytestmark = pytest.mark.gpu
TOL = 1e-2


def rel_l2(a, b, batch):
    a = np.asarray(a, np.float64).reshape(batch, -1)
    b = np.asarray(b, np.float64).reshape(batch, -1)
    return float((np.linalg.norm(a - b, axis=1) / np.linalg.norm(b, axis=1)).max())


@pytest.fixture(scope="module")
def calibrated():
    return calibrated_yolov3_specs()


@pytest.mark.parametrize("which", ["baseline", "calibrated"])
def test_yolov3_bf16split_heads(ctx, calibrated, which):
    specs = synth.yolov3_specs() if which == "baseline" else calibrated
    batch = 2
    x = synth.input_images(5, "yolov3", batch, (3, 416, 416))
    inner = [1, 36, 61, 85, 97]
    ref = O.run_network(specs, x, keep=HEADS + inner)
    net = TNNet(ctx, specs, batch, (3, 416, 416), math_mode=MATH_BF16_SPLIT)
    ps = C.c_int64()
    lib.tb_net_layer_layout(net.handle, 36, C.byref(ps))
    assert ps.value > 0, "the BF16-split network did not take the NHWC plan"
    xd = torch.from_numpy(x).to(ctx.torch_device)
    net.forward(xd, use_graph=False)
    for i in inner:
        e = rel_l2(net.output(i).cpu().numpy(), ref[i], batch)
        assert e <= 1e-3, (which, i, e)
    eager = [net.output(h).clone() for h in HEADS]
    errs = []
    for h, g in zip(HEADS, eager):
        e = rel_l2(g.cpu().numpy(), ref[h], batch)
        errs.append(e)
        assert e <= TOL, (which, h, e)
    print(which, "head relative L2:", errs)
    net.forward(xd, use_graph=True)
    for h, e in zip(HEADS, eager):
        assert torch.equal(net.output(h), e)
    if which == "calibrated":
        # the same boxes: the detection index sets equal, apart from candidates whose objectness
        # lies within 1e-3 of the threshold
        recs, probs, counts = net.detections(416, 416, 0.25, capacity=16384)
        exp = oracle_detections(ref, batch, 0.25)
        for b in range(batch):
            meta = exp[b][0]
            got = {(int(r["head"]), int(r["index"]), int(r["anchor"])) for r in recs[b, :counts[b]]}
            want = {tuple(int(v) for v in m) for m in meta}
            obj = {}
            for hi, h in enumerate(HEADS):
                o = ref[h].reshape(batch, 3, 85, -1)[b, :, 4]
                for a in range(3):
                    for i in range(o.shape[1]):
                        obj[(hi, i, a)] = o[a, i]
            for k in got ^ want:
                assert abs(obj[k] - 0.25) < 1e-3, (b, k, obj[k])
            assert len(want) > 100
    net.close()


@pytest.mark.parametrize("shape", ["256,1,2", "128,1,2"])
def test_yolov3_bf16split_cta_pairs(ctx, shape, monkeypatch):
    """Every conv of the BF16-split network on one CTA-pair tile shape (cta_group::2 kind::f16
    MMAs, pinned through the TB_NHWC_FORCE test hook): the heads stay within the bar."""
    monkeypatch.setenv("TB_NHWC_FORCE", shape)
    specs = synth.yolov3_specs()
    batch = 2
    x = synth.input_images(7, "yolov3", batch, (3, 416, 416))
    ref = O.run_network(specs, x, keep=HEADS)
    net = TNNet(ctx, specs, batch, (3, 416, 416), math_mode=MATH_BF16_SPLIT)
    net.forward(torch.from_numpy(x).to(ctx.torch_device), use_graph=False)
    for h in HEADS:
        e = rel_l2(net.output(h).cpu().numpy(), ref[h], batch)
        assert e <= 1e-3, (shape, h, e)
    net.close()
