"""DetectionGather (the per-step detection extraction + gather to rank 0 through the C ABI), one rank.

The overlapped mode snapshots the yolo outputs and extracts / gathers / downloads on a side stream
while the next forward runs; its records must equal the serialized mode's for the same forward, even
when the next forward (on other images) overwrites the yolo outputs right after the step."""
import numpy as np
import pytest
import torch

from tensorium_b200 import Context, MATH_FP32, synth
from tensorium_b200 import dist as tbd
from tensorium_b200.net import TNNet

pytestmark = pytest.mark.gpu

INPUT = (3, 416, 416)


def _same(a, b):
    assert len(a) == len(b)
    for ra, rb in zip(a, b):
        assert ra.shape == rb.shape and ra.tobytes() == rb.tobytes()


def test_overlapped_gather_matches_serialized():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    ctx = Context(0)
    B = 2
    net = TNNet(ctx, synth.yolov3_specs(), B, INPUT, math_mode=MATH_FP32)
    xs = [torch.from_numpy(synth.input_images(s, "yolov3", B, INPUT)).to(ctx.torch_device) for s in (3, 4)]
    plain = tbd.DetectionGather(net, 1, 0, capacity=4096, thresh=0.1)
    ov = tbd.DetectionGather(net, 1, 0, capacity=4096, thresh=0.1, overlap=True)
    ref = []
    for x in xs:
        net.forward(x)
        plain.step(download=True)
        plain.wait()
        ref.append(plain.unpack())
    assert sum(len(r) for r in ref[0]) > 0
    # overlapped: the second forward is queued right behind the first step's snapshot
    net.forward(xs[0])
    ov.step(download=True)
    net.forward(xs[1])
    ov.join()
    ov.wait()
    _same(ov.unpack(), ref[0])
    ov.step(download=True)
    ov.join()
    ov.wait()
    _same(ov.unpack(), ref[1])
    plain.close()
    ov.close()
    net.close()
    ctx.close()
