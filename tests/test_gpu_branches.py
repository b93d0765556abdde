"""The executor's branch schedule (layers off the longest remaining path on a second stream; FP32
NCHW plans, and the NHWC tensor-core plans with a workspace of the branch stream's own) changes only
when kernels run, never what they compute: every yolo output of YOLOv3 equals the one-stream
schedule's (TB_NET_BRANCHES=0), bit for bit, eager and graph-replayed (the tensor-core plans' split-K
fix-up is deterministic)."""
import numpy as np
import pytest
import torch

from tensorium_b200 import Context, MATH_BF16_SPLIT, MATH_FP32, MATH_TF32, synth
from tensorium_b200.net import TNNet

pytestmark = pytest.mark.gpu

INPUT = (3, 416, 416)


def _heads(ctx, x, use_graph, mm):
    net = TNNet(ctx, synth.yolov3_specs(), x.shape[0], INPUT, math_mode=mm)
    outs = []
    for g in (use_graph, use_graph):  # twice: the second graph replay reuses the captured graph
        net.forward(x, use_graph=g)
        torch.cuda.synchronize()
        outs.append([net.output(i).cpu().numpy().copy() for i in net.yolo_layers])
    net.close()
    return outs


@pytest.mark.parametrize("mm", [MATH_FP32, MATH_TF32, MATH_BF16_SPLIT])
@pytest.mark.parametrize("use_graph", [False, True])
def test_branch_schedule_is_bit_identical(use_graph, mm, monkeypatch):
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    # the tensor-core plans' split choices come from the cost model in both networks (a measured
    # choice could differ between them and change the summation order)
    monkeypatch.setenv("TB_AUTOTUNE", "0")
    ctx = Context(0)
    x = torch.from_numpy(synth.input_images(5, "yolov3", 2, INPUT)).to(ctx.torch_device)
    two = _heads(ctx, x, use_graph, mm)
    monkeypatch.setenv("TB_NET_BRANCHES", "0")
    one = _heads(ctx, x, use_graph, mm)
    for a_run, b_run in zip(two, one):
        for a, b in zip(a_run, b_run):
            assert np.array_equal(a, b)
    ctx.close()
