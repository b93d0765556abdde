"""The first layer of the tensor-core (NHWC) network plans computed directly from the NCHW input
into its NHWC output (one FP32 FMA chain per output over TF32-rounded operands, or exact fp32
operands in BF16-split mode), against the CPU oracle and against the receptive-field route
(TB_FIRST_DIRECT=0: the input converted to receptive-field rows, then a 1x1 tensor-core conv)."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from tensorium_b200 import MATH_BF16_SPLIT, MATH_TF32, synth
from tensorium_b200.net import TNNet

pytestmark = pytest.mark.gpu


def rel_l2(a, b, batch):
    a = np.asarray(a, np.float64).reshape(batch, -1)
    b = np.asarray(b, np.float64).reshape(batch, -1)
    return float((np.linalg.norm(a - b, axis=1) / np.linalg.norm(b, axis=1)).max())


def specs_for(c, f, k, stride, size):
    s0 = synth.conv_spec(11, "first", c, f, k, stride, (k - 1) // 2, synth.ACT["leaky"], False)
    s0["biases"] = synth.normal(11, "first.b", (f,), 0.0, 0.1)
    s1 = synth.conv_spec(11, "second", f, 64, 3, 1, 1, synth.ACT["leaky"], False)
    return [s0, s1], (c, size, size)


# (C, F, k, stride, input size): YOLOv3's 3 -> 32 3x3; a ragged filter count at stride 2; a
# one-channel 5x5 (K = 25)
CASES = [(3, 32, 3, 1, 96), (3, 40, 3, 2, 130), (1, 96, 5, 1, 72)]


@pytest.mark.parametrize("C,F,k,stride,size", CASES)
@pytest.mark.parametrize("math", [MATH_TF32, MATH_BF16_SPLIT])
def test_first_layer_direct(ctx, monkeypatch, C, F, k, stride, size, math):
    specs, shape = specs_for(C, F, k, stride, size)
    batch = 2
    x = synth.input_images(4, "first", batch, shape)
    ref = O.run_network(specs, x, keep=[0, 1])
    xd = torch.from_numpy(x).to(ctx.torch_device)
    outs = {}
    for route in ("1", "0"):
        monkeypatch.setenv("TB_FIRST_DIRECT", route)
        net = TNNet(ctx, specs, batch, shape, math_mode=math)
        net.forward(xd, use_graph=False)
        outs[route] = [net.output(i).cpu().numpy() for i in (0, 1)]
        net.forward(xd, use_graph=True)
        assert np.array_equal(net.output(0).cpu().numpy(), outs[route][0])
        net.close()
    d0 = outs["1"][0]
    e0 = rel_l2(d0, ref[0], batch)
    if math == MATH_BF16_SPLIT:
        # exact fp32 operands, one FMA chain per output: rounding-level distance from the oracle
        # (plus the pair encoding of the stored value, 16 mantissa bits)
        assert e0 <= 2e-5, e0
    else:
        assert e0 <= 1e-3, e0  # TF32 operands
    assert rel_l2(outs["0"][0], ref[0], batch) <= 1e-3
    assert rel_l2(d0, outs["0"][0], batch) <= 1e-3
    assert rel_l2(outs["1"][1], ref[1], batch) <= 1e-2
