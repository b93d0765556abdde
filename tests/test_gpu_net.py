"""Whole networks on the GPU executor against the CPU oracle.

The FP32 path is order-exact, so every conv / shortcut / route / upsample output of a network is
compared bit for bit, free running (each layer fed the GPU's own previous output) as well as
teacher forced; yolo outputs: w/h entries bit for bit, logistic entries within 1 ulp.  Covered:
YOLOv3-416 at batch 1, 2 and the benched configuration (batch 8, fused plan, measured tile
choices, CUDA-graph replay), a batchnorm-calibrated YOLOv3 whose heads are not saturated (exact
detections; TF32 path within its bar), and the MNIST- and CIFAR-shaped configs."""
import numpy as np
import pytest
import torch

from conftest import assert_bit_exact, assert_yolo_parity, logistic_ulps
from netcheck import HEADS, RAWS, assert_same_detections, calibrated_yolov3_specs
from oracle import oracle as O
from tensorium_b200 import MATH_TF32, synth
from tensorium_b200.net import TNNet

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def yolo_specs():
    return synth.yolov3_specs()


def maps_of(specs, shape, i, batch=1):
    return batch * synth.layer_shapes(specs, shape)[i][0]


def test_yolov3_every_layer_teacher_forced(ctx, yolo_specs):
    """Every layer of YOLOv3-416 (unfused plan, batch 1), each checked against the oracle run on
    the GPU's own inputs to that layer."""
    shape = (3, 416, 416)
    shapes = synth.layer_shapes(yolo_specs, shape)
    x = synth.input_images(3, "yolov3", 1, shape)
    net = TNNet(ctx, yolo_specs, 1, shape, fuse_batchnorm=True, fusion=False)
    net.forward(torch.from_numpy(x).to(ctx.torch_device), use_graph=False)
    outs = {}

    def get(j):
        if j not in outs:
            outs[j] = net.output(j).cpu().numpy().reshape((1,) + shapes[j])
        return outs[j]

    for i, s in enumerate(yolo_specs):
        prev = x if i == 0 else get(i - 1)
        ref = O.run_layer(yolo_specs, i, prev, get)
        if s["type"] == "yolo":
            assert_yolo_parity(get(i), ref, 3, 80, i)
        else:
            assert_bit_exact(get(i), ref, shapes[i][0], (i, s["type"]))


def test_yolov3_free_running_bit_exact(ctx, yolo_specs):
    """Free-running forward (unfused plan) against the free-running oracle: all 104 non-yolo
    layer outputs identical -- no error accumulates, although the random-weight activations grow
    to ~1e5."""
    shape = (3, 416, 416)
    x = synth.input_images(3, "yolov3", 1, shape)
    ref = O.run_network(yolo_specs, x)
    net = TNNet(ctx, yolo_specs, 1, shape, fuse_batchnorm=True, fusion=False)
    net.forward(torch.from_numpy(x).to(ctx.torch_device), use_graph=False)
    for i, s in enumerate(yolo_specs):
        got = net.output(i).cpu().numpy()
        if s["type"] == "yolo":
            assert_yolo_parity(got.reshape(ref[i].shape), ref[i], 3, 80, i)
        else:
            assert_bit_exact(got.reshape(ref[i].shape), ref[i], maps_of(yolo_specs, shape, i), (i, s["type"]))


@pytest.mark.parametrize("batch", [1, 2])
def test_yolov3_fused_heads_and_detections(ctx, yolo_specs, batch):
    x = synth.input_images(3, "yolov3", batch, (3, 416, 416))
    ref = O.run_network(yolo_specs, x, keep=HEADS)
    net = TNNet(ctx, yolo_specs, batch, (3, 416, 416))
    out = net.predict(x, layers=HEADS)
    for h, got in zip(HEADS, out):
        assert_yolo_parity(got.reshape(ref[h].shape), ref[h], 3, 80, h)
    assert assert_same_detections(net, ref, batch) > 0


def test_yolov3_benched_configuration(ctx, yolo_specs):
    """The configuration bench.py times: YOLOv3-416, batch 8, fused plan (shortcuts as residual
    epilogues, yolo logistic in the head convs, zero-copy routes), tile shapes measured at
    set-up, CUDA-graph replay -- the three heads against the oracle run image by image, and the
    detections."""
    batch = 8
    x = synth.input_images(3, "yolov3", batch, (3, 416, 416))
    net = TNNet(ctx, yolo_specs, batch, (3, 416, 416))
    xd = torch.from_numpy(x).to(ctx.torch_device)
    for _ in range(2):
        net.forward(xd, use_graph=True)
    torch.cuda.synchronize()
    got = {h: net.output(h).cpu().numpy() for h in HEADS}
    ref = {h: [] for h in HEADS}
    for b in range(batch):
        r = O.run_network(yolo_specs, x[b:b + 1], keep=HEADS)
        for h in HEADS:
            ref[h].append(r[h])
    ref = {h: np.concatenate(v) for h, v in ref.items()}
    for h in HEADS:
        assert_yolo_parity(got[h].reshape(ref[h].shape), ref[h], 3, 80, h)
    assert assert_same_detections(net, ref, batch) > 0
    net.close()


@pytest.fixture(scope="module")
def calibrated():
    return calibrated_yolov3_specs()


def test_calibrated_yolov3_fp32_detections(ctx, calibrated):
    """Batchnorm-calibrated YOLOv3 (activations O(1), objectness spread over (0, 1)): heads and
    detections of the fused batch-2 forward equal the oracle's."""
    batch = 2
    x = synth.input_images(5, "yolov3", batch, (3, 416, 416))
    ref = O.run_network(calibrated, x, keep=HEADS + RAWS)
    obj = np.concatenate([ref[h].reshape(batch, 3, 85, -1)[:, :, 4].ravel() for h in HEADS])
    assert 0.2 < np.mean((obj > 0.01) & (obj < 0.99)), "calibrated heads should not saturate"
    for r in RAWS:
        assert np.abs(ref[r]).max() < 100
    net = TNNet(ctx, calibrated, batch, (3, 416, 416))
    out = net.predict(x, layers=HEADS)
    for h, got in zip(HEADS, out):
        assert_yolo_parity(got.reshape(ref[h].shape), ref[h], 3, 80, h)
    n = assert_same_detections(net, ref, batch, thresh=0.25)
    assert n > 0
    net.close()


def test_calibrated_yolov3_tf32(ctx, calibrated):
    """TF32 path on the calibrated YOLOv3: a measurement more than a bar.  TF32 operands keep 10
    mantissa bits; on a well-conditioned net the rounding compounds through 75 convs to a head
    error of ~1.5e-2 relative L2 (a CPU emulation with TF32-rounded operands shows the same), above
    the north star's 1e-2 -- the tensor-core path that meets it is TB_MATH_BF16_SPLIT
    (test_gpu_bf16split).  Asserted here: the error stays below 5e-2 and the 20 strongest
    candidates of each image (by objectness) are found, apart from those within 1e-2 of the 20th."""
    batch = 2
    x = synth.input_images(5, "yolov3", batch, (3, 416, 416))
    ref = O.run_network(calibrated, x, keep=HEADS)
    net = TNNet(ctx, calibrated, batch, (3, 416, 416), math_mode=MATH_TF32)
    out = net.predict(x, layers=HEADS)
    go = np.concatenate([g.reshape(batch, 3, 85, -1)[:, :, 4].reshape(batch, -1) for g in out], axis=1)
    ro = np.concatenate([ref[h].reshape(batch, 3, 85, -1)[:, :, 4].reshape(batch, -1) for h in HEADS], axis=1)
    errs = []
    for g, h in zip(out, HEADS):
        a = g.reshape(batch, -1).astype(np.float64)
        b = ref[h].reshape(batch, -1).astype(np.float64)
        errs.append(float((np.linalg.norm(a - b, axis=1) / np.linalg.norm(b, axis=1)).max()))
    print("TF32 on the calibrated YOLOv3, head relative L2:", errs)
    assert max(errs) <= 5e-2, errs
    k = 20
    for b in range(batch):
        order = np.argsort(-ro[b], kind="stable")
        kth = ro[b, order[k - 1]]
        sure = set(order[:k][ro[b, order[:k]] > kth + 1e-2])
        top_gpu = set(np.argsort(-go[b], kind="stable")[:k])
        assert sure <= top_gpu, (b, sorted(sure - top_gpu))
    net.close()


def test_yolov3_graph_replay_matches_eager(ctx, yolo_specs):
    x = torch.from_numpy(synth.input_images(4, "yolov3", 2, (3, 416, 416))).to(ctx.torch_device)
    net = TNNet(ctx, yolo_specs, 2, (3, 416, 416))
    net.forward(x, use_graph=False)
    eager = net.output(106).clone()
    eager_launches = net.launch_count
    for _ in range(2):
        net.forward(x, use_graph=True)
    assert torch.equal(net.output(106), eager)
    assert net.launch_count == eager_launches
    assert net.flops == pytest.approx(2 * 65.864075264e9, rel=1e-9)


def test_mnist_config(ctx):
    """conv / maxpool / connected layers bit-exact (the connected layers in the
    reference's sdot_avx2 order), softmax within 2 ulp (exp)."""
    specs = synth.mnist_specs()
    x = synth.input_images(1, "mnist", 256, (1, 28, 28))
    ref = O.run_network(specs, x, keep=[0, 1, 2, 3, 4, 5, 6])
    net = TNNet(ctx, specs, 256, (1, 28, 28))
    out = net.predict(x, layers=[0, 1, 2, 3, 4, 5, 6])
    for got, i in zip(out, range(6)):
        assert_bit_exact(got.reshape(ref[i].shape), ref[i], 256, i)
    assert logistic_ulps(out[6], ref[6]) <= 2.0
    assert np.array_equal(out[6].argmax(1), ref[6].argmax(1))


def test_cifar_config(ctx):
    """BASELINE config 2 (batch 64 of the 1024): convs, maxpools, the 1x1 conv and avgpool
    bit-exact; softmax within 2 ulp."""
    specs = synth.cifar_specs()
    x = synth.input_images(2, "cifar", 64, (3, 32, 32))
    ref = O.run_network(specs, x, keep=[3, 7, 9, 10, 11])
    net = TNNet(ctx, specs, 64, (3, 32, 32))
    out = net.predict(x, layers=[3, 7, 9, 10, 11])
    for got, i in zip(out[:4], (3, 7, 9, 10)):
        assert_bit_exact(got.reshape(ref[i].shape), ref[i], 64, i)
    assert logistic_ulps(out[4], ref[11]) <= 2.0
    assert np.array_equal(out[4].argmax(1), ref[11].argmax(1))


def test_unfused_batchnorm_network(ctx):
    specs = synth.cifar_specs()
    x = synth.input_images(2, "cifar", 4, (3, 32, 32))
    ref = O.run_network(specs, x, fuse_batchnorm=False, keep=[7])
    net = TNNet(ctx, specs, 4, (3, 32, 32), fuse_batchnorm=False)
    got = net.predict(x, layers=[7])[0]
    assert_bit_exact(got.reshape(ref[7].shape), ref[7], 4 * 512, "unfused batchnorm net")


def test_stream_predictor_matches_predict(ctx):
    """StreamPredictor (uploads / downloads overlapped with the forward) returns, for every
    submitted batch, what predict returns for it."""
    from tensorium_b200.net import StreamPredictor
    specs = synth.cifar_specs()
    net = TNNet(ctx, specs, 16, (3, 32, 32))
    batches = [synth.input_images(20 + i, "cifar", 16, (3, 32, 32)) for i in range(5)]
    want = [net.predict(b, layers=[9, 11]) for b in batches]
    sp = StreamPredictor(net, [9, 11])
    h_ins = [torch.from_numpy(b).pin_memory() for b in batches]
    h_outs = [[torch.empty(net.output(l).shape).pin_memory() for l in (9, 11)] for _ in batches]
    for hi, ho in zip(h_ins, h_outs):
        sp.submit(hi, ho)
    sp.wait()
    for w, ho in zip(want, h_outs):
        for a, b in zip(w, ho):
            assert np.array_equal(a, b.numpy())
    net.close()
