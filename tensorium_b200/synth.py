"""Deterministic synthetic inputs and weights for the benchmark configurations.

No dataset, cfg file or .weights file is available (the reference's samples load them from
outside the repository: Samples/FPC/MSCOCO_Yolo/MSCOCOYolo.pas:30-38), so every tensor is made
here from a seed:

* SplitMix64 stream per tensor, seeded from (base seed, tensor name);
* uniform[0,1): the top 24 bits of each 64-bit draw times 2^-24 (exact in fp32);
* normal: Box-Muller on two 53-bit uniforms, computed in float64, rounded to fp32.

Image b of a batch is the same for every batch size (the stream runs over the flattened batch).
The network builders return plain layer specifications (dicts) that both the device executor
(tensorium_b200.net) and the CPU oracle consume.
"""
from __future__ import annotations

import zlib

import numpy as np

_GOLDEN = np.uint64(0x9E3779B97F4A7C15)
_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)


def _seed_of(seed: int, name: str) -> np.uint64:
    return np.uint64((seed * 0x100000001B3 + zlib.crc32(name.encode())) & 0xFFFFFFFFFFFFFFFF)


def splitmix64(seed: int, name: str, n: int) -> np.ndarray:
    """n successive SplitMix64 outputs of the stream (seed, name)."""
    with np.errstate(over="ignore"):
        z = _seed_of(seed, name) + np.arange(1, n + 1, dtype=np.uint64) * _GOLDEN
        z = (z ^ (z >> np.uint64(30))) * _M1
        z = (z ^ (z >> np.uint64(27))) * _M2
        z = z ^ (z >> np.uint64(31))
    return z


def uniform(seed: int, name: str, shape, lo: float = 0.0, hi: float = 1.0) -> np.ndarray:
    n = int(np.prod(shape))
    u = (splitmix64(seed, name, n) >> np.uint64(40)).astype(np.float64) * (1.0 / (1 << 24))
    if lo != 0.0 or hi != 1.0:
        u = lo + (hi - lo) * u
    return u.astype(np.float32).reshape(shape)


def normal(seed: int, name: str, shape, mean: float = 0.0, std: float = 1.0) -> np.ndarray:
    n = int(np.prod(shape))
    m = (n + 1) // 2
    z = splitmix64(seed, name, 2 * m)
    u1 = ((z[0::2] >> np.uint64(11)).astype(np.float64) + 1.0) * (1.0 / (1 << 53))  # (0, 1]
    u2 = (z[1::2] >> np.uint64(11)).astype(np.float64) * (1.0 / (1 << 53))
    r = np.sqrt(-2.0 * np.log(u1))
    g = np.empty(2 * m, dtype=np.float64)
    g[0::2] = r * np.cos(2.0 * np.pi * u2)
    g[1::2] = r * np.sin(2.0 * np.pi * u2)
    return (mean + std * g[:n]).astype(np.float32).reshape(shape)


# ------------------------------------------------------------------------------------------
# layer specifications
# ------------------------------------------------------------------------------------------
ACT = {"logistic": 0, "relu": 1, "linear": 4, "leaky": 9}

YOLO_ANCHORS = np.array([10, 13, 16, 30, 33, 23, 30, 61, 62, 45, 59, 119, 116, 90, 156, 198, 373, 326],
                        dtype=np.float32)


def conv_spec(seed, name, c, filters, size, stride, pad, act, bn, weight_std=None):
    """Conv layer spec with He-normal weights and, with bn, the BASELINE config-0 statistics:
    gamma = 1, beta = 0, running mean N(0, 0.1), running variance U[0.5, 1.5)."""
    fan_in = c * size * size
    std = weight_std if weight_std is not None else float(np.sqrt(2.0 / fan_in))
    s = {"type": "conv", "filters": filters, "size": size, "stride": stride, "pad": pad,
         "activation": act, "batch_normalize": bool(bn),
         "weights": normal(seed, name + ".w", (filters, fan_in), 0.0, std),
         "biases": np.zeros(filters, np.float32)}
    if bn:
        s["scales"] = np.ones(filters, np.float32)
        s["mean"] = normal(seed, name + ".mean", (filters,), 0.0, 0.1)
        s["var"] = uniform(seed, name + ".var", (filters,), 0.5, 1.5)
    return s


def yolov3_specs(seed: int = 3, classes: int = 80):
    """YOLOv3-416: darknet-53 backbone + 3 yolo heads, 107 layers (0-106), 75 convolutions.
    Every conv has batchnorm + leaky 0.1 except the three 1x1 head convs (3*(classes+5)
    filters, linear, bias).  Input (3, 416, 416)."""
    L = []

    def conv(filters, size, stride, act="leaky", bn=True):
        c = layer_shapes(L, (3, 416, 416))[-1][0] if L else 3
        L.append(conv_spec(seed, f"yolo.{len(L)}", c, filters, size, stride, (size - 1) // 2,
                           ACT[act], bn))

    def shortcut(frm):
        L.append({"type": "shortcut", "from": frm, "activation": ACT["linear"]})

    def route(*layers):
        L.append({"type": "route", "layers": list(layers)})

    def upsample():
        L.append({"type": "upsample", "stride": 2, "scale": 1.0})

    def yolo(mask):
        L.append({"type": "yolo", "classes": classes, "mask": list(mask), "anchors": YOLO_ANCHORS.copy(),
                  "scale_xy": 1.0})

    conv(32, 3, 1)
    for filters, blocks in ((64, 1), (128, 2), (256, 8), (512, 8), (1024, 4)):
        conv(filters, 3, 2)
        for _ in range(blocks):
            conv(filters // 2, 1, 1)
            conv(filters, 3, 1)
            shortcut(-3)
    nout = 3 * (classes + 5)
    for _ in range(3):
        conv(512, 1, 1)
        conv(1024, 3, 1)
    conv(nout, 1, 1, "linear", False)
    yolo((6, 7, 8))
    route(-4)
    conv(256, 1, 1)
    upsample()
    route(-1, 61)
    for _ in range(3):
        conv(256, 1, 1)
        conv(512, 3, 1)
    conv(nout, 1, 1, "linear", False)
    yolo((3, 4, 5))
    route(-4)
    conv(128, 1, 1)
    upsample()
    route(-1, 36)
    for _ in range(3):
        conv(128, 1, 1)
        conv(256, 3, 1)
    conv(nout, 1, 1, "linear", False)
    yolo((0, 1, 2))
    assert len(L) == 107, len(L)
    return L


def mnist_specs(seed: int = 1):
    """conv 5x5x32 p2 + ReLU -> maxpool 2/2 -> conv 5x5x64 p2 + ReLU ->
    maxpool 2/2 -> connected 3136->1024 ReLU -> connected 1024->10 -> softmax. He-normal."""
    return [conv_spec(seed, "mnist.0", 1, 32, 5, 1, 2, ACT["relu"], False),
            {"type": "maxpool", "size": 2, "stride": 2, "padding": 0},
            conv_spec(seed, "mnist.2", 32, 64, 5, 1, 2, ACT["relu"], False),
            {"type": "maxpool", "size": 2, "stride": 2, "padding": 0},
            {"type": "connected", "outputs": 1024, "activation": ACT["relu"],
             "weights": normal(seed, "mnist.4.w", (1024, 3136), 0.0, float(np.sqrt(2.0 / 3136))),
             "biases": np.zeros(1024, np.float32)},
            {"type": "connected", "outputs": 10, "activation": ACT["linear"],
             "weights": normal(seed, "mnist.5.w", (10, 1024), 0.0, float(np.sqrt(2.0 / 1024))),
             "biases": np.zeros(10, np.float32)},
            {"type": "softmax", "groups": 1, "temperature": 1.0}]


def cifar_specs(seed: int = 2):
    """3 stages of 2x [conv 3x3 (128/256/512) + BN + leaky], maxpool 2/2
    after each stage -> conv 1x1 -> 10 -> global avgpool -> softmax."""
    L = []
    c = 3
    for filters in (128, 256, 512):
        for _ in range(2):
            L.append(conv_spec(seed, f"cifar.{len(L)}", c, filters, 3, 1, 1, ACT["leaky"], True))
            c = filters
        L.append({"type": "maxpool", "size": 2, "stride": 2, "padding": 0})
    L.append(conv_spec(seed, f"cifar.{len(L)}", c, 10, 1, 1, 0, ACT["linear"], False))
    L.append({"type": "avgpool"})
    L.append({"type": "softmax", "groups": 1, "temperature": 1.0})
    return L


def config0_spec(seed: int = 0):
    """one conv 3->32, 3x3, stride 1, pad 1, BN, leaky, weights
    N(0, sqrt(2/27))."""
    return [conv_spec(seed, "cfg0", 3, 32, 3, 1, 1, ACT["leaky"], True,
                      weight_std=float(np.sqrt(2.0 / 27.0)))]


INPUT_SHAPES = {"cfg0": (3, 416, 416), "mnist": (1, 28, 28), "cifar": (3, 32, 32),
                "yolov3": (3, 416, 416)}


def input_images(seed: int, name: str, batch: int, shape) -> np.ndarray:
    return uniform(seed, f"input.{name}", (batch,) + tuple(shape))


def layer_shapes(specs, input_shape):
    """(c, h, w) output shape of every layer (darknet shape rules)."""
    shapes = []
    c, h, w = input_shape
    for i, s in enumerate(specs):
        t = s["type"]
        if t == "conv":
            c, h, w = (s["filters"], (h + 2 * s["pad"] - s["size"]) // s["stride"] + 1,
                       (w + 2 * s["pad"] - s["size"]) // s["stride"] + 1)
        elif t == "route":
            idx = [i + l if l < 0 else l for l in s["layers"]]
            c = sum(shapes[j][0] for j in idx)
            h, w = shapes[idx[0]][1], shapes[idx[0]][2]
        elif t == "upsample":
            h, w = h * s["stride"], w * s["stride"]
        elif t == "maxpool":
            p = s.get("padding", 0)
            h, w = (h + p - s["size"]) // s["stride"] + 1, (w + p - s["size"]) // s["stride"] + 1
        elif t == "connected":
            c, h, w = s["outputs"], 1, 1
        elif t == "avgpool":
            h, w = 1, 1
        shapes.append((c, h, w))
    return shapes


def conv_flops(specs, input_shape, batch=1) -> float:
    """2*M*N*K over conv and connected layers."""
    shapes = layer_shapes(specs, input_shape)
    f = 0.0
    prev = input_shape
    for s, out in zip(specs, shapes):
        if s["type"] == "conv":
            f += 2.0 * out[0] * out[1] * out[2] * prev[0] * s["size"] ** 2
        elif s["type"] == "connected":
            f += 2.0 * s["outputs"] * prev[0] * prev[1] * prev[2]
        prev = out
    return f * batch
