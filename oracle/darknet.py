"""Writer of darknet .cfg / .weights files from layer specifications (tensorium_b200.synth).

TEST INFRASTRUCTURE ONLY -- used by tests/ to make model files whose contents are known, so the
library's loader (tb_darknet_load) can be checked against the specifications it came from, and
its writer (tb_darknet_save_weights) against these bytes.  The product never imports it.

The byte layout restates the reference's own writer and reader:

* header: int32 major, minor, revision; then `seen` as uint64 when major * 10 + minor >= 2, else
  as uint32 (TDarknetParser.loadWeights, source/nparser.pas:1288-1306; saveWeights writes 0, 2, 5
  and a uint64, :1394-1408); connected weights are stored transposed when major or minor > 1000
  (:1307);
* per convolutional layer: biases[F], then scales[F], rolling_mean[F], rolling_variance[F] when
  batch-normalized, then weights[F * C * k * k] (loadConvolutionalWeights, :1140-1185);
* per connected layer: biases[O], weights[O * I] ([I][O] when transposed), then the three
  batchnorm arrays when batch-normalized (loadConnectedWeights, :1102-1128);
* other layers hold nothing in the file (shortcuts without weights_type).

Parity is pinned only by this restatement: the reference ships no .cfg or .weights file.
"""
from __future__ import annotations

import struct

import numpy as np

# TActivationType ordinals (source/ntypes.pas:66-71) -> cfg names (source/nparser.pas:1584-1611)
ACT_NAMES = {0: "logistic", 1: "relu", 2: "relu6", 3: "relie", 4: "linear", 5: "ramp", 6: "tanh",
             7: "plse", 8: "revleaky", 9: "leaky", 10: "elu", 11: "loggy", 13: "hardtan",
             14: "lhtan", 15: "selu"}


def cfg_text(specs, input_shape, batch=1, subdivisions=1):
    """The [net] section and one section per spec, darknet key names; every value the loader
    would otherwise default is written out."""
    c, h, w = input_shape
    out = ["[net]", f"batch={batch}", f"subdivisions={subdivisions}",
           f"height={h}", f"width={w}", f"channels={c}", ""]
    for i, s in enumerate(specs):
        t = s["type"]
        if t == "conv":
            out += ["[convolutional]"]
            if s["batch_normalize"]:
                out += ["batch_normalize=1"]
            out += [f"filters={s['filters']}", f"size={s['size']}", f"stride={s['stride']}"]
            out += ["pad=1"] if s["pad"] == s["size"] // 2 else [f"padding={s['pad']}"]
            out += [f"activation={ACT_NAMES[s['activation']]}"]
        elif t == "shortcut":
            out += ["[shortcut]", f"from={s['from']}", f"activation={ACT_NAMES[s.get('activation', 4)]}"]
        elif t == "route":
            out += ["[route]", "layers=" + ",".join(str(v) for v in s["layers"])]
        elif t == "upsample":
            out += ["[upsample]", f"stride={s['stride']}"]
        elif t == "yolo":
            n_anchor = len(s["anchors"]) // 2
            out += ["[yolo]", "mask=" + ",".join(str(v) for v in s["mask"]),
                    "anchors=" + ",".join(f"{float(v):g}" for v in s["anchors"]),
                    f"classes={s['classes']}", f"num={n_anchor}"]
            if s.get("scale_xy", 1.0) != 1.0:
                out += [f"scale_x_y={s['scale_xy']!r}"]
        elif t == "maxpool":
            out += ["[maxpool]", f"size={s['size']}", f"stride={s['stride']}",
                    f"padding={s.get('padding', 0)}"]
        elif t == "connected":
            out += ["[connected]", f"output={s['outputs']}",
                    f"activation={ACT_NAMES[s['activation']]}"]
        elif t == "softmax":
            out += ["[softmax]", f"groups={s.get('groups', 1)}"]
            if s.get("temperature", 1.0) != 1.0:
                out += [f"temperature={s['temperature']!r}"]
        elif t == "avgpool":
            out += ["[avgpool]"]
        elif t == "dropout":
            out += ["[dropout]", "probability=.5"]
        else:
            raise ValueError(f"layer {i}: no darknet section for {t}")
        out += [""]
    return "\n".join(out)


def weights_bytes(specs, major=0, minor=2, revision=5, seen=0, transpose=None):
    """The .weights file of the specs' arrays (float32, little endian)."""
    if transpose is None:
        transpose = major > 1000 or minor > 1000
    hdr = struct.pack("<iii", major, minor, revision)
    hdr += struct.pack("<Q", seen) if major * 10 + minor >= 2 else struct.pack("<I", seen)
    parts = [hdr]

    def put(a):
        parts.append(np.ascontiguousarray(a, "<f4").tobytes())

    for s in specs:
        if s["type"] == "conv":
            put(s.get("biases", np.zeros(s["filters"], np.float32)))
            if s["batch_normalize"]:
                put(s["scales"]); put(s["mean"]); put(s["var"])
            put(s["weights"])
        elif s["type"] == "connected":
            put(s.get("biases", np.zeros(s["outputs"], np.float32)))
            wt = np.asarray(s["weights"], np.float32).reshape(s["outputs"], -1)
            put(wt.T if transpose else wt)
            if s.get("batch_normalize"):
                put(s["scales"]); put(s["mean"]); put(s["var"])
    return b"".join(parts)


def write(specs, input_shape, cfg_path, weights_path, batch=1, **header):
    with open(cfg_path, "w") as f:
        f.write(cfg_text(specs, input_shape, batch))
    with open(weights_path, "wb") as f:
        f.write(weights_bytes(specs, **header))
