"""darknet .cfg / .weights loading (tb_darknet_load) and saving (tb_darknet_save_weights), host side.

Model files are written from layer specifications by oracle/darknet.py (the format restated from
TDarknetParser, source/nparser.pas); the library loads them into a host-only net (no context, no
GPU), and every layer and array read back through tb_net_layer_info / tb_net_layer_param must
equal the specification bit for bit."""
import numpy as np
import pytest

from oracle import darknet as D
from oracle import oracle as O
from tensorium_b200 import synth
from tensorium_b200._lib import TB_ERR_INVALID, TB_ERR_UNSUPPORTED, TBError
from tensorium_b200.net import TNNet


def absolute(specs):
    """Specs with relative shortcut / route indices made absolute (the form the net reports)."""
    out = []
    for i, s in enumerate(specs):
        s = dict(s)
        if s["type"] == "shortcut":
            s["from"] = i + s["from"] if s["from"] < 0 else s["from"]
        if s["type"] == "route":
            s["layers"] = [i + l if l < 0 else l for l in s["layers"]]
        out.append(s)
    return out


def assert_same(got, want):
    assert len(got) == len(want)
    for i, (g, w) in enumerate(zip(got, want)):
        assert g["type"] == w["type"], i
        for k, v in w.items():
            if k in ("type",):
                continue
            if isinstance(v, np.ndarray):
                assert g[k].dtype == v.dtype or k in ("mask",), (i, k)
                assert np.array_equal(np.asarray(g[k]).ravel(), v.ravel()), (i, k)
            elif k == "scale_xy" or k == "temperature" or k == "scale":
                assert np.float32(g[k]) == np.float32(v), (i, k)
            elif k == "batch_normalize":
                assert bool(g[k]) == bool(v), (i, k)
            else:
                assert g.get(k, v) == v, (i, k, g.get(k), v)


def load(tmp_path, specs, shape, batch=1, header=None, cfg=None, **kw):
    c, w = tmp_path / "m.cfg", tmp_path / "m.weights"
    c.write_text(cfg if cfg is not None else D.cfg_text(specs, shape, batch))
    w.write_bytes(D.weights_bytes(specs, **(header or {})))
    return TNNet.from_darknet(None, c, w, **kw), c, w


def test_yolov3_round_trip(tmp_path):
    """YOLOv3-416: 107 layers, 75 convs (62 M weights) come back unchanged, shapes as the specs'."""
    specs = synth.yolov3_specs()
    net, cfg, wts = load(tmp_path, specs, (3, 416, 416))
    assert net.batch == 1 and net.input_shape == (3, 416, 416)
    got = net.layer_specs(params=True)
    assert_same(got, absolute(specs))
    assert [g["_out"] for g in got] == synth.layer_shapes(specs, (3, 416, 416))
    assert net.yolo_layers == [82, 94, 106]
    # saveWeights gives the same bytes back
    out = tmp_path / "saved.weights"
    net.save_weights(out)
    assert out.read_bytes() == wts.read_bytes()
    net.close()


@pytest.mark.parametrize("name", ["mnist", "cifar", "cfg0"])
def test_classifier_round_trip(tmp_path, name):
    """Configs 0-2: maxpool, connected, avgpool and softmax sections."""
    specs = {"mnist": synth.mnist_specs, "cifar": synth.cifar_specs, "cfg0": synth.config0_spec}[name]()
    shape = synth.INPUT_SHAPES[name]
    net, _, _ = load(tmp_path, specs, shape, batch=4)
    assert net.batch == 4 and net.input_shape == tuple(shape)
    assert_same(net.layer_specs(), absolute(specs))
    net.close()


def test_old_header_and_transposed_connected(tmp_path):
    """Version 0.1 files keep a 32-bit `seen`; major or minor > 1000 stores connected weights
    transposed ([inputs][outputs]) -- both read back to the same network."""
    specs = synth.mnist_specs()
    for header in ({"major": 0, "minor": 1}, {"major": 0, "minor": 1001}, {"major": 1001, "minor": 0}):
        net, _, w = load(tmp_path, specs, (1, 28, 28), header=header)
        assert_same(net.layer_specs(), absolute(specs))
        net.close()


def test_connected_batchnorm_folded_on_load(tmp_path):
    """A batch-normalized [connected] layer is folded into weights and biases on load with the
    fuseBatchNorm arithmetic (source/nConvolutionLayer.pas:102-126)."""
    rng = np.random.default_rng(5)
    w = rng.standard_normal((8, 12)).astype(np.float32)
    b = rng.standard_normal(8).astype(np.float32)
    sc = rng.uniform(0.5, 1.5, 8).astype(np.float32)
    mu = rng.standard_normal(8).astype(np.float32) * 0.1
    var = rng.uniform(0.5, 1.5, 8).astype(np.float32)
    specs = [{"type": "connected", "outputs": 8, "activation": 4, "weights": w, "biases": b,
              "batch_normalize": True, "scales": sc, "mean": mu, "var": var}]
    cfg = D.cfg_text(specs, (12, 1, 1)).replace("output=8", "output=8\nbatch_normalize=1")
    net, _, _ = load(tmp_path, specs, (12, 1, 1), cfg=cfg)
    got = net.layer_specs()[0]
    fw, fb = O.fuse_bn(w, b, sc, mu, var)
    assert np.array_equal(got["weights"], fw) and np.array_equal(got["biases"], fb)
    net.close()


CFG_QUIRKS = """# comment line
[NET]   ; trailing comment
batch = 8
subdivisions=2
 width = 16   # blanks and comments
height\t=\t16
channels=3

[conv]
batch_normalize=1
filters=16
size=3
stride=1
pad=1
activation=LEAKY

[max]
size=2
stride=2

[dropout]
probability=.5

[conv]
filters=8
size=1
stride=1
padding=0
activation=linear

[route]
layers = -1, -3

[soft]
groups = 1
"""


def test_cfg_text_rules(tmp_path):
    """TCFGList.loadFromFile rules (source/nconfig.pas:60-82,280-323): blanks and tabs dropped,
    ';' / '#' comments, case-insensitive section names and aliases ([conv], [max], [soft]),
    pad=1 -> size/2, maxpool padding defaulting to size-1, batch = batch / subdivisions, and
    [dropout] kept as a layer so route indices match the file."""
    c = tmp_path / "q.cfg"
    c.write_text(CFG_QUIRKS)
    net = TNNet.from_darknet(None, c)
    assert net.batch == 4 and net.input_shape == (3, 16, 16)
    s = net.layer_specs()
    assert [x["type"] for x in s] == ["conv", "maxpool", "route", "conv", "route", "softmax"]
    assert s[0]["pad"] == 1 and s[0]["activation"] == 9 and s[0]["batch_normalize"]
    assert s[1]["padding"] == 1 and s[1]["_out"] == (16, 8, 8)          # (16 + 1 - 2) / 2 + 1
    assert s[2]["layers"] == [1] and s[2]["_out"] == (16, 8, 8)         # dropout: identity
    assert s[4]["layers"] == [3, 1] and s[4]["_out"] == (24, 8, 8)
    # no weights file: conv weights zero, batchnorm scales 1, variances 1
    assert not s[0]["weights"].any() and (s[0]["scales"] == 1).all() and (s[0]["var"] == 1).all()
    net.close()
    # TDarknetParser.Create's batch override applies when it differs from the cfg batch
    assert TNNet.from_darknet(None, c, batch=3).batch == 3
    assert TNNet.from_darknet(None, c, batch=8).batch == 4


def test_weights_file_ends(tmp_path):
    """A file that stops at a layer boundary leaves the later layers at zero (loadWeights stops
    at EOF); one that stops inside a layer's arrays is an error; cutoff reads only the first
    layers."""
    specs = synth.cifar_specs()
    shape = synth.INPUT_SHAPES["cifar"]
    full = D.weights_bytes(specs)
    first = D.weights_bytes(specs[:2])          # layers 0 and 1
    c, w = tmp_path / "m.cfg", tmp_path / "m.weights"
    c.write_text(D.cfg_text(specs, shape))
    w.write_bytes(first)
    got = TNNet.from_darknet(None, c, w).layer_specs()
    assert np.array_equal(got[1]["weights"], specs[1]["weights"])
    assert not got[3]["weights"].any()
    w.write_bytes(first[:-4])
    with pytest.raises(TBError) as e:
        TNNet.from_darknet(None, c, w)
    assert e.value.code == TB_ERR_INVALID and "layer 1" in str(e.value)
    w.write_bytes(full)
    got = TNNet.from_darknet(None, c, w, cutoff=1).layer_specs()
    assert np.array_equal(got[0]["weights"], specs[0]["weights"]) and not got[1]["weights"].any()


@pytest.mark.parametrize("section,needle", [
    ("[lstm]\noutput=4", "[lstm]"),
    ("[convolutional]\nfilters=4\nsize=3\ngroups=2\nactivation=leaky", "groups"),
    ("[convolutional]\nfilters=4\nsize=3\nactivation=mish", "activation"),
    ("[shortcut]\nfrom=-1,-2", "more than one"),
])
def test_unsupported_sections_are_named(tmp_path, section, needle):
    c = tmp_path / "u.cfg"
    c.write_text("[net]\nwidth=8\nheight=8\nchannels=4\n\n[convolutional]\nfilters=4\nsize=1\n"
                 "activation=linear\n\n" + section + "\n")
    with pytest.raises(TBError) as e:
        TNNet.from_darknet(None, c)
    assert e.value.code == TB_ERR_UNSUPPORTED and needle in str(e.value)


def test_bad_files(tmp_path):
    c = tmp_path / "b.cfg"
    c.write_text("[convolutional]\nfilters=4\n")
    with pytest.raises(TBError) as e:
        TNNet.from_darknet(None, c)
    assert "[net]" in str(e.value)
    with pytest.raises(TBError):
        TNNet.from_darknet(None, tmp_path / "missing.cfg")
    c.write_text("[net]\nwidth=8\nheight=8\nchannels=x\n")
    with pytest.raises(TBError) as e:
        TNNet.from_darknet(None, c)
    assert "not an integer" in str(e.value)
