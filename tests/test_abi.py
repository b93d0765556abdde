"""The C-ABI library: it loads, exports every function include/tensorium_b200.h declares, and
its host-only entry points behave (no GPU needed)."""
import ctypes as C
import re

import numpy as np

from conftest import ROOT
from tensorium_b200 import _lib
from tensorium_b200._lib import ConvDesc, check, lib


def header_functions():
    text = (ROOT / "include" / "tensorium_b200.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(?:int|void\s*\*|const char\s*\*)\s*(tb(?:compat)?_\w+)\s*\(", text)))


def test_every_declared_symbol_is_exported():
    names = header_functions()
    assert len(names) > 50
    for n in names:
        assert hasattr(lib, n), f"{n} missing from libtensorium_b200.so"


def test_binding_covers_header():
    names = set(header_functions()) - {"tb_last_error"}
    assert names == set(_lib.SIGNATURES), names ^ set(_lib.SIGNATURES)


def test_version_and_structs():
    assert lib.tb_version() == 100
    assert C.sizeof(ConvDesc) == 17 * 8
    assert C.sizeof(_lib.Detection) == 48
    assert C.sizeof(_lib.YoloHead) == 64


def test_conv_shape_and_packing_counts():
    d = ConvDesc(1, 3, 416, 416, 32, 3, 3, 1, 1, 1, 1, 1, 1, 9, 0, 0, 0)
    oh, ow, n = C.c_int64(), C.c_int64(), C.c_int64()
    check(lib.tb_conv_out_shape(C.byref(d), C.byref(oh), C.byref(ow)))
    assert (oh.value, ow.value) == (416, 416)
    check(lib.tb_conv_packed_weights_count(C.byref(d), C.byref(n)))
    assert n.value == 32 * 32  # CRS: K = 27 padded to 32, M = 32
    d2 = ConvDesc(1, 512, 13, 13, 255, 1, 1, 1, 1, 0, 0, 1, 1, 4, 0, 0, 0)
    check(lib.tb_conv_packed_weights_count(C.byref(d2), C.byref(n)))
    assert n.value == 512 * 256  # RSC: K = 512, M = 255 padded to 256
    d3 = ConvDesc(1, 3, 416, 416, 64, 3, 3, 2, 2, 1, 1, 1, 1, 9, 0, 0, 0)
    check(lib.tb_conv_out_shape(C.byref(d3), C.byref(oh), C.byref(ow)))
    assert (oh.value, ow.value) == (208, 208)


def test_invalid_arguments_report_errors():
    d = ConvDesc(1, 0, 4, 4, 1, 3, 3, 1, 1, 1, 1, 1, 1, 9, 0, 0, 0)
    oh = C.c_int64()
    rc = lib.tb_conv_out_shape(C.byref(d), C.byref(oh), C.byref(oh))
    assert rc == _lib.TB_ERR_INVALID
    assert "bad shape" in _lib.last_error()
    assert lib.tb_xnor_packed_weights_count(0, 1, 1, C.byref(oh)) == _lib.TB_ERR_INVALID
    assert lib.tb_sync(None) == _lib.TB_ERR_INVALID


def test_fold_bn_matches_oracle_bit_exact():
    from oracle import oracle as O
    rng = np.random.default_rng(1)
    w = rng.standard_normal((16, 27)).astype(np.float32)
    b = rng.standard_normal(16).astype(np.float32)
    sc = rng.uniform(0.5, 2, 16).astype(np.float32)
    mu = rng.standard_normal(16).astype(np.float32)
    var = rng.uniform(0, 1.5, 16).astype(np.float32)
    var[0] = 0.0  # hits the max(var, 1e-6) branch
    ow, ob = O.fuse_bn(w, b, sc, mu, var)
    w2, b2 = w.copy(), b.copy()
    check(lib.tb_conv_fold_bn(16, 27, w2.ctypes.data, b2.ctypes.data, sc.ctypes.data, mu.ctypes.data,
                              var.ctypes.data))
    assert np.array_equal(w2, ow) and np.array_equal(b2, ob)


def test_init_without_gpu_fails_cleanly():
    import torch
    if torch.cuda.is_available():
        return
    h = C.c_void_p()
    rc = lib.tb_init(0, None, C.byref(h))
    assert rc < 0 and not h.value


def test_integration_unit_declares_every_function():
    """The Pascal binding unit in INTEGRATION.md declares every function of the header."""
    text = (ROOT / "INTEGRATION.md").read_text()
    declared = set(re.findall(r"function (tb(?:compat)?_\w+)\b[^;]*;[^\n]*external libB200", text))
    missing = set(header_functions()) - declared
    assert not missing, sorted(missing)
