"""ctypes wrapper of liboracle.so (oracle.cpp): the CPU restatement of the reference path.

TEST INFRASTRUCTURE ONLY -- loaded by tests/, __graft_entry__.smoke() and bench.py's CPU
baseline; the product never imports it.  PARITY UNPINNED: the reference (FreePascal) cannot be
built or run here and ships no golden vectors; see the header of oracle.cpp.

``run_network`` walks layer specifications (tensorium_b200.synth) the way TNNet.forward
(source/nnet.pas:275-317) walks its layers.  Route is evaluated per image (darknet channel
concatenation); the reference's TTensor.concat copies whole tensors back to back, which is the
same thing at batch 1 (source/ntensors.pas:12045-12061), so batched inputs run image by image.
"""
from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle.so"


def build() -> Path:
    r = subprocess.run(["make", "-s", "-C", str(HERE)], capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"oracle build failed:\n{r.stdout}\n{r.stderr}")
    return LIB_PATH


def _load():
    src = HERE / "oracle.cpp"
    if not LIB_PATH.exists() or (src.exists() and src.stat().st_mtime > LIB_PATH.stat().st_mtime):
        build()
    lib = C.CDLL(str(LIB_PATH))
    P, I, F = C.c_void_p, C.c_int64, C.c_float
    sig = {
        "or_activate": [I, P, I],
        "or_im2col": [I] * 11 + [P, P],
        "or_sgemm_nn": [I, I, I, F, P, I, P, I, F, P, I],
        "or_sgemm_nt": [I, I, I, F, P, I, P, I, F, P, I],
        "or_sgemm_tn": [I, I, I, F, P, I, P, I, F, P, I],
        "or_sgemm_tt": [I, I, I, F, P, I, P, I, F, P, I],
        "or_fuse_bn": [I, I, P, P, P, P, P],
        "or_conv2d_fwd": [I] * 13 + [P, P, P, P, P, P, I, P],
        "or_maxpool": [I] * 8 + [P, P, P],
        "or_upsample": [I, I, I, I, I, F, P, P],
        "or_concat": [I, P, P, P],
        "or_shortcut": [I, P, P, P, I],
        "or_yolo_fwd": [I, I, I, I, I, P, P, F],
        "or_yolo_detections": [P, I, I, I, I, I, P, P, I, I, I, I, F, I, I, I, P, P, P],
        "or_connected": [I, I, I, P, P, P, I, P],
        "or_softmax": [I, I, I, F, P, P],
        "or_avgpool": [I, I, I, I, P, P],
        "or_xnor_mean": [I, I, P, P],
        "or_xnor_conv": [I] * 9 + [P, P, P, P, P],
        "or_nms_sort": [I, I, P, P, P, F, P],
        "or_image_from_bytes": [I, I, P, I, I, I, I, P],
        "or_resize": [I, I, I, P, I, I, P],
        "or_letterbox": [I, I, I, P, I, I, P, P, P],
        "or_num_threads": [],
        "or_set_threads": [I],
    }
    for k, a in sig.items():
        f = getattr(lib, k)
        f.argtypes = a
        f.restype = None
    lib.or_num_threads.restype = I
    lib.or_yolo_detections.restype = I
    return lib


lib = _load()


def _p(a):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be contiguous"
    return C.c_void_p(a.ctypes.data)


def f32(a):
    return None if a is None else np.ascontiguousarray(a, dtype=np.float32)


def sgemm(trans_a, trans_b, M, N, K, alpha, A, lda, B, ldb, beta, Cm, ldc):
    """cblas_sgemm (row major) in the reference CPU routines' orders; returns the updated C."""
    A, B = f32(A), f32(B)
    out = f32(Cm).copy()
    fn = {(0, 0): lib.or_sgemm_nn, (0, 1): lib.or_sgemm_nt, (1, 0): lib.or_sgemm_tn,
          (1, 1): lib.or_sgemm_tt}[(int(bool(trans_a)), int(bool(trans_b)))]
    fn(M, N, K, alpha, _p(A), lda, _p(B), ldb, beta, _p(out), ldc)
    return out


# ---- single layers ----------------------------------------------------------------------
def conv2d(x, w, bias, filters, size, stride, pad, act, bn=None, dilation=1):
    """x [B,C,H,W]; w [F, C*k*k]; bn = (scales, mean, var) for the unfused path."""
    x = f32(x)
    B, Cc, H, W = x.shape
    oh = (H + 2 * pad - (dilation * (size - 1) + 1)) // stride + 1
    ow = (W + 2 * pad - (dilation * (size - 1) + 1)) // stride + 1
    # gemm runs with beta = 0, i.e. C := C*0 first (source/ntensors.pas:2259-2261); the
    # reference's output tensor starts zeroed, so start from zeros (NaN*0 would stay NaN)
    y = np.zeros((B, filters, oh, ow), np.float32)
    w, bias = f32(w), f32(bias)
    sc, mu, var = (f32(t) for t in bn) if bn is not None else (None, None, None)
    lib.or_conv2d_fwd(B, Cc, H, W, filters, size, size, stride, stride, pad, pad, dilation, dilation,
                      _p(x), _p(w), _p(bias), _p(sc), _p(mu), _p(var), act, _p(y))
    return y


def fuse_bn(w, b, scales, mean, var):
    w = f32(w).copy()
    b = f32(b).copy()
    lib.or_fuse_bn(w.shape[0], w.shape[1], _p(w), _p(b), _p(f32(scales)), _p(f32(mean)), _p(f32(var)))
    return w, b


def maxpool(x, size, stride, padding=0, want_index=False):
    x = f32(x)
    B, Cc, H, W = x.shape
    oh = (H + padding - size) // stride + 1
    ow = (W + padding - size) // stride + 1
    y = np.empty((B, Cc, oh, ow), np.float32)
    idx = np.empty((B, Cc, oh, ow), np.int64) if want_index else None
    lib.or_maxpool(B, Cc, H, W, size, stride, stride, padding, _p(x), _p(y), _p(idx))
    return (y, idx) if want_index else y


def upsample(x, stride, scale=1.0):
    x = f32(x)
    B, Cc, H, W = x.shape
    y = np.empty((B, Cc, H * stride, W * stride), np.float32)
    lib.or_upsample(B, Cc, H, W, stride, scale, _p(x), _p(y))
    return y


def concat(inputs):
    """TTensor.concat: whole tensors back to back."""
    ins = [f32(t) for t in inputs]
    out = np.empty(sum(t.size for t in ins), np.float32)
    arr = (C.c_void_p * len(ins))(*[t.ctypes.data for t in ins])
    sizes = (C.c_int64 * len(ins))(*[t.size for t in ins])
    lib.or_concat(len(ins), arr, sizes, _p(out))
    return out


def shortcut(a, b, act=4):
    a, b = f32(a), f32(b)
    y = np.empty_like(a)
    lib.or_shortcut(a.size, _p(a), _p(b), _p(y), act)
    return y


def yolo(x, n, classes, scale_xy=1.0):
    x = f32(x)
    B, Cc, H, W = x.shape
    y = np.empty_like(x)
    lib.or_yolo_fwd(B, n, classes, H, W, _p(x), _p(y), scale_xy)
    return y


def yolo_detections(out, b, n, classes, h, w, mask, anchors, img_w, img_h, net_w, net_h, thresh,
                    relative=True, letter=False, capacity=20000):
    out = f32(out)
    mask = np.ascontiguousarray(mask, np.int64)
    anchors = f32(anchors)
    boxes = np.zeros((capacity, 5), np.float32)
    meta = np.zeros((capacity, 3), np.int64)
    probs = np.zeros((capacity, classes), np.float32)
    cnt = lib.or_yolo_detections(_p(out), b, n, classes, h, w, _p(mask), _p(anchors), img_w, img_h,
                                 net_w, net_h, thresh, int(relative), int(letter), capacity,
                                 _p(boxes), _p(meta), _p(probs))
    k = min(cnt, capacity)
    return cnt, boxes[:k], meta[:k], probs[:k]


def nms_sort(boxes, objectness, probs, thresh):
    """TDetectionsHelper.doNMSSort: probs (n x classes) with the suppressed entries zeroed, in the
    original detection order, and the final record order the reference leaves."""
    boxes = f32(boxes).reshape(-1, 4)
    obj = f32(objectness)
    probs = f32(probs).copy()
    n, classes = probs.shape
    order = np.zeros(n, np.int64)
    lib.or_nms_sort(n, classes, _p(boxes), _p(obj), _p(probs), thresh, _p(order))
    return probs, order


def image_from_bytes(img, bgr=False, pixel_scale=0):
    """TImageData.loadFromFile's conversion of an 8-bit image [h][w] or [h][w][bpp] to planar
    floats [3][h][w] (pixel_scale 0: v*257/65280 as the FPC build, 1: v/255 as the Delphi build)."""
    img = np.ascontiguousarray(img, np.uint8)
    h, w = img.shape[:2]
    bpp = 1 if img.ndim == 2 else img.shape[2]
    out = np.empty((3, h, w), np.float32)
    lib.or_image_from_bytes(w, h, _p(img), w * bpp, bpp, 1 if bgr else 0, pixel_scale, _p(out))
    return out


def resize(x, aw, ah):
    """TImageData.resize of a planar image [c][h][w] to [c][ah][aw]."""
    x = f32(x)
    c, h, w = x.shape
    out = np.empty((c, ah, aw), np.float32)
    lib.or_resize(c, h, w, _p(x), aw, ah, _p(out))
    return out


def letterbox(x, aw, ah):
    """TImageData.letterBoxEx: (image [c][ah][aw], ratio, (new_w, new_h, dx, dy))."""
    x = f32(x)
    c, h, w = x.shape
    out = np.empty((c, ah, aw), np.float32)
    meta = np.zeros(4, np.int64)
    ratio = np.zeros(1, np.float32)
    lib.or_letterbox(c, h, w, _p(x), aw, ah, _p(out), _p(meta), _p(ratio))
    return out, float(ratio[0]), tuple(int(v) for v in meta)


def connected(x, w, b, act):
    x = f32(x.reshape(x.shape[0], -1))
    w = f32(w)
    y = np.zeros((x.shape[0], w.shape[0]), np.float32)  # beta = 0 on a zeroed tensor
    lib.or_connected(x.shape[0], x.shape[1], w.shape[0], _p(x), _p(w), _p(f32(b)), act, _p(y))
    return y


def softmax(x, groups=1, temp=1.0):
    x = f32(x.reshape(x.shape[0], -1))
    y = np.empty_like(x)
    lib.or_softmax(x.shape[0], x.shape[1], groups, temp, _p(x), _p(y))
    return y


def avgpool(x):
    x = f32(x)
    B, Cc, H, W = x.shape
    y = np.empty((B, Cc), np.float32)
    lib.or_avgpool(B, Cc, H, W, _p(x), _p(y))
    return y


def activate(x, act):
    x = f32(x).copy()
    lib.or_activate(x.size, _p(x), act)
    return x


def xnor_mean(w):
    w = f32(w)
    m = np.empty(w.shape[0], np.float32)
    lib.or_xnor_mean(w.shape[0], w.shape[1], _p(w), _p(m))
    return m


def xnor_conv(x, w, mean, filters, size, stride, pad, pad_mode=0):
    x = f32(x)
    B, Cc, H, W = x.shape
    oh = (H + 2 * pad - size) // stride + 1
    ow = (W + 2 * pad - size) // stride + 1
    y = np.empty((B, filters, oh, ow), np.float32)
    cnt = np.empty((B, filters, oh, ow), np.int32)
    lib.or_xnor_conv(B, Cc, H, W, filters, size, stride, pad, pad_mode, _p(x), _p(f32(w)),
                     _p(f32(mean)), _p(cnt), _p(y))
    return cnt, y


# ---- whole network ----------------------------------------------------------------------
def _src(i, rel):
    return i + rel if rel < 0 else rel


def run_layer(specs, i, prev, get, fuse_batchnorm=True):
    """Output of layer i (NCHW) given its input `prev` and get(j) = output of layer j."""
    s = specs[i]
    t = s["type"]
    if t == "conv":
        w, b = s["weights"], s["biases"]
        bn = None
        if s["batch_normalize"]:
            if fuse_batchnorm:
                w, b = fuse_bn(w, b, s["scales"], s["mean"], s["var"])
            else:
                bn = (s["scales"], s["mean"], s["var"])
        return conv2d(prev, w, b, s["filters"], s["size"], s["stride"], s["pad"], s["activation"], bn)
    if t == "shortcut":
        return shortcut(prev, get(_src(i, s["from"])), s.get("activation", 4))
    if t == "route":
        return np.concatenate([get(_src(i, l)) for l in s["layers"]], axis=1)
    if t == "upsample":
        return upsample(prev, s["stride"], s.get("scale", 1.0))
    if t == "yolo":
        return yolo(prev, len(s["mask"]), s["classes"], s.get("scale_xy", 1.0))
    if t == "maxpool":
        return maxpool(prev, s["size"], s["stride"], s.get("padding", 0))
    if t == "connected":
        return connected(prev, s["weights"], s["biases"], s["activation"])[:, :, None, None]
    if t == "softmax":
        return softmax(prev, s.get("groups", 1), s.get("temperature", 1.0)).reshape(prev.shape)
    if t == "avgpool":
        return avgpool(prev)[:, :, None, None]
    raise ValueError(t)


def run_network(specs, x, fuse_batchnorm=True, keep=None):
    """{layer: output [B, per_image]} for every layer (or the indices in `keep`)."""
    x = f32(x)
    if x.shape[0] > 1:
        per = [run_network(specs, x[b:b + 1], fuse_batchnorm, keep) for b in range(x.shape[0])]
        return {k: np.concatenate([p[k] for p in per], axis=0) for k in per[0]}
    outs = {}
    prev = x
    keep_set = set(range(len(specs))) if keep is None else set(keep)
    needed = set()
    for i, s in enumerate(specs):
        if s["type"] == "route":
            needed.update(_src(i, l) for l in s["layers"])
        if s["type"] == "shortcut":
            needed.add(_src(i, s["from"]))
    store = {}
    for i in range(len(specs)):
        y = run_layer(specs, i, prev, store.__getitem__, fuse_batchnorm)
        if i in needed:
            store[i] = y
        if i in keep_set:
            outs[i] = y.reshape(y.shape[0], -1)
        prev = y
    return outs


def num_threads() -> int:
    return int(lib.or_num_threads())


def set_threads(n: int) -> None:
    lib.or_set_threads(int(n))
