"""TNNet for the B200 path: a whole network held by the C++ executor (``tb_net``).

Mirrors TNNet.forward / predict / fuseBatchNorm / Detections (source/nnet.pas:268-317,
452-472, 584-677): layers are declared from layer specifications (tensorium_b200.synth), weights
are uploaded once per GPU, and ``forward`` replays the whole network as one CUDA graph.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from ._lib import LAYER_TYPES, MATH_BF16_SPLIT, MATH_FP32, PARAM, LayerInfo, check, lib
from .context import Context, ptr
from .layers import TYoloLayer, get_detections
from .synth import layer_shapes


def _f32(a):
    return None if a is None else np.ascontiguousarray(a, np.float32)


class TNNet:
    def __init__(self, ctx: Context, specs, batch: int, input_shape, fuse_batchnorm: bool = True,
                 fusion: bool = True, math_mode: int = MATH_FP32):
        self.ctx = ctx
        self.math_mode = int(math_mode)
        self.specs = specs
        self.batch = int(batch)
        self.input_shape = tuple(input_shape)
        self.shapes = layer_shapes(specs, self.input_shape)
        self.handle = C.c_void_p()
        c, h, w = self.input_shape
        check(lib.tb_net_create(ctx.handle, self.batch, c, h, w, C.byref(self.handle)))
        ctx.adopt(self)
        self.yolo_layers = []
        keep = []
        for i, s in enumerate(specs):
            self._add(i, s, keep)
        check(lib.tb_net_set_fusion(self.handle, 1 if fusion else 0))
        if fuse_batchnorm:
            check(lib.tb_net_fuse_batchnorm(self.handle))
        check(lib.tb_net_finalize(self.handle, math_mode))

    def _add(self, i, s, keep):
        t = s["type"]
        h = self.handle
        if t == "conv":
            arrs = [_f32(s.get(k)) for k in ("weights", "biases", "scales", "mean", "var")]
            keep += arrs
            check(lib.tb_net_add_conv(h, s["filters"], s["size"], s["stride"], s["pad"], s["activation"],
                                      1 if s["batch_normalize"] else 0, *[ptr(a) for a in arrs]))
        elif t == "shortcut":
            check(lib.tb_net_add_shortcut(h, s["from"], s.get("activation", 4)))
        elif t == "route":
            arr = (C.c_int64 * len(s["layers"]))(*s["layers"])
            check(lib.tb_net_add_route(h, len(s["layers"]), arr))
        elif t == "upsample":
            check(lib.tb_net_add_upsample(h, s["stride"], s.get("scale", 1.0)))
        elif t == "yolo":
            mask = np.ascontiguousarray(s["mask"], np.int64)
            anchors = _f32(s["anchors"])
            keep += [mask, anchors]
            check(lib.tb_net_add_yolo(h, s["classes"], len(mask), ptr(mask), len(anchors) // 2, ptr(anchors),
                                      s.get("scale_xy", 1.0)))
            self.yolo_layers.append(i)
        elif t == "maxpool":
            check(lib.tb_net_add_maxpool(h, s["size"], s["stride"], s.get("padding", 0)))
        elif t == "connected":
            w, b = _f32(s["weights"]), _f32(s.get("biases"))
            keep += [w, b]
            check(lib.tb_net_add_connected(h, s["outputs"], s["activation"], ptr(w), ptr(b)))
        elif t == "softmax":
            check(lib.tb_net_add_softmax(h, s.get("groups", 1), s.get("temperature", 1.0)))
        elif t == "avgpool":
            check(lib.tb_net_add_avgpool(h))
        else:
            raise ValueError(f"layer {i}: unknown type {t}")

    # -- darknet model files ---------------------------------------------------------------
    @classmethod
    def from_darknet(cls, ctx, cfg_path, weights_path=None, batch: int = 0, cutoff: int = 0,
                     fuse_batchnorm: bool = True, fusion: bool = True, math_mode: int = MATH_FP32):
        """TDarknetParser.Create(cfg, batch) + loadWeights(weights, cutoff)
        (source/nparser.pas:782-940, 1275-1340), parsed and read by the library
        (tb_darknet_load).  ctx = None gives a host-only net (inspect, save; no forward)."""
        self = cls.__new__(cls)
        self.ctx = ctx
        self.math_mode = int(math_mode)
        self.handle = C.c_void_p()
        check(lib.tb_darknet_load(ctx.handle if ctx is not None else None, str(cfg_path).encode(),
                                  None if weights_path is None else str(weights_path).encode(),
                                  int(batch), int(cutoff), C.byref(self.handle)))
        b, c, h, w = (C.c_int64() for _ in range(4))
        check(lib.tb_net_input_shape(self.handle, C.byref(b), C.byref(c), C.byref(h), C.byref(w)))
        self.batch, self.input_shape = b.value, (c.value, h.value, w.value)
        self.specs = self.layer_specs(params=False)
        self.shapes = [s.pop("_out") for s in self.specs]
        self.yolo_layers = [i for i, s in enumerate(self.specs) if s["type"] == "yolo"]
        if ctx is None:
            return self
        ctx.adopt(self)
        check(lib.tb_net_set_fusion(self.handle, 1 if fusion else 0))
        if fuse_batchnorm:
            check(lib.tb_net_fuse_batchnorm(self.handle))
        check(lib.tb_net_finalize(self.handle, math_mode))
        return self

    def layer_specs(self, params: bool = True):
        """The net's layers as layer specifications (the dicts tensorium_b200.synth builds), read
        back from the library; params=True copies the host-side weight arrays too.  Each spec
        also carries "_out", the layer's output shape (c, h, w)."""
        n = C.c_int64()
        check(lib.tb_net_layer_count(self.handle, C.byref(n)))
        return [self._spec_of(i, params) for i in range(n.value)]

    def _param(self, i, name, dtype=np.float32):
        cnt = C.c_int64()
        check(lib.tb_net_layer_param(self.handle, i, PARAM[name], None, 0, C.byref(cnt)))
        a = np.empty(cnt.value, dtype)
        check(lib.tb_net_layer_param(self.handle, i, PARAM[name], a.ctypes.data_as(C.c_void_p), cnt.value, None))
        return a

    def _spec_of(self, i, params):
        d = LayerInfo()
        check(lib.tb_net_layer_info(self.handle, i, C.byref(d)))
        t = LAYER_TYPES[d.type]
        s = {"type": t, "_out": (d.out_c, d.out_h, d.out_w)}
        if t == "conv":
            s.update(filters=d.filters, size=d.ksize, stride=d.stride, pad=d.pad, activation=d.activation,
                     batch_normalize=bool(d.batch_normalize))
            if params:
                s["weights"] = self._param(i, "weights").reshape(d.filters, -1)
                s["biases"] = self._param(i, "biases")
                if d.batch_normalize:
                    s["scales"], s["mean"], s["var"] = (self._param(i, k) for k in ("scales", "mean", "var"))
        elif t == "connected":
            s.update(outputs=d.filters, activation=d.activation)
            if params:
                s["weights"] = self._param(i, "weights").reshape(d.filters, -1)
                s["biases"] = self._param(i, "biases")
        elif t == "shortcut":
            s.update({"from": d.from_, "activation": d.activation})
        elif t == "route":
            s["layers"] = [int(v) for v in self._param(i, "route_inputs", np.int64)]
        elif t == "upsample":
            s.update(stride=d.stride, scale=d.scale)
        elif t == "yolo":
            s.update(classes=d.classes, mask=[int(v) for v in self._param(i, "yolo_mask", np.int64)],
                     anchors=self._param(i, "yolo_anchors"), scale_xy=d.scale)
        elif t == "maxpool":
            s.update(size=d.ksize, stride=d.stride, padding=d.pad)
        elif t == "softmax":
            s.update(groups=d.groups, temperature=d.scale)
        return s

    def save_weights(self, path, seen: int = 0) -> None:
        """TDarknetParser.saveWeights (source/nparser.pas:1394-1440) of the host-side arrays
        (batchnorm arrays only for conv layers whose batchnorm is not folded)."""
        check(lib.tb_darknet_save_weights(self.handle, str(path).encode(), int(seen)))

    # -- execution ----------------------------------------------------------------------
    def forward(self, x: torch.Tensor, use_graph: bool = True) -> None:
        """TNNet.forward on a device tensor [batch, c, h, w] (asynchronous)."""
        assert x.is_cuda and x.dtype == torch.float32 and x.is_contiguous()
        assert tuple(x.shape) == (self.batch,) + self.input_shape, x.shape
        check(lib.tb_net_forward(self.handle, ptr(x), 1 if use_graph else 0))

    def output(self, layer: int = -1) -> torch.Tensor:
        """A layer's output as [batch, per_image] in NCHW order: a device view (strided for route
        slices), or, for an activation the executor keeps NHWC, an NCHW copy of it."""
        if layer < 0:
            layer += len(self.specs)
        p = C.c_void_p()
        n = C.c_int64()
        bs = C.c_int64()
        check(lib.tb_net_layer_output(self.handle, layer, C.byref(p), C.byref(n), C.byref(bs)))
        ps = C.c_int64()
        check(lib.tb_net_layer_layout(self.handle, layer, C.byref(ps)))
        if ps.value == 0:
            return _view(p.value, self.batch, n.value, bs.value, self.ctx.torch_device)
        c, h, w = self.shapes[layer]
        numel = (self.batch - 1) * bs.value + (h * w - 1) * ps.value + c
        t = torch.as_tensor(_CAI(p.value, numel), device=self.ctx.torch_device)
        nhwc = t.as_strided((self.batch, h, w, c), (bs.value, w * ps.value, ps.value, 1))
        out = nhwc.permute(0, 3, 1, 2).contiguous().reshape(self.batch, c * h * w)
        if self.math_mode == MATH_BF16_SPLIT:  # 32-bit slots of bf16 (hi, lo) pairs: hi + lo
            u = out.view(torch.int32)
            hi = torch.bitwise_left_shift(u, 16).view(torch.float32)
            lo = torch.bitwise_and(u, -65536).view(torch.float32)
            out = hi + lo
        return out

    def predict(self, x_host: np.ndarray, layers=None):
        """TNNet.predict (source/nnet.pas:452-472): host input in, host outputs back
        (default: the last layer) as numpy arrays [batch, per_image]."""
        x = self.staging(x_host)
        self.forward(x)
        layers = layers if layers is not None else [len(self.specs) - 1]
        return [self.output(l).cpu().numpy() for l in layers]

    def predict_images(self, images, letterbox: bool = False, layers=None, pipeline=None):
        """The YOLO sample's per-image loop (img.resize or letterBoxEx, then predict;
        Samples/FPC/MSCOCO_Yolo/MSCOCOYolo.pas:348-350,454) for a whole batch of decoded 8-bit
        images: bytes to the GPU, resized / letterboxed into the input on the GPU, forward.
        Returns the outputs like predict, and the ratios and placements of the images."""
        from .image import ImagePipeline
        if pipeline is None:
            pipeline = getattr(self, "_pipeline", None) or ImagePipeline(self.ctx)
            self._pipeline = pipeline
        c, h, w = self.input_shape
        assert c == 3 and len(images) == self.batch, (c, len(images))
        if getattr(self, "_x", None) is None or tuple(self._x.shape) != (self.batch,) + self.input_shape:
            self._x = torch.empty((self.batch,) + self.input_shape, dtype=torch.float32,
                                  device=self.ctx.torch_device)
        _, ratios, place = pipeline.to_tensor(images, w, h, letterbox, out=self._x)
        self.forward(self._x)
        layers = layers if layers is not None else [len(self.specs) - 1]
        return [self.output(l).cpu().numpy() for l in layers], ratios, place

    def staging(self, x_host):
        if getattr(self, "_x", None) is None or tuple(self._x.shape) != tuple(x_host.shape):
            self._x = torch.empty(x_host.shape, dtype=torch.float32, device=self.ctx.torch_device)
        self._x.copy_(torch.from_numpy(np.ascontiguousarray(x_host, np.float32)))
        return self._x

    def yolo_heads(self):
        heads, outs = [], []
        for i in self.yolo_layers:
            s = self.specs[i]
            c, hh, ww = self.shapes[i]
            heads.append(TYoloLayer(self.batch, ww, hh, len(s["mask"]), len(s["anchors"]) // 2, s["mask"],
                                    s["classes"], s["anchors"], s.get("scale_xy", 1.0)))
            outs.append(self.output(i))
        return heads, outs

    def detections(self, img_w, img_h, thresh=0.45, relative=True, letter=False, capacity=4096, nms=None):
        """TNNet.Detections over every yolo layer, extracted on the GPU; with nms = a threshold,
        followed by TDetectionsHelper.doNMSSort on the GPU (the sample's detections.doNMSSort)."""
        heads, outs = self.yolo_heads()
        net_c, net_h, net_w = self.input_shape
        return get_detections(self.ctx, heads, outs, self.batch, img_w, img_h, net_w, net_h, thresh,
                              relative, letter, capacity, nms)

    def profile(self, x: torch.Tensor) -> np.ndarray:
        """Device milliseconds of every layer in one eager forward (CUDA events)."""
        ms = (C.c_double * len(self.specs))()
        check(lib.tb_net_profile(self.handle, ptr(x), ms))
        return np.array(ms[:])

    @property
    def flops(self) -> float:
        f = C.c_double()
        check(lib.tb_net_flops(self.handle, C.byref(f)))
        return f.value

    @property
    def launch_count(self) -> int:
        n = C.c_int64()
        check(lib.tb_net_launch_count(self.handle, C.byref(n)))
        return n.value

    def close(self):
        if self.handle and (self.ctx is None or self.ctx.handle):
            lib.tb_net_destroy(self.handle)
            self.handle = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class StreamPredictor:
    """TNNet.predict for a stream of batches, with the host copies overlapped with the forward.

    Each ``submit(h_in, h_outs)`` schedules, for one batch: the host-to-device copy of ``h_in``
    (pinned) on an upload stream, the forward (CUDA graph) on the compute stream once the copy has
    landed, on-device copies of the requested outputs into one of two staging sets, and their
    device-to-host copies into ``h_outs`` (pinned) on a download stream (a separate stream, so
    that an upload never queues behind a download that waits for the previous forward). With two input and two output
    staging buffers, batch i+1's upload and batch i-1's download run while batch i computes.
    ``wait()`` blocks until every submitted batch has landed in its host buffers. The forward sees a
    fixed input buffer (one graph); each batch reaches it by a device-to-device copy.
    """

    def __init__(self, net: TNNet, layers):
        self.net = net
        self.layers = list(layers)
        dev = net.ctx.torch_device
        shape = (net.batch,) + net.input_shape
        self.x = torch.empty(shape, dtype=torch.float32, device=dev)
        self.d_in = [torch.empty(shape, dtype=torch.float32, device=dev) for _ in range(2)]
        self.d_out = [[torch.empty(net.output(l).shape, dtype=torch.float32, device=dev) for l in self.layers]
                      for _ in range(2)]
        # the stream the context launches on (the forward's stream), whatever torch's current one is
        raw = lib.tb_get_stream(net.ctx.handle)
        self.compute = torch.cuda.ExternalStream(raw, device=dev) if raw else torch.cuda.default_stream(dev)
        self.upload = torch.cuda.Stream(device=dev)
        self.download = torch.cuda.Stream(device=dev)
        self.ev_h2d = [torch.cuda.Event() for _ in range(2)]
        self.ev_in_free = [torch.cuda.Event() for _ in range(2)]
        self.ev_out_ready = [torch.cuda.Event() for _ in range(2)]
        self.ev_out_free = [torch.cuda.Event() for _ in range(2)]
        self.used = [False, False]
        self.i = 0
        net.forward(self.x)  # capture the graph for the fixed input buffer

    def submit(self, h_in: torch.Tensor, h_outs) -> None:
        k = self.i & 1
        self.i += 1
        with torch.cuda.stream(self.upload):
            if self.used[k]:
                self.upload.wait_event(self.ev_in_free[k])
            self.d_in[k].copy_(h_in, non_blocking=True)
            self.ev_h2d[k].record(self.upload)
        with torch.cuda.stream(self.compute):
            self.compute.wait_event(self.ev_h2d[k])
            self.x.copy_(self.d_in[k])
            self.ev_in_free[k].record(self.compute)
            self.net.forward(self.x)
            if self.used[k]:
                self.compute.wait_event(self.ev_out_free[k])
            for l, d in zip(self.layers, self.d_out[k]):
                d.copy_(self.net.output(l))
            self.ev_out_ready[k].record(self.compute)
        with torch.cuda.stream(self.download):
            self.download.wait_event(self.ev_out_ready[k])
            for o, d in zip(h_outs, self.d_out[k]):
                o.copy_(d, non_blocking=True)
            self.ev_out_free[k].record(self.download)
        self.used[k] = True

    def wait(self) -> None:
        self.upload.synchronize()
        self.compute.synchronize()
        self.download.synchronize()


class _CAI:
    def __init__(self, addr, numel):
        self.__cuda_array_interface__ = {"shape": (numel,), "typestr": "<f4", "data": (addr, False),
                                         "version": 3, "strides": None}


def _view(addr, batch, n, bs, device):
    """A [batch, n] tensor over device memory at `addr` with row stride `bs` (no copy)."""
    numel = (batch - 1) * bs + n
    return torch.as_tensor(_CAI(addr, numel), device=device).as_strided((batch, n), (bs, 1))
