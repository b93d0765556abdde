"""Host-side mirror of the reference's layer API for the conv inference path.

Each class keeps the name, constructor arguments and forward semantics of the Pascal layer it
stands for, and its forward runs the B200 kernels through the C ABI -- the calls a Pascal
``forwardGPU`` makes after binding include/tensorium_b200.h.  Tensors are ``[batch, c, h, w]``
fp32 torch tensors on the context's GPU (TSingleTensor.devData).

    TConvolutionalLayer   source/nConvolutionLayer.pas:140-321, 457-569, 1022-1153
    TMaxPoolLayer         source/nMaxPoolLayer.pas:59-124, 363-463, 656-687
    TUpSampleLayer        source/nupsamplelayer.pas:35-131, 187-212
    TConcatLayer (route)  source/nconcatlayer.pas:40-119, 206-232
    TAddLayer (shortcut)  source/naddlayer.pas:52-56, 667-725, 877-921
    TYoloLayer            source/nyololayer.pas:283-290, 399-498, 786-825, 1072-1110
    TXNORConvolutionLayer source/nxnorconvolutionlayer.pas:769-913
    TConnectedLayer       source/nconnectedlayer.pas:62-66, 157-184
    TSoftmaxLayer         source/nsoftmaxlayer.pas:49-52, 139-167
    TAvgPoolLayer         source/navgpoollayer.pas:27-30, 60-84
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from typing import Optional

import numpy as np
import torch

from . import synth
from ._lib import ACT, XNOR_PAD_BIT0, ConvDesc, Detection, YoloHead, check, lib
from .context import Context, ptr


def _act(a) -> int:
    return ACT[a] if isinstance(a, str) else int(a)


def _dev(ctx, a, dtype=np.float32):
    return torch.from_numpy(np.ascontiguousarray(a, dtype)).to(ctx.torch_device)


@dataclass
class TNNetState:
    """The part of TNNetState (source/nbaselayer.pas) the forward path reads."""
    input: torch.Tensor
    isTraining: bool = False


class TBaseLayer:
    output: Optional[torch.Tensor] = None
    ctx: Optional[Context] = None

    def bind(self, ctx: Context):
        self.ctx = ctx
        return self


class TConvolutionalLayer(TBaseLayer):
    def __init__(self, ABatch, Aheight, Awidth, Achannels, Afilters, AGroups=1, AKernelSize=3,
                 AStride_x=1, AStride_y=1, ADilation=1, APadding=-1, AActivation="logistic",
                 ABatch_normalize=False, seed=0):
        if AGroups not in (0, 1):
            raise NotImplementedError("grouped convolution is not on the YOLOv3 / config path")
        self.batch, self.h, self.w, self.c = ABatch, Aheight, Awidth, Achannels
        self.n = self.filters = Afilters
        self.kernelSize = AKernelSize
        self.stride_x, self.stride_y = AStride_x, AStride_y
        self.dilation = ADilation
        # default padding: ADilation - 1 + kernelSize div 2 (:188-191)
        self.Padding = ADilation - 1 + AKernelSize // 2 if APadding < 0 else APadding
        self.ActivationType = _act(AActivation)
        self.isBatchNormalized = bool(ABatch_normalize)
        fan_in = Achannels * AKernelSize * AKernelSize
        scale = float(np.sqrt(2.0 / fan_in))  # He-uniform range (:216-220)
        self.weights = synth.uniform(seed, "conv.w", (Afilters, fan_in), -scale, scale)
        self.biases = np.zeros(Afilters, np.float32)
        if self.isBatchNormalized:
            self.scales = np.ones(Afilters, np.float32)
            self.rolling_mean = np.zeros(Afilters, np.float32)
            self.rolling_variance = np.ones(Afilters, np.float32)
        self._dev = None

    def outHeight(self):
        return (self.h + 2 * self.Padding - self.dilation * (self.kernelSize - 1) - 1) // self.stride_y + 1

    def outWidth(self):
        return (self.w + 2 * self.Padding - self.dilation * (self.kernelSize - 1) - 1) // self.stride_x + 1

    def desc(self, batch=None) -> ConvDesc:
        return ConvDesc(batch or self.batch, self.c, self.h, self.w, self.filters, self.kernelSize,
                        self.kernelSize, self.stride_y, self.stride_x, self.Padding, self.Padding,
                        self.dilation, self.dilation, self.ActivationType, 0, 0, 0)

    def fuseBatchNorm(self):
        """TBaseConvolutionalLayer.fuseBatchNorm (:102-126), on the host."""
        if not self.isBatchNormalized:
            return
        w = np.ascontiguousarray(self.weights, np.float32).copy()
        b = np.ascontiguousarray(self.biases, np.float32).copy()
        check(lib.tb_conv_fold_bn(self.filters, w.shape[1], ptr(w), ptr(b), ptr(np.ascontiguousarray(self.scales)),
                                  ptr(np.ascontiguousarray(self.rolling_mean)),
                                  ptr(np.ascontiguousarray(self.rolling_variance))))
        self.weights, self.biases = w, b
        self.isBatchNormalized = False
        self._dev = None

    def upload(self, ctx: Context = None):
        """Push weights once and re-lay them for the kernel (weights.pushToDevice)."""
        if ctx is not None:
            self.bind(ctx)
        ctx = self.ctx
        d = self.desc()
        n = C.c_int64()
        check(lib.tb_conv_packed_weights_count(C.byref(d), C.byref(n)))
        raw = _dev(ctx, self.weights)
        packed = ctx.empty((n.value,))
        check(lib.tb_conv_pack_weights(ctx.handle, C.byref(d), ptr(raw), ptr(packed)))
        dev = {"w": packed, "b": _dev(ctx, self.biases), "raw": raw}
        if self.isBatchNormalized:
            dev["scales"] = _dev(ctx, self.scales)
            dev["mean"] = _dev(ctx, self.rolling_mean)
            dev["var"] = _dev(ctx, self.rolling_variance)
        self._dev = dev

    def forward(self, state: TNNetState, residual=None, out=None, math_mode=-1):
        x = state.input
        batch = x.shape[0]
        if self._dev is None:
            self.upload()
        d = self.desc(batch)
        y = out if out is not None else self.ctx.empty((batch, self.filters, self.outHeight(), self.outWidth()))
        dv = self._dev
        bn = self.isBatchNormalized
        w = dv["w"]
        tc = C.c_int64(0)
        check(lib.tb_conv_uses_tensor_cores(C.byref(d), math_mode if math_mode >= 0 else self.ctx.math_mode,
                                            C.byref(tc)))
        if tc.value:
            if "w_tf32" not in dv:  # weights rounded to TF32 for the tensor-core mainloop
                dv["w_tf32"] = torch.empty_like(w)
                check(lib.tb_conv_pack_weights_tf32(self.ctx.handle, C.byref(self.desc()), ptr(dv["raw"]),
                                                    ptr(dv["w_tf32"])))
            w = dv["w_tf32"]
        check(lib.tb_conv2d_fwd(self.ctx.handle, C.byref(d), ptr(x), ptr(w), ptr(dv["b"]),
                                ptr(dv["scales"] if bn else None), ptr(dv["mean"] if bn else None),
                                ptr(dv["var"] if bn else None), ptr(residual), ptr(y), math_mode))
        self.output = y
        return y


class TMaxPoolLayer(TBaseLayer):
    def __init__(self, aBatch, aHeight, aWidth, aChannels, aKernelSize, aStride_x=0, aStride_y=0,
                 aPadding=0):
        self.batch, self.h, self.w, self.c = aBatch, aHeight, aWidth, aChannels
        self.kernelSize = aKernelSize
        self.stride_x = aStride_x or aKernelSize
        self.stride_y = aStride_y or aKernelSize
        self.Padding = aPadding
        self.outH = (aHeight + aPadding - aKernelSize) // self.stride_y + 1
        self.outW = (aWidth + aPadding - aKernelSize) // self.stride_x + 1
        self.outC = aChannels

    def forward(self, state: TNNetState, indexes: Optional[torch.Tensor] = None):
        x = state.input
        y = self.ctx.empty((x.shape[0], self.c, self.outH, self.outW))
        check(lib.tb_maxpool_fwd(self.ctx.handle, x.shape[0], self.c, self.h, self.w, self.kernelSize,
                                 self.stride_x, self.stride_y, self.Padding, ptr(x), ptr(y), ptr(indexes)))
        self.output = y
        return y


class TUpSampleLayer(TBaseLayer):
    def __init__(self, ABatch, AWidth, AHeight, AChannels, AStride, AScale=1.0):
        if AStride < 0:
            raise NotImplementedError("reverse upsample (negative stride) is not on the inference path")
        self.batch, self.w, self.h, self.c = ABatch, AWidth, AHeight, AChannels
        self.stride, self.scale = AStride, AScale

    def forward(self, state: TNNetState, out=None, out_batch_stride=0):
        x = state.input
        y = out if out is not None else self.ctx.empty((x.shape[0], self.c, self.h * self.stride, self.w * self.stride))
        check(lib.tb_upsample_fwd(self.ctx.handle, x.shape[0], self.c, self.h, self.w, self.stride,
                                  self.scale, ptr(x), ptr(y), out_batch_stride))
        self.output = y
        return y


class TConcatLayer(TBaseLayer):
    """Route. per_sample=True is darknet's per-image channel concatenation (what the network
    executor implements); per_sample=False reproduces TTensor.concat's whole-tensor copy."""

    def __init__(self, aBatch, aInputLayers, aInputSizes, per_sample=True):
        self.batch = aBatch
        self.inputLayers = list(aInputLayers)
        self.inputSizes = list(aInputSizes)
        self.per_sample = per_sample

    def forward_tensors(self, inputs):
        batch = inputs[0].shape[0]
        y = self.ctx.empty((batch, sum(self.inputSizes)))
        arr = (C.c_void_p * len(inputs))(*[t.data_ptr() for t in inputs])
        sizes = (C.c_int64 * len(inputs))(*self.inputSizes)
        check(lib.tb_route_fwd(self.ctx.handle, batch, len(inputs), arr, sizes, ptr(y),
                               1 if self.per_sample else 0))
        self.output = y
        return y


TRouteLayer = TConcatLayer


class TAddLayer(TBaseLayer):
    """Shortcut, single-input branch (source/naddlayer.pas:696-699)."""

    def __init__(self, aBatch, aInputLayers, aActivation="linear"):
        self.batch = aBatch
        self.inputLayers = list(aInputLayers)
        self.ActivationType = _act(aActivation)

    def forward_tensors(self, a, b):
        y = torch.empty_like(a)
        check(lib.tb_shortcut_fwd(self.ctx.handle, a.numel(), ptr(a), ptr(b), ptr(y), self.ActivationType))
        self.output = y
        return y


class TYoloLayer(TBaseLayer):
    def __init__(self, ABatch, aWidth, aHeight, aN, ATotal, AMask, aClasses, anchors=None, scaleXY=1.0):
        self.batch, self.w, self.h, self.n, self.total = ABatch, aWidth, aHeight, aN, ATotal
        self.mask = np.ascontiguousarray(AMask, np.int64)
        self.classes = aClasses
        self.biases = np.ascontiguousarray(anchors if anchors is not None else synth.YOLO_ANCHORS, np.float32)
        self.scaleXY = scaleXY

    def forward(self, state: TNNetState):
        x = state.input
        y = torch.empty_like(x)
        check(lib.tb_yolo_fwd(self.ctx.handle, x.shape[0], self.n, self.classes, self.h, self.w,
                              ptr(x), ptr(y), self.scaleXY))
        self.output = y
        return y

    def head(self, output: torch.Tensor) -> YoloHead:
        return YoloHead(output.data_ptr(), self.n, self.classes, self.h, self.w,
                        self.mask.ctypes.data, self.biases.ctypes.data, 0)


DET_DTYPE = np.dtype([("x", "<f4"), ("y", "<f4"), ("w", "<f4"), ("h", "<f4"), ("objectness", "<f4"),
                      ("batch", "<i4"), ("head", "<i4"), ("index", "<i4"), ("anchor", "<i4"),
                      ("res", "<i4", 3)])


def get_detections(ctx: Context, heads, outputs, batch, img_w, img_h, net_w, net_h, thresh,
                   relative=True, letter=False, capacity=4096, nms=None):
    """TNNet.Detections for every image (source/nnet.pas:584-677): detection records, class
    probabilities and counts, extracted on the GPU in the reference order."""
    hs = (YoloHead * len(heads))(*[h.head(o) for h, o in zip(heads, outputs)])
    classes = max(h.classes for h in heads)
    dets = torch.zeros(batch * capacity * C.sizeof(Detection), dtype=torch.uint8, device=ctx.torch_device)
    prob = ctx.empty((batch * capacity, classes))
    counts = (C.c_int64 * batch)()
    check(lib.tb_yolo_detect(ctx.handle, batch, len(heads), hs, img_w, img_h, net_w, net_h, thresh,
                             1 if relative else 0, 1 if letter else 0, capacity, ptr(dets), ptr(prob), counts))
    if nms is not None:  # TDetectionsHelper.doNMSSort(classes, nms) on the device
        check(lib.tb_yolo_nms(ctx.handle, batch, capacity, counts, classes, nms, ptr(dets), ptr(prob)))
    recs = dets.cpu().numpy().view(DET_DTYPE).reshape(batch, capacity)
    return recs, prob.cpu().numpy().reshape(batch, capacity, classes), np.array(counts[:], np.int64)


def nms_sort(ctx: Context, dets: torch.Tensor, prob: torch.Tensor, counts, capacity: int, classes: int,
             thresh: float = 0.45):
    """TDetectionsHelper.doNMSSort on device records (tb_detection bytes, batch*capacity) and
    probabilities (batch*capacity x classes), in place."""
    batch = len(counts)
    c = (C.c_int64 * batch)(*[int(v) for v in counts])
    check(lib.tb_yolo_nms(ctx.handle, batch, capacity, c, classes, thresh, ptr(dets), ptr(prob)))


class TXNORConvolutionLayer(TBaseLayer):
    def __init__(self, ABatch, Aheight, Awidth, Achannels, Afilters, AKernelSize=3, AStride=1,
                 APadding=1, AActivation="linear", pad_mode=XNOR_PAD_BIT0):
        self.batch, self.h, self.w, self.c = ABatch, Aheight, Awidth, Achannels
        self.filters, self.kernelSize, self.stride, self.Padding = Afilters, AKernelSize, AStride, APadding
        self.ActivationType = _act(AActivation)
        self.pad_mode = pad_mode
        self.outH = (Aheight + 2 * APadding - AKernelSize) // AStride + 1
        self.outW = (Awidth + 2 * APadding - AKernelSize) // AStride + 1
        self.biases = None

    def upload(self, ctx: Context, weights: np.ndarray):
        self.bind(ctx)
        n = C.c_int64()
        check(lib.tb_xnor_packed_weights_count(self.filters, self.c, self.kernelSize, C.byref(n)))
        w = _dev(ctx, weights)
        self.packed = torch.empty(n.value, dtype=torch.int32, device=ctx.torch_device)
        self.mean = ctx.empty((self.filters,))
        check(lib.tb_xnor_pack_weights(ctx.handle, self.filters, self.c, self.kernelSize, ptr(w),
                                       ptr(self.packed), ptr(self.mean)))

    def forward(self, state: TNNetState, counts: Optional[torch.Tensor] = None):
        x = state.input
        y = self.ctx.empty((x.shape[0], self.filters, self.outH, self.outW))
        check(lib.tb_xnor_conv_fwd(self.ctx.handle, x.shape[0], self.c, self.h, self.w, self.filters,
                                   self.kernelSize, self.stride, self.Padding, self.pad_mode, ptr(x),
                                   ptr(self.packed), ptr(self.mean), ptr(self.biases), self.ActivationType,
                                   ptr(counts), ptr(y)))
        self.output = y
        return y


class TConnectedLayer(TBaseLayer):
    def __init__(self, ABatch, ASteps, AInputs, aOutputs, AActivationType="linear", weights=None, biases=None):
        self.batch, self.inputs, self.outputs = ABatch, AInputs, aOutputs
        self.ActivationType = _act(AActivationType)
        self.weights = weights if weights is not None else np.zeros((aOutputs, AInputs), np.float32)
        self.biases = biases if biases is not None else np.zeros(aOutputs, np.float32)
        self._dev = None

    def upload(self, ctx: Context = None):
        if ctx is not None:
            self.bind(ctx)
        ctx = self.ctx
        d = ConvDesc(self.batch, self.inputs, 1, 1, self.outputs, 1, 1, 1, 1, 0, 0, 1, 1,
                     self.ActivationType, 0, 0, 0)
        n = C.c_int64()
        check(lib.tb_conv_packed_weights_count(C.byref(d), C.byref(n)))
        raw = _dev(ctx, self.weights)
        packed = ctx.empty((n.value,))
        check(lib.tb_conv_pack_weights(ctx.handle, C.byref(d), ptr(raw), ptr(packed)))
        self._dev = (packed, _dev(ctx, self.biases), raw)

    def forward(self, state: TNNetState):
        x = state.input
        if self._dev is None:
            self.upload()
        y = self.ctx.empty((x.shape[0], self.outputs))
        check(lib.tb_fc_fwd(self.ctx.handle, x.shape[0], self.inputs, self.outputs, ptr(x),
                            ptr(self._dev[0]), ptr(self._dev[1]), self.ActivationType, ptr(y)))
        self.output = y
        return y


class TSoftmaxLayer(TBaseLayer):
    def __init__(self, aBatch, aInputs, aGroups=1, temperature=1.0):
        self.batch, self.inputs, self.groups, self.temperature = aBatch, aInputs, aGroups, temperature

    def forward(self, state: TNNetState):
        x = state.input
        y = torch.empty_like(x)
        check(lib.tb_softmax_fwd(self.ctx.handle, x.shape[0], self.inputs, self.groups, self.temperature,
                                 ptr(x), ptr(y)))
        self.output = y
        return y


class TAvgPoolLayer(TBaseLayer):
    def __init__(self, aBatch, aWidth, aHeight, aChannels):
        self.batch, self.w, self.h, self.c = aBatch, aWidth, aHeight, aChannels

    def forward(self, state: TNNetState):
        x = state.input
        y = self.ctx.empty((x.shape[0], self.c))
        check(lib.tb_avgpool_fwd(self.ctx.handle, x.shape[0], self.c, self.h, self.w, ptr(x), ptr(y)))
        self.output = y
        return y
