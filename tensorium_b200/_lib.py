"""ctypes binding of the C ABI in include/tensorium_b200.h.

The shared library is built in-tree (``python -m tensorium_b200.build``).  There is no CPU
fallback: importing this module without the library raises ImportError, and every failed call
raises :class:`TBError` with the library's own message.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libtensorium_b200.so"

TB_OK = 0
TB_ERR_INVALID = -1
TB_ERR_CUDA = -2
TB_ERR_UNSUPPORTED = -3
TB_ERR_OOM = -4
TB_ERR_TIMEOUT = -5
TB_ERR_STATE = -6
TB_ERR_DEVICE = -7

# TActivationType ordinals (source/ntypes.pas:66-71)
ACT = {
    "logistic": 0, "relu": 1, "relu6": 2, "relie": 3, "linear": 4, "ramp": 5, "tanh": 6,
    "plse": 7, "revleaky": 8, "leaky": 9, "elu": 10, "loggy": 11, "hardtan": 13, "lhtan": 14,
    "selu": 15,
}

MATH_FP32 = 0
MATH_TF32 = 1
MATH_FP32_TILED = 2  # FP32 with the summation reordered (tiles, split-K): not bit-exact
MATH_BF16_SPLIT = 3  # tensor cores on bf16 (hi, lo) operand pairs, networks only

XNOR_PAD_BIT0 = 0
XNOR_PAD_ZERO = 1


class TBError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"[{code}] {msg}")
        self.code = code


class ConvDesc(C.Structure):
    _fields_ = [(n, C.c_int64) for n in (
        "batch", "channels", "height", "width", "filters", "kernel_h", "kernel_w",
        "stride_y", "stride_x", "pad_y", "pad_x", "dilation_y", "dilation_x", "activation",
        "in_batch_stride", "out_batch_stride", "res_batch_stride")]


class Options(C.Structure):
    _fields_ = [("math_mode", C.c_int64), ("workspace_bytes", C.c_int64), ("flags", C.c_int64)]


class Detection(C.Structure):
    _fields_ = [("x", C.c_float), ("y", C.c_float), ("w", C.c_float), ("h", C.c_float),
                ("objectness", C.c_float), ("batch", C.c_int32), ("head", C.c_int32),
                ("index", C.c_int32), ("anchor", C.c_int32), ("reserved", C.c_int32 * 3)]


class YoloHead(C.Structure):
    _fields_ = [("output", C.c_void_p), ("n", C.c_int64), ("classes", C.c_int64),
                ("h", C.c_int64), ("w", C.c_int64), ("mask_host", C.c_void_p),
                ("anchors_host", C.c_void_p), ("new_coords", C.c_int64)]


class Image(C.Structure):
    _fields_ = [("pixels", C.c_void_p), ("width", C.c_int64), ("height", C.c_int64),
                ("row_stride", C.c_int64), ("bytes_per_pixel", C.c_int64), ("bgr", C.c_int64)]


PIXEL_FPC = 0
PIXEL_255 = 1


class LayerInfo(C.Structure):
    _fields_ = [(n, C.c_int64) for n in (
        "type", "c", "h", "w", "out_c", "out_h", "out_w", "filters", "ksize", "stride", "pad",
        "activation", "batch_normalize", "from_", "n_inputs", "classes", "n", "total_anchors",
        "groups")] + [("scale", C.c_float), ("reserved", C.c_float), ("weights_count", C.c_int64)]


# TB_LAYER_* / TB_PARAM_* (include/tensorium_b200.h)
LAYER_TYPES = {1: "conv", 2: "shortcut", 3: "route", 4: "upsample", 5: "yolo", 6: "maxpool",
               7: "connected", 8: "softmax", 9: "avgpool"}
PARAM = {"weights": 0, "biases": 1, "scales": 2, "mean": 3, "var": 4, "route_inputs": 5,
         "yolo_mask": 6, "yolo_anchors": 7}

P = C.c_void_p
I64 = C.c_int64
F32 = C.c_float
PI64 = C.POINTER(C.c_int64)

# name -> argtypes (all return int unless listed in _RESTYPES)
SIGNATURES = {
    "tb_version": [],
    "tb_device_count": [PI64],
    "tb_init": [I64, C.POINTER(Options), C.POINTER(P)],
    "tb_shutdown": [P],
    "tb_set_stream": [P, P],
    "tb_get_stream": [P],
    "tb_sync": [P],
    "tb_malloc": [P, I64, C.POINTER(P)],
    "tb_free": [P, P],
    "tb_memcpy_h2d": [P, P, P, I64],
    "tb_memcpy_d2h": [P, P, P, I64],
    "tb_workspace_reserve": [P, I64],
    "tb_workspace_size": [P, C.POINTER(I64)],
    "tb_activate": [P, I64, P, I64, I64],
    "tb_forward_bias": [P, I64, P, I64, I64, P, I64, I64],
    "tb_copy": [P, I64, P, I64, I64, P, I64, I64],
    "tb_fill": [P, I64, P, I64, F32, I64],
    "tb_addvv": [P, I64, P, I64, I64, P, I64, I64, P, I64, I64],
    "tb_fmavss": [P, I64, P, I64, F32, F32, P],
    "tb_bn_fwd": [P, I64, I64, I64, P, P, P, P, P, P],
    "tb_group_available": [PI64],
    "tb_group_init": [I64, PI64, C.POINTER(P)],
    "tb_group_unique_id": [P],
    "tb_group_init_rank": [P, I64, I64, P, I64, C.POINTER(P)],
    "tb_group_size": [P, PI64, PI64, PI64],
    "tb_group_context": [P, I64, C.POINTER(P)],
    "tb_group_gather": [P, C.POINTER(P), PI64, P],
    "tb_group_gather_async": [P, C.POINTER(P), PI64, P],
    "tb_group_wait": [P],
    "tb_group_destroy": [P],
    # TNNCuda method shims (argument lists of source/nncuda.pas:100-151)
    "tbcompat_createDeviceBuffer": [P, I64, C.POINTER(P)],
    "tbcompat_freeDeviceBuffer": [P, P],
    "tbcompat_readBuffer": [P, P, I64, P],
    "tbcompat_writeBuffer": [P, P, I64, P],
    "tbcompat_finish": [P],
    "tbcompat_ActivateArray": [P, I64, P, I64, C.c_int32],
    "tbcompat_forwardBias": [P, I64, P, I64, I64, P, I64, I64],
    "tbcompat_forwardScale": [P, I64, P, I64, I64, P, I64, I64],
    "tbcompat_forwardScaleAdd": [P, I64, P, I64, I64, P, P, I64, I64],
    "tbcompat_normalize": [P, I64, I64, I64, P, I64, P, I64, P, I64],
    "tbcompat_gemm": [P, C.c_int32, C.c_int32, I64, I64, I64, F32, P, I64, I64, P, I64, I64, F32, P, I64, I64],
    "tbcompat_gemmStridedBatched": [P, C.c_int32, C.c_int32, I64, I64, I64, F32, P, I64, I64, I64, P, I64, I64,
                                    I64, F32, P, I64, I64, I64, I64],
    "tbcompat_addvv": [P, I64, P, I64, I64, P, I64, I64, P, I64, I64],
    "tbcompat_fill": [P, I64, P, I64, F32, I64],
    "tbcompat_copy": [P, I64, P, I64, I64, P, I64, I64],
    "tbcompat_fmavss": [P, I64, P, I64, F32, F32, P],
    "tbcompat_softmaxBatch": [P, I64, P, I64, I64, I64, I64, I64, I64, F32, P, I64],
    "tbcompat_forwardMaxPool": [P, I64, I64, I64, I64, P, I64, I64, I64, I64, I64, I64, I64, P, P],
    "tbcompat_im2col": [P, I64, I64, I64, I64, I64, I64, I64, I64, I64, I64, I64, P, I64, P, I64],
    "tbcompat_upSample": [P, I64, I64, I64, I64, P, I64, C.c_int32, F32, P, C.c_int32],
    "tb_conv_out_shape": [C.POINTER(ConvDesc), PI64, PI64],
    "tb_conv_packed_weights_count": [C.POINTER(ConvDesc), PI64],
    "tb_conv_pack_weights": [P, C.POINTER(ConvDesc), P, P],
    "tb_conv_uses_tensor_cores": [C.POINTER(ConvDesc), I64, PI64],
    "tb_conv_pack_weights_tf32": [P, C.POINTER(ConvDesc), P, P],
    "tb_conv_fold_bn": [I64, I64, P, P, P, P, P],
    "tb_conv_nhwc_packed_count": [C.POINTER(ConvDesc), PI64],
    "tb_conv_pack_weights_nhwc": [P, C.POINTER(ConvDesc), P, P],
    "tb_conv2d_fwd_nhwc": [P, C.POINTER(ConvDesc), P, I64, P, P, P, I64, P, I64],
    "tb_conv_autotune": [P, C.POINTER(ConvDesc), P, P, P],
    "tb_conv2d_fwd": [P, C.POINTER(ConvDesc), P, P, P, P, P, P, P, P, I64],
    "tb_conv2d_fwd_noalloc": [P, C.POINTER(ConvDesc), P, P, P, P, P, P, P, P],
    "tb_maxpool_fwd": [P, I64, I64, I64, I64, I64, I64, I64, I64, P, P, P],
    "tb_upsample_fwd": [P, I64, I64, I64, I64, I64, F32, P, P, I64],
    "tb_route_fwd": [P, I64, I64, P, P, P, I64],
    "tb_shortcut_fwd": [P, I64, P, P, P, I64],
    "tb_yolo_fwd": [P, I64, I64, I64, I64, I64, P, P, F32],
    "tb_yolo_detect": [P, I64, I64, C.POINTER(YoloHead), I64, I64, I64, I64, F32, I64, I64, I64,
                       P, P, PI64],
    "tb_yolo_detect_device": [P, I64, I64, C.POINTER(YoloHead), I64, I64, I64, I64, F32, I64, I64, I64,
                       P, P, P],
    "tb_yolo_nms": [P, I64, I64, PI64, I64, F32, P, P],
    "tb_xnor_packed_weights_count": [I64, I64, I64, PI64],
    "tb_xnor_pack_weights": [P, I64, I64, I64, P, P, P],
    "tb_xnor_conv_fwd": [P, I64, I64, I64, I64, I64, I64, I64, I64, I64, P, P, P, P, I64, P, P],
    "tb_fc_fwd": [P, I64, I64, I64, P, P, P, I64, P],
    "tb_softmax_fwd": [P, I64, I64, I64, F32, P, P],
    "tb_avgpool_fwd": [P, I64, I64, I64, I64, P, P],
    "tb_net_create": [P, I64, I64, I64, I64, C.POINTER(P)],
    "tb_net_destroy": [P],
    "tb_net_add_conv": [P, I64, I64, I64, I64, I64, I64, P, P, P, P, P],
    "tb_net_add_shortcut": [P, I64, I64],
    "tb_net_add_route": [P, I64, P],
    "tb_net_add_upsample": [P, I64, F32],
    "tb_net_add_yolo": [P, I64, I64, P, I64, P, F32],
    "tb_net_add_maxpool": [P, I64, I64, I64],
    "tb_net_add_connected": [P, I64, I64, P, P],
    "tb_net_add_softmax": [P, I64, F32],
    "tb_net_add_avgpool": [P],
    "tb_net_set_fusion": [P, I64],
    "tb_net_fuse_batchnorm": [P],
    "tb_net_finalize": [P, I64],
    "tb_net_forward": [P, P, I64],
    "tb_net_layer_output": [P, I64, C.POINTER(P), PI64, PI64],
    "tb_net_layer_count": [P, PI64],
    "tb_net_layer_layout": [P, I64, PI64],
    "tb_net_launch_count": [P, PI64],
    "tb_net_flops": [P, C.POINTER(C.c_double)],
    "tb_net_profile": [P, P, C.POINTER(C.c_double)],
    "tb_net_input_shape": [P, PI64, PI64, PI64, PI64],
    "tb_net_layer_info": [P, I64, C.POINTER(LayerInfo)],
    "tb_net_layer_param": [P, I64, I64, P, I64, PI64],
    "tb_images_to_tensor": [P, I64, C.POINTER(Image), I64, I64, I64, I64, P, I64,
                            C.POINTER(C.c_float), PI64],
    "tb_darknet_load": [P, C.c_char_p, C.c_char_p, I64, I64, C.POINTER(P)],
    "tb_darknet_save_weights": [P, C.c_char_p, I64],
    "tb_diag_fp32_fma_tflops": [P, C.POINTER(C.c_double)],
    "tb_diag_popc_tbitmac": [P, C.POINTER(C.c_double)],
    "tb_diag_tc_mma_rate": [P, I64, C.POINTER(C.c_double), C.POINTER(C.c_double)],
    "tb_diag_conv_tc_phases": [P, P, P, P, P, C.POINTER(C.c_double)],
    "tb_diag_conv_nhwc_phases": [P, P, P, I64, P, P, I64, C.POINTER(C.c_double)],
}
_RESTYPES = {"tb_get_stream": P}


def _load():
    if not LIB_PATH.exists():
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `python -m tensorium_b200.build` "
            "(this package has no CPU fallback)")
    lib = C.CDLL(str(LIB_PATH))
    lib.tb_last_error.restype = C.c_char_p
    lib.tb_last_error.argtypes = []
    for name, args in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = _RESTYPES.get(name, C.c_int)
    return lib


lib = _load()


def last_error() -> str:
    return lib.tb_last_error().decode(errors="replace")


def check(rc: int) -> int:
    """Raise TBError for a negative status; return non-negative values (layer indices)."""
    if rc < 0:
        raise TBError(rc, last_error())
    return rc
