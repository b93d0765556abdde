"""Input pipeline: decoded 8-bit images to the network's input batch on the GPU.

Mirrors TImageData.loadFromFile + resize / letterBoxEx + toTensor (source/ntypes.pas:651-657,
669-694, 837-943), which the YOLO sample runs on the CPU before predict
(Samples/FPC/MSCOCO_Yolo/MSCOCOYolo.pas:348-350, 454).  File decoding (PNG / JPEG) stays with the
caller's decoder; the bytes it yields are copied to the GPU as bytes (a quarter of the fp32
input), and ``tb_images_to_tensor`` converts, resizes or letterboxes them into the batch, bit-exact
with the reference's single-precision arithmetic.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from ._lib import PIXEL_255, PIXEL_FPC, Image, check, lib
from .context import Context, ptr

__all__ = ["ImagePipeline", "PIXEL_FPC", "PIXEL_255"]


class ImagePipeline:
    """Reusable pinned staging (host) and byte buffer (device) for batches of images."""

    def __init__(self, ctx: Context, pixel_scale: int = PIXEL_FPC):
        self.ctx = ctx
        self.pixel_scale = int(pixel_scale)
        self._host = None
        self._dev = None
        self._copied = None  # event after the last H2D copy out of the pinned buffer

    def _buffers(self, nbytes):
        if self._host is None or self._host.numel() < nbytes:
            n = max(nbytes, 1 << 20)
            self._host = torch.empty(n, dtype=torch.uint8, pin_memory=True)
            self._dev = torch.empty(n, dtype=torch.uint8, device=self.ctx.torch_device)
        return self._host, self._dev

    def upload(self, images, bgr=False):
        """Copy host images (numpy uint8 [h][w] or [h][w][1|3|4]) into the device byte buffer,
        16-byte aligned each; returns their tb_image descriptions."""
        arrs = [np.ascontiguousarray(a, np.uint8) for a in images]
        offs, total = [], 0
        for a in arrs:
            offs.append(total)
            total += (a.nbytes + 15) // 16 * 16
        if self._copied is not None:  # the previous copy may still be reading the pinned buffer
            self._copied.synchronize()
        host, dev = self._buffers(total)
        hv = host.numpy()
        for a, o in zip(arrs, offs):
            hv[o:o + a.nbytes] = a.reshape(-1)
        dev[:total].copy_(host[:total], non_blocking=True)
        self._copied = torch.cuda.Event()
        self._copied.record()
        base = dev.data_ptr()
        descs = []
        for a, o in zip(arrs, offs):
            h, w = a.shape[:2]
            bpp = 1 if a.ndim == 2 else a.shape[2]
            descs.append(Image(base + o, w, h, w * bpp, bpp, 1 if bgr else 0))
        return descs

    def to_tensor(self, images, out_w, out_h, letterbox=False, out=None, bgr=False):
        """Images (host numpy arrays, or tb_image descriptions of device bytes) -> planar fp32 batch
        [n, 3, out_h, out_w] (``out`` may be a slice of a larger input buffer).  Returns
        (out, ratios [n], placements [n, 4] = resized w, h, x offset, y offset)."""
        descs = images if images and isinstance(images[0], Image) else self.upload(images, bgr)
        n = len(descs)
        if out is None:
            out = torch.empty((n, 3, out_h, out_w), dtype=torch.float32, device=self.ctx.torch_device)
        assert out.is_cuda and out.dtype == torch.float32 and out.shape[0] >= n
        assert tuple(out.shape[1:]) == (3, out_h, out_w) and out[0].is_contiguous()
        arr = (Image * max(n, 1))(*descs)
        ratios = (C.c_float * max(n, 1))()
        place = (C.c_int64 * (4 * max(n, 1)))()
        check(lib.tb_images_to_tensor(self.ctx.handle, n, arr, out_w, out_h, 1 if letterbox else 0,
                                      self.pixel_scale, ptr(out), out.stride(0), ratios, place))
        return (out, np.array(ratios[:n], np.float32),
                np.array(place[:4 * n], np.int64).reshape(n, 4))
