"""Per-GPU context: the Python face of ``tb_ctx`` (TNNCuda.Create / Destroy,
source/nncuda.pas:448-467).

One context per GPU, each with its own stream and scratch workspace; calls on one context are
serialised by the caller, different contexts may be driven from different threads (one per GPU).
torch is used only to own device buffers and to share its current stream, never to compute.
"""
from __future__ import annotations

import ctypes as C
import weakref

import torch

from ._lib import MATH_FP32, Options, check, lib


class Context:
    def __init__(self, device: int = 0, math_mode: int = MATH_FP32, workspace_bytes: int = 0,
                 use_torch_stream: bool = True):
        self.device = int(device)
        self.math_mode = int(math_mode)
        self.handle = C.c_void_p()
        opts = Options(math_mode, workspace_bytes, 0)
        check(lib.tb_init(self.device, C.byref(opts), C.byref(self.handle)))
        self.torch_device = torch.device("cuda", self.device)
        self.stream = None
        self._dependents = weakref.WeakSet()  # objects holding library handles tied to this context
        if use_torch_stream:
            self.set_stream(torch.cuda.current_stream(self.device))

    def set_stream(self, stream) -> None:
        """Launch on a torch.cuda.Stream (or a raw cudaStream_t int)."""
        raw = stream.cuda_stream if hasattr(stream, "cuda_stream") else int(stream)
        check(lib.tb_set_stream(self.handle, C.c_void_p(raw)))
        self.stream = stream

    def sync(self) -> None:
        check(lib.tb_sync(self.handle))

    def reserve(self, nbytes: int) -> None:
        check(lib.tb_workspace_reserve(self.handle, int(nbytes)))

    def empty(self, shape, dtype=torch.float32) -> torch.Tensor:
        return torch.empty(shape, dtype=dtype, device=self.torch_device)

    def adopt(self, obj) -> None:
        """Register an object with a close() that must run before this context shuts down."""
        self._dependents.add(obj)

    def close(self) -> None:
        if self.handle:
            for d in list(self._dependents):
                d.close()
            lib.tb_shutdown(self.handle)
            self.handle = C.c_void_p()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def ptr(t) -> C.c_void_p:
    """Device (or host) address of a tensor / numpy array, or NULL for None."""
    if t is None:
        return C.c_void_p(0)
    if isinstance(t, torch.Tensor):
        return C.c_void_p(t.data_ptr())
    return C.c_void_p(t.ctypes.data)


def device_count() -> int:
    n = C.c_int64()
    check(lib.tb_device_count(C.byref(n)))
    return n.value
