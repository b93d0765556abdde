"""Data-parallel plumbing for inference across the GPUs of one node.

Every hot-path op is per image, so a batch is partitioned into contiguous slices, one per rank
(one process per GPU), with no collective on the data path.  torch.distributed (NCCL between
GPUs, gloo for CPU tests) is used only for: the max-over-ranks timing, and the optional final
gather of per-image detections to rank 0 in global image order.  (The reference is single-GPU:
multi-GPU appears only as "todo" comments, source/nConvolutionLayer.pas:472,498.)
"""
from __future__ import annotations

import datetime
import os

import numpy as np
import torch
import torch.distributed as dist


def shard(global_batch: int, world: int, rank: int):
    """(start, count) of this rank's contiguous slice: chunks of ceil(B/G) images."""
    if world <= 0 or not (0 <= rank < world):
        raise ValueError("bad world / rank")
    per = -(-global_batch // world)
    start = min(rank * per, global_batch)
    return start, max(0, min(per, global_batch - start))


def init(backend: str = "nccl", timeout_s: float = 120.0, device_id=None):
    """Initialise the process group from torchrun's environment (MASTER_ADDR 127.0.0.1)."""
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    kw = {"timeout": datetime.timedelta(seconds=timeout_s)}
    if device_id is not None:
        kw["device_id"] = device_id
    dist.init_process_group(backend, **kw)
    return dist.get_world_size(), dist.get_rank()


def max_over_ranks(value: float, device=None) -> float:
    if not dist.is_available() or not dist.is_initialized() or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_detections(per_image, dst: int = 0):
    """Gather this rank's list of per-image detection records (any picklable objects, in local
    image order) to rank `dst`; returns the concatenation in global image order on dst, None
    elsewhere."""
    if not dist.is_initialized() or dist.get_world_size() == 1:
        return list(per_image)
    world = dist.get_world_size()
    out = [None] * world if dist.get_rank() == dst else None
    dist.gather_object(list(per_image), out, dst=dst)
    if out is None:
        return None
    merged = []
    for part in out:
        merged.extend(part)
    return merged


def detections_per_image(recs: np.ndarray, probs: np.ndarray, counts: np.ndarray, capacity: int):
    """Split the arrays returned by TNNet.detections into one (records, probs) pair per image."""
    out = []
    for b in range(len(counts)):
        k = int(min(counts[b], capacity))
        out.append((recs[b, :k].copy(), probs[b, :k].copy()))
    return out


class DetectionGather:
    """The final exchange of a sharded forward, through the library's C ABI: every step, each rank
    extracts its images' detections on its GPU (tb_yolo_detect: fixed-capacity records plus
    counts) and tb_group_gather moves the packed buffers [counts (batch int64) | records
    (batch*capacity tb_detection)] to rank 0 over NCCL, in rank order (= global image order).

    The group is formed with tb_group_init_rank; torch.distributed only carries its 128-byte id
    from rank 0 to the others.  With one rank the gather is a device copy."""

    def __init__(self, net, world: int, rank: int, capacity: int = 1024, thresh: float = 0.45,
                 timeout_ms: int = 120000, overlap: bool = False):
        """overlap: each step copies the yolo outputs into staging buffers on the forward's stream
        (a ~30 MB device copy) and runs the extraction, the gather and the download on a side
        stream (a second library context bound to it), so the next forward starts at once;
        join() makes the forward's stream wait for the side stream's last step."""
        import ctypes as C
        from ._lib import Detection, YoloHead, check, lib
        from .context import Context
        self._C, self._lib, self._check = C, lib, check
        self.net, self.world, self.rank = net, world, rank
        self.capacity, self.thresh = capacity, thresh
        self.overlap = overlap
        ctx = net.ctx
        self.sctx = None
        if overlap:
            self.side = torch.cuda.Stream(ctx.torch_device)
            self.sctx = Context(ctx.device, use_torch_stream=False)
            self.sctx.set_stream(self.side)
            self.ev_copied, self.ev_free, self.ev_done = torch.cuda.Event(), torch.cuda.Event(), torch.cuda.Event()
            self._free_recorded = False
        gctx = self.sctx if overlap else ctx
        uid = (C.c_uint8 * 128)()
        if rank == 0:
            check(lib.tb_group_unique_id(uid))
        if world > 1:
            box = [bytes(uid)]
            dist.broadcast_object_list(box, src=0)
            uid = (C.c_uint8 * 128).from_buffer_copy(box[0])
        self.group = C.c_void_p()
        check(lib.tb_group_init_rank(gctx.handle, world, rank, uid, timeout_ms, C.byref(self.group)))
        heads, outs = net.yolo_heads()
        self.heads = heads
        self.outs = outs
        self.stage = [torch.empty_like(o) for o in outs] if overlap else outs
        self.hs = (YoloHead * len(heads))(*[h.head(o) for h, o in zip(heads, self.stage)])
        self.classes = max(h.classes for h in heads)
        B = net.batch
        self.rec_bytes = B * capacity * C.sizeof(Detection)
        self.pack_bytes = 8 * B + self.rec_bytes
        self.pack = torch.zeros(self.pack_bytes, dtype=torch.uint8, device=ctx.torch_device)
        self.prob = torch.empty(B * capacity * self.classes, dtype=torch.float32, device=ctx.torch_device)
        self.sizes = (C.c_int64 * world)(*([self.pack_bytes] * world))
        self.send = (C.c_void_p * 1)(self.pack.data_ptr())
        if rank == 0:
            self.out = torch.empty(world * self.pack_bytes, dtype=torch.uint8, device=ctx.torch_device)
            self.host = torch.empty(world * self.pack_bytes, dtype=torch.uint8).pin_memory()
        else:
            self.out = self.host = None
        torch.cuda.synchronize(ctx.torch_device)  # buffers zeroed before any side-stream use

    def step(self, download: bool = True):
        """Detections of the last forward, gathered on rank 0 (and, with download, copied to its
        pinned host buffer), all queued behind the forward: the counts stay on the device
        (tb_yolo_detect_device) and the NCCL gather is only enqueued (tb_group_gather_async), so
        the host never waits inside a step.  wait() bounds the wait for the queued transfers."""
        C, lib, check = self._C, self._lib, self._check
        ctx = self.net.ctx
        B = self.net.batch
        dctx = ctx
        if self.overlap:
            cs = ctx.stream if hasattr(ctx.stream, "wait_event") else torch.cuda.current_stream(ctx.torch_device)
            with torch.cuda.stream(cs):
                if self._free_recorded:  # the previous extraction has read the staging buffers
                    cs.wait_event(self.ev_free)
                for st, o in zip(self.stage, self.outs):
                    st.copy_(o)
                self.ev_copied.record(cs)
            self.side.wait_event(self.ev_copied)
            dctx = self.sctx
        check(lib.tb_yolo_detect_device(dctx.handle, B, len(self.heads), self.hs, 416, 416, 416, 416, self.thresh,
                                        1, 0, self.capacity, C.c_void_p(self.pack.data_ptr() + 8 * B),
                                        C.c_void_p(self.prob.data_ptr()), C.c_void_p(self.pack.data_ptr())))
        if self.overlap:
            self.ev_free.record(self.side)
            self._free_recorded = True
        out = C.c_void_p(self.out.data_ptr()) if self.out is not None else None
        check(lib.tb_group_gather_async(self.group, self.send, self.sizes, out))
        if download and self.host is not None:
            with torch.cuda.stream(self.side if self.overlap else torch.cuda.current_stream(ctx.torch_device)):
                self.host.copy_(self.out, non_blocking=True)
        if self.overlap:
            self.ev_done.record(self.side)

    def join(self):
        """Make the forward's stream wait for everything the last step queued on the side stream."""
        if self.overlap:
            ctx = self.net.ctx
            cs = ctx.stream if hasattr(ctx.stream, "wait_event") else torch.cuda.current_stream(ctx.torch_device)
            cs.wait_event(self.ev_done)

    def wait(self):
        self._check(self._lib.tb_group_wait(self.group))
        if self.overlap:
            self.side.synchronize()

    @property
    def d2h_bytes(self) -> int:
        return self.world * self.pack_bytes if self.rank == 0 else 0

    def unpack(self):
        """Rank 0, after the last step's copy completed: per global image, its detection records."""
        from .layers import DET_DTYPE
        if self.host is None:
            return None
        B, cap = self.net.batch, self.capacity
        res = []
        raw = self.host.numpy()
        for r in range(self.world):
            part = raw[r * self.pack_bytes:(r + 1) * self.pack_bytes]
            counts = np.minimum(part[:8 * B].view(np.int64), cap)
            recs = part[8 * B:].view(DET_DTYPE).reshape(B, cap)
            res.extend(recs[b, :int(counts[b])].copy() for b in range(B))
        return res

    def close(self):
        if self.group:
            self._lib.tb_group_destroy(self.group)
            self.group = self._C.c_void_p()
        if self.sctx is not None:
            self.sctx.close()
            self.sctx = None
