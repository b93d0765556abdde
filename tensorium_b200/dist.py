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
