"""Multi-rank host logic on CPU (gloo, world size 2): batch sharding, max-over-ranks timing,
ordered gather of detections, and failure detection when a rank dies before a collective.
No GPU is involved; the failure is made on the host (a rank that exits), never on a device."""
import os
import socket
import sys

import numpy as np
import pytest
import torch.multiprocessing as mp

from conftest import ROOT


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, mode, q):
    sys.path.insert(0, str(ROOT))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    import torch.distributed as dist
    from tensorium_b200 import dist as tbd
    try:
        tbd.init("gloo", timeout_s=5.0 if mode == "fail" else 60.0)
        if mode == "fail":
            if rank == 1:
                os._exit(3)  # this rank dies between steps, before the collective
            try:
                tbd.max_over_ranks(1.0)
                q.put((rank, "no-error"))
            except Exception as e:  # the survivor sees an error instead of hanging
                q.put((rank, "error:" + type(e).__name__))
            return
        start, count = tbd.shard(13, world, rank)
        per_image = [("img", start + i) for i in range(count)]
        t = tbd.max_over_ranks(10.0 * (rank + 1))
        merged = tbd.gather_detections(per_image)
        q.put((rank, (start, count, t, merged)))
        dist.destroy_process_group()
    except Exception as e:
        q.put((rank, "exception:" + repr(e)))


def _run(mode, world=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    expected = world if mode != "fail" else 1
    for _ in range(expected):
        r, v = q.get(timeout=120)
        res[r] = v
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return res


def test_shard_covers_batch_exactly():
    from tensorium_b200.dist import shard
    for B in (1, 7, 64, 1024):
        for G in (1, 2, 3, 4, 8):
            seen = []
            for r in range(G):
                s, c = shard(B, G, r)
                seen.extend(range(s, s + c))
            assert seen == list(range(B))


def test_two_ranks_time_and_gather():
    res = _run("ok")
    s0, c0, t0, merged = res[0]
    s1, c1, t1, none = res[1]
    assert (s0, c0, s1, c1) == (0, 7, 7, 6)
    assert t0 == t1 == 20.0  # max over ranks
    assert merged == [("img", i) for i in range(13)] and none is None  # global image order on rank 0


def test_dead_rank_is_detected_not_hung():
    res = _run("fail")
    assert res[0].startswith("error:"), res
