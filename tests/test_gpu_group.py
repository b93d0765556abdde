"""The multi-GPU group of the C ABI (tb_group_*, NCCL): the gather of per-GPU results to rank 0,
a group driven by one process and a group of one process per GPU, and the bounded wait when a
rank never joins (the failure is made on the host: the second rank is simply never started)."""
import ctypes as C
import os
import subprocess
import sys
import textwrap

import numpy as np
import pytest
import torch

from tensorium_b200._lib import TB_ERR_TIMEOUT, check, lib
from tensorium_b200.context import Context, ptr

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_nccl_loads():
    v = C.c_int64()
    check(lib.tb_group_available(C.byref(v)))
    assert v.value >= 22700


@pytest.mark.parametrize("ngpu", [1, 2])
def test_single_process_group_gather(ngpu):
    if torch.cuda.device_count() < ngpu:
        pytest.skip(f"needs {ngpu} GPUs")
    g = C.c_void_p()
    devs = (C.c_int64 * ngpu)(*range(ngpu))
    check(lib.tb_group_init(ngpu, devs, C.byref(g)))
    try:
        sizes = [1000 + 24 * r for r in range(ngpu)]
        bufs = []
        for r in range(ngpu):
            bufs.append(torch.arange(sizes[r], dtype=torch.uint8, device=f"cuda:{r}") + r)
        out = torch.zeros(sum(sizes), dtype=torch.uint8, device="cuda:0")
        send = (C.c_void_p * ngpu)(*[b.data_ptr() for b in bufs])
        nbytes = (C.c_int64 * ngpu)(*sizes)
        for _ in range(2):
            check(lib.tb_group_gather(g, send, nbytes, C.c_void_p(out.data_ptr())))
        want = torch.cat([b.cpu() for b in bufs])
        assert torch.equal(out.cpu(), want)
    finally:
        lib.tb_group_destroy(g)


def test_rank_that_never_joins_times_out():
    """Rank 0 of a 2-rank group whose rank 1 is never started: the non-blocking NCCL
    initialisation runs into its 3 s deadline, the communicator is aborted and the call returns
    TB_ERR_TIMEOUT (no hang); the context stays usable."""
    with Context(0) as c:
        uid = (C.c_uint8 * 128)()
        check(lib.tb_group_unique_id(uid))
        g = C.c_void_p()
        rc = lib.tb_group_init_rank(c.handle, 2, 0, uid, 3000, C.byref(g))
        assert rc == TB_ERR_TIMEOUT, rc
        assert "did not take part" in lib.tb_last_error().decode()
        x = torch.ones(16, device=c.torch_device)
        check(lib.tb_fill(c.handle, 16, ptr(x), 0, 2.0, 1))
        c.sync()
        assert float(x.sum()) == 32.0


WORKER = textwrap.dedent("""
    import ctypes as C, sys, time, os
    sys.path.insert(0, {root!r})
    import torch
    from tensorium_b200._lib import check, lib
    from tensorium_b200.context import Context
    rank, n, idfile = int(sys.argv[1]), int(sys.argv[2]), sys.argv[3]
    with Context(rank) as c:
        if rank == 0:
            uid = (C.c_uint8 * 128)()
            check(lib.tb_group_unique_id(uid))
            open(idfile + ".tmp", "wb").write(bytes(uid)); os.rename(idfile + ".tmp", idfile)
        else:
            while not os.path.exists(idfile): time.sleep(0.01)
            uid = (C.c_uint8 * 128).from_buffer_copy(open(idfile, "rb").read())
        g = C.c_void_p()
        check(lib.tb_group_init_rank(c.handle, n, rank, uid, 30000, C.byref(g)))
        sizes = [512 * (r + 1) for r in range(n)]
        buf = torch.full((sizes[rank],), rank + 7, dtype=torch.uint8, device=c.torch_device)
        out = torch.zeros(sum(sizes), dtype=torch.uint8, device=c.torch_device)
        send = (C.c_void_p * 1)(buf.data_ptr())
        check(lib.tb_group_gather(g, send, (C.c_int64 * n)(*sizes), C.c_void_p(out.data_ptr())))
        if rank == 0:
            want = torch.cat([torch.full((sizes[r],), r + 7, dtype=torch.uint8) for r in range(n)])
            assert torch.equal(out.cpu(), want)
        lib.tb_group_destroy(g)
    print("ok", rank)
""")


def test_one_process_per_gpu_group(tmp_path):
    n = min(torch.cuda.device_count(), 4)
    if n < 2:
        pytest.skip("needs 2 GPUs")
    script = tmp_path / "worker.py"
    script.write_text(WORKER.format(root=ROOT))
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    procs = [subprocess.Popen([sys.executable, str(script), str(r), str(n), str(tmp_path / "uid")], env=env,
                              stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True) for r in range(n)]
    outs = [p.communicate(timeout=180)[0] for p in procs]
    for r, (p, o) in enumerate(zip(procs, outs)):
        assert p.returncode == 0, o
        assert f"ok {r}" in o
