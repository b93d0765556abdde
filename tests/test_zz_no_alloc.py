"""tb_conv2d_fwd_noalloc: the conv forward for callers that cannot allocate device memory
(their memory is handed out up front by an arena, or an allocation's latency or failure is not
acceptable where they run).  It runs the tiled FP32 kernels (the results of tb_conv2d_fwd with
TB_MATH_FP32_TILED) and keeps their split-K scratch in a fixed array inside the library.

Checked here through the C ABI against tb_conv2d_fwd on the same inputs and against the CPU
oracle (the tiled kernels reorder the sum: max|a-b|/max|b| <= 1e-4 per map), on two calls in a
row (the shared scratch keeps the previous call's contents; the second call must not depend on
them); that a fresh context's workspace does not grow; and that a YOLOv3 batch-8 13x13 layer,
whose chosen split would exceed the scratch, runs with a lower split.  This file is collected
last so that a run stopping at the first failure has already run every other test; it also
passes alone in a fresh process."""
import ctypes as C

import numpy as np
import pytest
import torch

from conftest import FP32_TOL, worst_map_err
from oracle import oracle as O
from tensorium_b200 import MATH_FP32_TILED
from tensorium_b200._lib import TB_ERR_INVALID, ConvDesc, check, lib
from tensorium_b200.context import Context, ptr

pytestmark = pytest.mark.gpu


def _packed(ctx, d, w):
    n = C.c_int64()
    check(lib.tb_conv_packed_weights_count(C.byref(d), C.byref(n)))
    raw = torch.from_numpy(w).to(ctx.torch_device)
    packed = torch.empty(n.value, dtype=torch.float32, device=ctx.torch_device)
    check(lib.tb_conv_pack_weights(ctx.handle, C.byref(d), ptr(raw), ptr(packed)))
    return packed


def _ws_bytes(ctx):
    n = C.c_int64()
    check(lib.tb_workspace_size(ctx.handle, C.byref(n)))
    return n.value


def _layer(rng, B, Cin, H, F, k=3):
    d = ConvDesc(B, Cin, H, H, F, k, k, 1, 1, k // 2, k // 2, 1, 1, 9, 0, 0, 0)
    w = (rng.standard_normal((F, Cin * k * k)) * np.sqrt(2.0 / (Cin * k * k))).astype(np.float32)
    b = (rng.standard_normal(F) * 0.1).astype(np.float32)
    return d, w, b


@pytest.mark.parametrize("force", [None, "64,64,4", "128,128,3"])
def test_noalloc_matches_conv2d_fwd_twice(ctx, force, monkeypatch):
    if force:
        monkeypatch.setenv("TB_CONV_FORCE", force)  # make sure the split-K scratch is used
    rng = np.random.default_rng(5)
    B, Cin, H, F = 2, 256, 13, 512
    d, w, b = _layer(rng, B, Cin, H, F)
    packed = _packed(ctx, d, w)
    bd = torch.from_numpy(b).to(ctx.torch_device)
    for call in range(2):
        xh = rng.uniform(0, 1, (B, Cin, H, H)).astype(np.float32)
        x = torch.from_numpy(xh).to(ctx.torch_device)
        y_ref = torch.empty((B, F, H, H), device=ctx.torch_device)
        y_na = torch.full((B, F, H, H), float("nan"), device=ctx.torch_device)
        check(lib.tb_conv2d_fwd(ctx.handle, C.byref(d), ptr(x), ptr(packed), ptr(bd), None, None, None,
                                None, ptr(y_ref), MATH_FP32_TILED))
        check(lib.tb_conv2d_fwd_noalloc(ctx.handle, C.byref(d), ptr(x), ptr(packed), ptr(bd), None, None,
                                        None, None, ptr(y_na)))
        torch.cuda.synchronize()
        a, r = y_na.cpu().numpy(), y_ref.cpu().numpy()
        assert np.array_equal(a, r), call  # same tiles and split order: identical results
        assert worst_map_err(a, O.conv2d(xh, w, b, F, 3, 1, 1, 9), B * F) <= FP32_TOL, call


def test_noalloc_on_a_fresh_context_allocates_nothing(monkeypatch):
    """Only the no-alloc entry point runs on a context with a 1 MiB workspace, with a pinned split
    whose partial sums (2.8 MB) exceed it: the workspace does not grow, the result is right."""
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    monkeypatch.setenv("TB_CONV_FORCE", "64,64,4")
    rng = np.random.default_rng(6)
    B, Cin, H, F = 2, 256, 13, 512
    with Context(0, workspace_bytes=1 << 20) as c:
        d, w, b = _layer(rng, B, Cin, H, F)
        packed = _packed(c, d, w)
        bd = torch.from_numpy(b).to(c.torch_device)
        xh = rng.uniform(0, 1, (B, Cin, H, H)).astype(np.float32)
        x = torch.from_numpy(xh).to(c.torch_device)
        y = torch.empty((B, F, H, H), device=c.torch_device)
        before = _ws_bytes(c)
        for _ in range(2):
            check(lib.tb_conv2d_fwd_noalloc(c.handle, C.byref(d), ptr(x), ptr(packed), ptr(bd), None, None,
                                            None, None, ptr(y)))
        torch.cuda.synchronize()
        assert _ws_bytes(c) == before <= (1 << 20)
        assert worst_map_err(y.cpu().numpy(), O.conv2d(xh, w, b, F, 3, 1, 1, 9), B * F) <= FP32_TOL


def test_noalloc_lowers_the_split_of_a_yolov3_batch8_layer(ctx):
    """YOLOv3 layer 64 at batch 8 (512 -> 1024 filters, 3x3, 13x13): the split the tiled kernels
    choose needs more than the 16 MiB of static scratch, so the entry point lowers it; the result
    is within the tiled path's bound of the oracle and the same on a second call."""
    rng = np.random.default_rng(7)
    B, Cin, H, F = 8, 512, 13, 1024
    d, w, b = _layer(rng, B, Cin, H, F)
    packed = _packed(ctx, d, w)
    bd = torch.from_numpy(b).to(ctx.torch_device)
    xh = rng.uniform(0, 1, (B, Cin, H, H)).astype(np.float32)
    x = torch.from_numpy(xh).to(ctx.torch_device)
    ys = []
    for _ in range(2):
        y = torch.full((B, F, H, H), float("nan"), device=ctx.torch_device)
        check(lib.tb_conv2d_fwd_noalloc(ctx.handle, C.byref(d), ptr(x), ptr(packed), ptr(bd), None, None,
                                        None, None, ptr(y)))
        ys.append(y.cpu().numpy())
    assert np.array_equal(ys[0], ys[1])
    ref = np.concatenate([O.conv2d(xh[i:i + 1], w, b, F, 3, 1, 1, 9) for i in range(B)])
    assert worst_map_err(ys[0], ref, B * F) <= FP32_TOL


def test_noalloc_rejects_a_pinned_split_beyond_its_scratch(ctx, monkeypatch):
    monkeypatch.setenv("TB_CONV_FORCE", "128,128,8")
    B, Cin, H, F = 8, 256, 52, 512  # 8 splits x 512 x 21632 floats >> 16 MiB
    d = ConvDesc(B, Cin, H, H, F, 3, 3, 1, 1, 1, 1, 1, 1, 9, 0, 0, 0)
    w = np.zeros((F, Cin * 9), np.float32)
    packed = _packed(ctx, d, w)
    x = torch.zeros((B, Cin, H, H), device=ctx.torch_device)
    y = torch.empty((B, F, H, H), device=ctx.torch_device)
    rc = lib.tb_conv2d_fwd_noalloc(ctx.handle, C.byref(d), ptr(x), ptr(packed), None, None, None, None,
                                   None, ptr(y))
    assert rc == TB_ERR_INVALID
    assert "static scratch" in lib.tb_last_error().decode()
