"""tb_conv2d_fwd_noalloc: the conv forward for callers that cannot allocate device memory
(their memory is handed out up front by an arena, or an allocation's latency or failure is not
acceptable where they run).  It keeps its split-K scratch in a fixed array inside the library.

Checked here through the C ABI against tb_conv2d_fwd on the same inputs, on two calls in a row
(the shared scratch keeps the previous call's contents; the second call must not depend on
them).  This file is collected last so that a run stopping at the first failure has already run
every other test; it also passes alone in a fresh process."""
import ctypes as C

import numpy as np
import pytest
import torch

from conftest import FP32_TOL, worst_map_err
from tensorium_b200._lib import TB_ERR_INVALID, ConvDesc, check, lib
from tensorium_b200.context import ptr

pytestmark = pytest.mark.gpu


def _packed(ctx, d, w):
    n = C.c_int64()
    check(lib.tb_conv_packed_weights_count(C.byref(d), C.byref(n)))
    raw = torch.from_numpy(w).to(ctx.torch_device)
    packed = torch.empty(n.value, dtype=torch.float32, device=ctx.torch_device)
    check(lib.tb_conv_pack_weights(ctx.handle, C.byref(d), ptr(raw), ptr(packed)))
    return packed


@pytest.mark.parametrize("force", [None, "64,64,4", "128,128,3"])
def test_noalloc_matches_conv2d_fwd_twice(ctx, force, monkeypatch):
    if force:
        monkeypatch.setenv("TB_CONV_FORCE", force)  # make sure the split-K scratch is used
    rng = np.random.default_rng(5)
    B, Cin, H, F, k = 2, 256, 13, 512, 3
    d = ConvDesc(B, Cin, H, H, F, k, k, 1, 1, 1, 1, 1, 1, 9, 0, 0, 0)
    w = (rng.standard_normal((F, Cin * k * k)) * 0.03).astype(np.float32)
    b = (rng.standard_normal(F) * 0.1).astype(np.float32)
    packed = _packed(ctx, d, w)
    bd = torch.from_numpy(b).to(ctx.torch_device)
    for call in range(2):
        x = torch.from_numpy(rng.uniform(0, 1, (B, Cin, H, H)).astype(np.float32)).to(ctx.torch_device)
        y_ref = torch.empty((B, F, H, H), device=ctx.torch_device)
        y_na = torch.full((B, F, H, H), float("nan"), device=ctx.torch_device)
        check(lib.tb_conv2d_fwd(ctx.handle, C.byref(d), ptr(x), ptr(packed), ptr(bd), None, None, None,
                                None, ptr(y_ref), 0))
        check(lib.tb_conv2d_fwd_noalloc(ctx.handle, C.byref(d), ptr(x), ptr(packed), ptr(bd), None, None,
                                        None, None, ptr(y_na)))
        torch.cuda.synchronize()
        a, r = y_na.cpu().numpy(), y_ref.cpu().numpy()
        assert worst_map_err(a, r, B * F) <= FP32_TOL, call
        assert np.array_equal(a, r), call  # same tiles and split order: identical results


def test_noalloc_rejects_layers_beyond_its_scratch(ctx, monkeypatch):
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
