"""TNNCuda method shims (tbcompat_*) and tb_bn_fwd through the C ABI against the CPU oracle.

The shims keep the reference CPU routines' arithmetic, so every comparison is bit for bit: the
four GEMM orders of cblas_sgemm, the reference's own GPU conv sequence (im2col per image,
gemmStridedBatched, forwardBias, ActivateArray) rebuilt from the shims against the oracle conv,
the unfused batchnorm sequence (normalize, forwardScale, forwardBias) and tb_bn_fwd, maxpool,
upsample, softmax and the BLAS-1 helpers."""
import ctypes as C

import numpy as np
import pytest
import torch

from conftest import assert_bit_exact, logistic_ulps
from oracle import oracle as O
from tensorium_b200._lib import TB_ERR_UNSUPPORTED, check, lib
from tensorium_b200.context import ptr

pytestmark = pytest.mark.gpu


def dev(ctx, a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(ctx.torch_device)


@pytest.mark.parametrize("ta,tb", [(0, 0), (0, 1), (1, 0), (1, 1)])
@pytest.mark.parametrize("alpha,beta", [(1.0, 0.0), (1.5, 0.5), (0.75, 1.0)])
def test_gemm_orders(ctx, ta, tb, alpha, beta):
    rng = np.random.default_rng(10 * ta + tb)
    M, N, K = 37, 53, 129
    lda, ldb, ldc = (M if ta else K) + 3, (K if tb else N) + 5, N + 2
    A = rng.standard_normal(((K if ta else M), lda)).astype(np.float32)
    B = rng.standard_normal(((N if tb else K), ldb)).astype(np.float32)
    Cm = rng.standard_normal((M, ldc)).astype(np.float32)
    want = O.sgemm(ta, tb, M, N, K, alpha, A, lda, B, ldb, beta, Cm, ldc)
    a_off, b_off, c_off = 7, 3, 11
    Ad = dev(ctx, np.r_[np.zeros(a_off, np.float32), A.ravel()])
    Bd = dev(ctx, np.r_[np.zeros(b_off, np.float32), B.ravel()])
    Cd = dev(ctx, np.r_[np.zeros(c_off, np.float32), Cm.ravel()])
    check(lib.tbcompat_gemm(ctx.handle, ta, tb, M, N, K, alpha, ptr(Ad), a_off, lda, ptr(Bd), b_off, ldb, beta,
                            ptr(Cd), c_off, ldc))
    got = Cd.cpu().numpy()[c_off:].reshape(M, ldc)
    assert_bit_exact(got, want, M, (ta, tb, alpha, beta))


def test_reference_gpu_conv_sequence_from_shims(ctx):
    """TConvolutionalLayer.forwardGPU's sequence (source/nConvolutionLayer.pas:1055-1122): im2col
    per image, one gemmStridedBatched over the batch, forwardBias, ActivateArray -- rebuilt from
    the shims, it equals the oracle's conv bit for bit."""
    rng = np.random.default_rng(3)
    B, Cc, H, F, k, s, p = 3, 16, 19, 24, 3, 2, 1
    x = rng.uniform(0, 1, (B, Cc, H, H)).astype(np.float32)
    w = (rng.standard_normal((F, Cc * k * k)) * 0.2).astype(np.float32)
    b = (rng.standard_normal(F) * 0.1).astype(np.float32)
    oh = (H + 2 * p - k) // s + 1
    K, Nn = Cc * k * k, oh * oh
    xd, wd, bd = dev(ctx, x), dev(ctx, w), dev(ctx, b)
    col = torch.empty(B * K * Nn, device=ctx.torch_device)
    y = torch.zeros(B * F * Nn, device=ctx.torch_device)
    for i in range(B):
        check(lib.tbcompat_im2col(ctx.handle, Cc, H, H, k, k, p, p, s, s, 1, 1, ptr(xd), i * Cc * H * H, ptr(col),
                                  i * K * Nn))
    check(lib.tbcompat_gemmStridedBatched(ctx.handle, 0, 0, F, Nn, K, 1.0, ptr(wd), 0, K, 0, ptr(col), 0, Nn, K * Nn,
                                          0.0, ptr(y), 0, Nn, F * Nn, B))
    check(lib.tbcompat_forwardBias(ctx.handle, B * F * Nn, ptr(y), 0, F, ptr(bd), 1, B))
    check(lib.tbcompat_ActivateArray(ctx.handle, B * F * Nn, ptr(y), 0, 9))
    want = O.conv2d(x, w, b, F, k, s, p, 9)
    assert_bit_exact(y.cpu().numpy().reshape(want.shape), want, B * F, "conv from shims")
    # the im2col layout itself is the oracle's sim2Col
    cref = np.zeros((K, Nn), np.float32)
    lib_o = O.lib
    lib_o.or_im2col(Cc, H, H, k, k, p, p, s, s, 1, 1, O._p(np.ascontiguousarray(x[2])), O._p(cref))
    assert np.array_equal(col.cpu().numpy()[2 * K * Nn:].reshape(K, Nn), cref)


def test_batchnorm_sequence_and_tb_bn_fwd(ctx):
    rng = np.random.default_rng(4)
    B, Cc, S = 3, 10, 7 * 7
    x = rng.standard_normal((B, Cc, S)).astype(np.float32) * 3
    mean = rng.standard_normal(Cc).astype(np.float32)
    var = rng.uniform(0.5, 1.5, Cc).astype(np.float32)
    var[0] = 1e-9  # max(sqrt(var), 1e-6) binds
    sc = rng.uniform(0.5, 2, Cc).astype(np.float32)
    bi = rng.standard_normal(Cc).astype(np.float32)
    want = O.conv2d(x.reshape(B, Cc, 7, 7), np.eye(Cc, dtype=np.float32), bi, Cc, 1, 1, 0, 4,
                    bn=(sc, mean, var)).reshape(B, Cc, S)  # identity 1x1 conv + unfused batchnorm
    xd = dev(ctx, x)
    md, vd, sd, bd = dev(ctx, mean), dev(ctx, var), dev(ctx, sc), dev(ctx, bi)
    y = xd.clone()
    check(lib.tbcompat_normalize(ctx.handle, Cc, B * Cc * S, B, ptr(md), 1, ptr(vd), 1, ptr(y), 0))
    check(lib.tbcompat_forwardScale(ctx.handle, B * Cc * S, ptr(y), 0, Cc, ptr(sd), 1, B))
    check(lib.tbcompat_forwardBias(ctx.handle, B * Cc * S, ptr(y), 0, Cc, ptr(bd), 1, B))
    assert_bit_exact(y.cpu().numpy(), want, B * Cc, "normalize / forwardScale / forwardBias")
    y2 = torch.empty_like(xd)
    check(lib.tb_bn_fwd(ctx.handle, B, Cc, S, ptr(xd), ptr(md), ptr(vd), ptr(sd), ptr(bd), ptr(y2)))
    assert_bit_exact(y2.cpu().numpy(), want, B * Cc, "tb_bn_fwd")
    y3 = xd.clone()
    check(lib.tbcompat_forwardScaleAdd(ctx.handle, B * Cc * S, ptr(y3), 0, Cc, ptr(sd), ptr(bd), 1, B))
    assert np.array_equal(y3.cpu().numpy(), x * sc[None, :, None] + bi[None, :, None])


def test_maxpool_upsample_softmax_and_blas1_shims(ctx):
    rng = np.random.default_rng(5)
    x = rng.standard_normal((2, 6, 13, 13)).astype(np.float32)
    xd = dev(ctx, x)
    oh = (13 + 1 - 2) // 2 + 1
    out = torch.empty((2, 6, oh, oh), device=ctx.torch_device)
    idx = torch.empty((2, 6, oh, oh), dtype=torch.int64, device=ctx.torch_device)
    check(lib.tbcompat_forwardMaxPool(ctx.handle, 2, 6, oh, oh, ptr(xd), 6, 13, 13, 2, 2, 1, 2, ptr(idx), ptr(out)))
    ry, ri = O.maxpool(x, 2, 2, padding=1, want_index=True)
    assert np.array_equal(out.cpu().numpy(), ry) and np.array_equal(idx.cpu().numpy(), ri)
    up = torch.empty((2, 6, 26, 26), device=ctx.torch_device)
    check(lib.tbcompat_upSample(ctx.handle, 2, 6, 13, 13, ptr(xd), 2, 1, 1.0, ptr(up), 0))
    assert np.array_equal(up.cpu().numpy(), O.upsample(x, 2))
    assert lib.tbcompat_upSample(ctx.handle, 2, 6, 13, 13, ptr(xd), 2, 0, 1.0, ptr(up), 0) == TB_ERR_UNSUPPORTED
    s = rng.standard_normal((4, 30)).astype(np.float32)
    sd = dev(ctx, s)
    so = torch.empty_like(sd)
    check(lib.tbcompat_softmaxBatch(ctx.handle, 10, ptr(sd), 0, 4, 30, 3, 10, 1, 1.0, ptr(so), 0))
    assert logistic_ulps(so.cpu().numpy(), O.softmax(s, groups=3)) <= 2.0
    a, b = rng.standard_normal(100).astype(np.float32), rng.standard_normal(100).astype(np.float32)
    ad, bd, cd = dev(ctx, a), dev(ctx, b), torch.zeros(100, device=ctx.torch_device)
    check(lib.tbcompat_addvv(ctx.handle, 50, ptr(ad), 0, 2, ptr(bd), 1, 2, ptr(cd), 0, 2))
    assert np.array_equal(cd.cpu().numpy()[0::2], a[0::2] + b[1::2])
    check(lib.tbcompat_copy(ctx.handle, 10, ptr(ad), 5, 1, ptr(cd), 1, 2))
    assert np.array_equal(cd.cpu().numpy()[1:20:2], a[5:15])
    check(lib.tbcompat_fill(ctx.handle, 10, ptr(cd), 0, 2.5, 3))
    assert np.all(cd.cpu().numpy()[0:30:3] == 2.5)
    check(lib.tbcompat_fmavss(ctx.handle, 20, ptr(ad), 10, 1.5, -0.25, ptr(cd)))
    assert np.array_equal(cd.cpu().numpy()[10:30], a[10:30] * np.float32(1.5) + np.float32(-0.25))
    host = np.arange(16, dtype=np.float32)
    m = C.c_void_p()
    check(lib.tbcompat_createDeviceBuffer(ctx.handle, 64, C.byref(m)))
    check(lib.tbcompat_writeBuffer(ctx.handle, m, 64, host.ctypes.data))
    back = np.zeros(16, np.float32)
    check(lib.tbcompat_readBuffer(ctx.handle, m, 64, back.ctypes.data))
    check(lib.tbcompat_finish(ctx.handle))
    check(lib.tbcompat_freeDeviceBuffer(ctx.handle, m))
    assert np.array_equal(back, host)
