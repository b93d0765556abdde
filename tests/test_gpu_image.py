"""GPU input pipeline (tb_images_to_tensor) against the oracle's restatement of TImageData
(loadFromFile's byte scale, resize, letterBoxEx): bit-exact, every image and pixel."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from tensorium_b200.image import PIXEL_255, PIXEL_FPC, ImagePipeline

pytestmark = pytest.mark.gpu


def oracle_batch(images, ow, oh, letterbox, bgr=False, scale=PIXEL_FPC):
    out, ratios, place = [], [], []
    for im in images:
        x = O.image_from_bytes(im, bgr=bgr, pixel_scale=scale)
        if letterbox:
            y, r, m = O.letterbox(x, ow, oh)
            ratios.append(r)
            place.append(m)
        else:
            y = O.resize(x, ow, oh)
        out.append(y)
    return np.stack(out), ratios, place


SHAPES = [  # (h, w, bytes per pixel)
    (480, 640, 3),     # VGA, width-limited letterbox
    (1080, 1920, 3),   # full HD downscale
    (600, 300, 4),     # RGBA, height-limited
    (37, 53, 1),       # gray, upscale
    (416, 416, 3),     # already network size: exact copy
    (4, 38, 3),        # tiny: the last-row quirk of the row pass
]


@pytest.mark.parametrize("direct", [False, True])
@pytest.mark.parametrize("letterbox", [False, True])
@pytest.mark.parametrize("scale", [PIXEL_FPC, PIXEL_255])
def test_batch_matches_oracle(ctx, letterbox, scale, direct, monkeypatch):
    """Both kernel forms: rows staged in shared memory (default) and direct gathers
    (TB_IMAGES_DIRECT=1, also what rows too wide for shared memory take)."""
    monkeypatch.setenv("TB_IMAGES_DIRECT", "1" if direct else "0")
    rng = np.random.default_rng(7 + letterbox + 2 * scale)
    images = [rng.integers(0, 256, (h, w, c) if c > 1 else (h, w), dtype=np.uint8) for h, w, c in SHAPES]
    pipe = ImagePipeline(ctx, scale)
    out, ratios, place = pipe.to_tensor(images, 416, 416, letterbox)
    ref, rr, rp = oracle_batch(images, 416, 416, letterbox, scale=scale)
    got = out.cpu().numpy()
    for i in range(len(images)):
        assert np.array_equal(got[i], ref[i]), (i, SHAPES[i], np.abs(got[i] - ref[i]).max())
    if letterbox:
        assert np.array_equal(ratios, np.float32(rr))
        assert [tuple(p) for p in place] == rp


def test_odd_sizes_bgr_strided_output(ctx):
    """Non-square, odd output sizes, BGR bytes, images written into a slice of a larger input
    buffer (batch stride > image size), and more images than one launch takes (64)."""
    rng = np.random.default_rng(11)
    images = [rng.integers(0, 256, (int(rng.integers(8, 90)), int(rng.integers(8, 90)), 3), dtype=np.uint8)
              for _ in range(70)]
    images += [rng.integers(0, 256, (47, 87, 3), dtype=np.uint8), rng.integers(0, 256, (8, 95, 3), dtype=np.uint8)]
    big = torch.full((72, 4, 29, 31), -1.0, device=ctx.torch_device)
    out = big[:, :3]
    pipe = ImagePipeline(ctx)
    for letterbox in (False, True):
        pipe.to_tensor(images, 31, 29, letterbox, out=out, bgr=True)
        ref, _, _ = oracle_batch(images, 31, 29, letterbox, bgr=True)
        assert np.array_equal(out.cpu().numpy(), ref)
        assert torch.all(big[:, 3] == -1.0)  # nothing outside the slices


def test_device_images_with_row_stride(ctx):
    """Images described in place inside a wider device frame: row stride > width * bpp and rows
    starting at odd byte addresses (the staged kernel's partial first and last words)."""
    from tensorium_b200._lib import Image
    rng = np.random.default_rng(13)
    frame = rng.integers(0, 256, (64, 101, 4), dtype=np.uint8)
    dframe = torch.from_numpy(frame).to(ctx.torch_device)
    cuts = [(3, 50, 1, 88), (1, 9, 5, 100), (0, 64, 0, 100), (10, 12, 7, 30)]
    # +1: each 4-byte pixel read from its second byte, so channels 0..2 are the frame's 1..3 (the
    # fourth byte, taken as alpha, is the next pixel's first and is ignored)
    descs = [Image(dframe.data_ptr() + (y0 * 101 + x0) * 4 + 1, x1 - x0, y1 - y0, 101 * 4, 4, 0)
             for y0, y1, x0, x1 in cuts]
    pipe = ImagePipeline(ctx)
    for letterbox in (False, True):
        out, _, _ = pipe.to_tensor(descs, 45, 37, letterbox)
        imgs = [frame[y0:y1, x0:x1, 1:4] for y0, y1, x0, x1 in cuts]
        ref, _, _ = oracle_batch(imgs, 45, 37, letterbox)
        assert np.array_equal(out.cpu().numpy(), ref)


def test_net_predict_images_matches_float_input(ctx):
    """TNNet.predict_images (bytes -> GPU letterbox -> forward) equals predict on the oracle's
    letterboxed floats."""
    from tensorium_b200 import synth
    from tensorium_b200.net import TNNet
    specs = synth.cifar_specs()
    rng = np.random.default_rng(3)
    images = [rng.integers(0, 256, (int(rng.integers(20, 80)), int(rng.integers(20, 80)), 3), dtype=np.uint8)
              for _ in range(4)]
    net = TNNet(ctx, specs, 4, (3, 32, 32))
    got, ratios, place = net.predict_images(images, letterbox=True, layers=[9, 11])
    ref_x, _, _ = oracle_batch(images, 32, 32, True)
    want = net.predict(ref_x, layers=[9, 11])
    for g, w in zip(got, want):
        assert np.array_equal(g, w)
    net.close()
