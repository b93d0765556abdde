"""Known answers for the oracle's restatement of the reference's image path (TImageData:
loadFromFile's byte scale, the two-pass bilinear resize, letterBoxEx), derived by hand."""
from fractions import Fraction

import numpy as np

from oracle import oracle as O


def test_byte_scales():
    """FPC build: v * 257 / $ff00 (white is 65535/65280 = 1.00390625, exact); Delphi: v / 255.
    Both correctly rounded from the exact quotient."""
    v = np.arange(256, dtype=np.uint8).reshape(16, 16)
    fpc = O.image_from_bytes(v)[0].ravel()
    d = O.image_from_bytes(v, pixel_scale=1)[0].ravel()
    assert fpc[255] == np.float32(1.00390625) and d[255] == 1.0 and fpc[0] == 0.0
    for k in range(256):
        for got, q in ((fpc[k], Fraction(257 * k, 65280)), (d[k], Fraction(k, 255))):
            # correctly rounded: no float32 lies strictly closer to q
            f = Fraction(float(got))
            for nb in (np.nextafter(got, np.float32(2)), np.nextafter(got, np.float32(-1))):
                assert abs(Fraction(float(nb)) - q) >= abs(f - q)


def test_channel_orders():
    img = np.zeros((2, 3, 4), np.uint8)
    img[..., 0], img[..., 1], img[..., 2], img[..., 3] = 10, 20, 30, 40
    rgb = O.image_from_bytes(img, pixel_scale=1)
    bgr = O.image_from_bytes(img, bgr=True, pixel_scale=1)
    assert np.allclose(rgb[:, 0, 0] * 255, [10, 20, 30]) and np.allclose(bgr[:, 0, 0] * 255, [30, 20, 10])
    gray = O.image_from_bytes(np.full((2, 2), 51, np.uint8), pixel_scale=1)
    assert np.all(gray == np.float32(0.2))


def test_resize_identity_constant_and_linear():
    rng = np.random.default_rng(1)
    x = rng.uniform(0, 1, (3, 5, 7)).astype(np.float32)
    assert np.array_equal(O.resize(x, 7, 5), x)                      # scale 1: exact copy
    c = np.full((3, 6, 9), 0.25, np.float32)
    assert np.all(O.resize(c, 17, 4) == np.float32(0.25))             # (1-d)*a + d*a for a = 2^-2
    # a horizontal ramp 0, 1, 2 upsampled to 5 columns: w_scale = 0.5 -> 0, 0.5, 1, 1.5, 2
    ramp = np.tile(np.arange(3, dtype=np.float32), (1, 2, 1))
    assert np.array_equal(O.resize(ramp, 5, 2)[0, 0], np.float32([0, 0.5, 1, 1.5, 2]))


def test_resize_last_row_keeps_only_one_term():
    """The second pass adds dy * part[iy + 1] on every row but the last.  4 rows -> 38: h_scale =
    fl(3/37) and the last row's sy = 37 * h_scale rounds to 2.9999998, so that row is
    (1 - dy) * part[2] with dy ~ 1 -- nearly 0, not the source's last row (30).  The quirk is
    the reference's and is kept."""
    x = np.array([[[0.0], [10.0], [20.0], [30.0]]], np.float32)  # [1][4][1]
    y = O.resize(x, 2, 38)
    hs = np.float32(3.0 / 37.0)
    sy = np.float32(37) * hs
    assert sy == np.float32(2.9999998) and int(sy) == 2
    dy = sy - np.float32(2)
    assert y[0, 37, 0] == (np.float32(1) - dy) * np.float32(20.0)
    assert 0 < y[0, 37, 0] < 1e-4
    # a row where sy lands on an integer takes part[iy] alone with weight 1
    assert y[0, 0, 0] == 0.0


def test_letterbox_placement():
    """640x480 into 416x416: width-limited, new 416x312, dx 0, dy 52, ratio 0.65; the border
    rows are 0.5 and the embedded rows are the resized image."""
    rng = np.random.default_rng(2)
    x = rng.uniform(0, 1, (3, 480, 640)).astype(np.float32)
    y, ratio, (nw, nh, dx, dy) = O.letterbox(x, 416, 416)
    assert (nw, nh, dx, dy) == (416, 312, 0, 52) and ratio == np.float32(0.65)
    assert np.all(y[:, :52] == 0.5) and np.all(y[:, 52 + 312:] == 0.5)
    assert np.array_equal(y[:, 52:52 + 312], O.resize(x, 416, 312))
    # height-limited: 300 x 600 (w x h) -> 208 x 416 centred with dx 104
    y, ratio, meta = O.letterbox(rng.uniform(0, 1, (3, 600, 300)).astype(np.float32), 416, 416)
    assert meta == (208, 416, 104, 0) and ratio == np.float32(416 / 600)
