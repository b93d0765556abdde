import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs the CUDA kernels through the C ABI)")


# ---- parity metrics -------------------------------------------------------------------------
# FP32 path (TB_MATH_FP32): the conv kernels keep the reference's summation order (one FMA per k,
# k ascending in im2col row order, no split of K), the connected layer its sdot_avx2 lane order,
# and every epilogue the reference's separate roundings, so results are compared BIT FOR BIT.
# The elementwise metric the parity target is stated in,
#     max_i |a_i - b_i| / max(|b_i|, 1e-3 * rms(map))  <= 1e-4  per activation map,
# is reported beside it (it is 0 when the results are identical).
# Paths that reorder the summation (TB_MATH_FP32_TILED, split-K; TF32) cannot meet that
# elementwise bound at the 1e-3*rms floor: two fp32 orders of a K = 4608 dot product already
# differ by ~1e-3 of the floor-level elements.  They are held to the infinity-norm form
# max|a-b| / max|b| <= 1e-4 (FP32_TILED) or relative L2 (TF32), as their tests state.

FP32_TOL = 1e-4     # elementwise bound of the FP32 parity target, per activation map
RMS_FLOOR = 1e-3    # denominator floor of the elementwise metric, as a fraction of the map's rms


def elem_rel_err(a, b):
    """max_i |a_i - b_i| / max(|b_i|, RMS_FLOOR * rms(b)) over one activation map."""
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    if b.size == 0:
        return 0.0
    assert np.all(np.isfinite(a)), "non-finite values in the result"
    rms = float(np.sqrt(np.mean(b * b)))
    den = np.maximum(np.abs(b), RMS_FLOOR * rms)
    d = np.abs(a - b)
    if rms == 0.0:
        return float(d.max())
    return float(np.max(d / den))


def worst_elem_err(a, b, maps):
    """Worst elem_rel_err over `maps` equal slices (activation maps) of a and b."""
    a = np.asarray(a).reshape(maps, -1)
    b = np.asarray(b).reshape(maps, -1)
    return max(elem_rel_err(a[i], b[i]) for i in range(maps))


def assert_bit_exact(got, ref, maps, what=""):
    """FP32-path parity: identical values (signed zeros compare equal), and the elementwise
    metric reported; returns it (0.0)."""
    got = np.asarray(got)
    ref = np.asarray(ref)
    assert got.shape == ref.shape, (what, got.shape, ref.shape)
    if not np.array_equal(got, ref):
        d = np.abs(got.astype(np.float64) - ref.astype(np.float64))
        i = int(np.argmax(d))
        raise AssertionError(f"{what}: not bit-exact: {int((d > 0).sum())} of {d.size} values differ, "
                             f"worst at {i}: {got.ravel()[i]!r} vs {ref.ravel()[i]!r}; "
                             f"elementwise metric {worst_elem_err(got, ref, maps):.3g}")
    return worst_elem_err(got, ref, maps)


def max_rel_err(a, b):
    """Infinity-norm relative error of one map, max|a-b| / max|b|: the bound used for the paths
    that reorder the summation (TB_MATH_FP32_TILED), see above."""
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    if b.size == 0:
        return 0.0
    assert np.all(np.isfinite(a)), "non-finite values in the result"
    scale = float(np.max(np.abs(b)))
    diff = float(np.max(np.abs(a - b)))
    return diff if scale == 0.0 else diff / scale


def worst_map_err(a, b, maps):
    """Worst max_rel_err over `maps` equal slices (the reordered paths' bound)."""
    a = np.asarray(a).reshape(maps, -1)
    b = np.asarray(b).reshape(maps, -1)
    return max(max_rel_err(a[i], b[i]) for i in range(maps))


def logistic_ulps(got, ref):
    """Largest difference in units of the last place (of ref) between two float32 arrays: used for
    the logistic outputs, whose double-precision exp is the libm's on the CPU and CUDA's on the GPU
    (both faithful; the single-precision result almost always agrees)."""
    got = np.asarray(got, np.float32)
    ref = np.asarray(ref, np.float32)
    ulp = np.spacing(np.abs(ref)).astype(np.float64)
    return float(np.max(np.abs(got.astype(np.float64) - ref.astype(np.float64)) / ulp)) if ref.size else 0.0


def assert_yolo_parity(got, ref, n, classes, what=""):
    """YOLO layer output (TYoloLayer.forward): entries 2, 3 (w, h) are the conv's values and must
    be identical; the logistic entries agree within 1 ulp."""
    B = got.shape[0]
    g = np.asarray(got).reshape(B, n, classes + 5, -1)
    r = np.asarray(ref).reshape(B, n, classes + 5, -1)
    assert np.array_equal(g[:, :, 2:4], r[:, :, 2:4]), (what, "w/h entries differ")
    lg = np.concatenate([g[:, :, 0:2], g[:, :, 4:]], axis=2)
    lr = np.concatenate([r[:, :, 0:2], r[:, :, 4:]], axis=2)
    u = logistic_ulps(lg, lr)
    assert u <= 1.0, (what, "logistic entries", u)
    return u


def yolo_err(got, ref, raw_ref, n, classes, tol):
    """Reordered paths only: worst error of a yolo output relative to what tolerance `tol` on the
    raw conv map allows (w, h: tol * max|raw|; logistic entries: slope <= 1/4)."""
    B = got.shape[0]
    g = got.reshape(B, n, classes + 5, -1).astype(np.float64)
    r = ref.reshape(B, n, classes + 5, -1).astype(np.float64)
    x = raw_ref.reshape(B, n, classes + 5, -1).astype(np.float64)
    worst = 0.0
    for b in range(B):
        for a in range(n):
            for e in range(classes + 5):
                d = np.max(np.abs(g[b, a, e] - r[b, a, e]))
                scale = np.max(np.abs(x[b, a, e]))
                allow = tol * scale if e in (2, 3) else tol * scale / 4 + 2 ** -23
                worst = max(worst, d / max(allow, 1e-30))
    return worst


@pytest.fixture(scope="session")
def ctx():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    from tensorium_b200 import Context
    c = Context(0)
    yield c
    torch.cuda.synchronize()
    c.close()
