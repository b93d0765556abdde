import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs the CUDA kernels through the C ABI)")


def max_rel_err(a, b):
    """Relative error of one activation map: max_i |a_i - b_i| / max_i |b_i| (the map's
    infinity-norm relative error).  An elementwise ratio is not used: a sum that cancels to
    near zero differs in its last bits under any change of summation order, so its elementwise
    ratio measures only the cancellation, not the kernel."""
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    if b.size == 0:
        return 0.0
    assert np.all(np.isfinite(a)), "non-finite values in the result"
    scale = float(np.max(np.abs(b)))
    diff = float(np.max(np.abs(a - b)))
    if scale == 0.0:
        return diff
    return diff / scale


def worst_map_err(a, b, maps):
    """Worst max_rel_err over `maps` equal slices (activation maps) of a and b."""
    a = np.asarray(a).reshape(maps, -1)
    b = np.asarray(b).reshape(maps, -1)
    return max(max_rel_err(a[i], b[i]) for i in range(maps))


def yolo_err(got, ref, raw_ref, n, classes, tol=None):
    """Worst error of a yolo output relative to what the FP32 tolerance allows.  Entries 2,3
    (w, h) are raw conv values: per-map relative error / FP32_TOL.  The other entries are
    logistic(x): |d logistic| <= |dx|/4, so the allowed error of a map is
    FP32_TOL * max|raw map| / 4 (plus one ulp of 1).  Returns a ratio; <= 1 passes."""
    tol = FP32_TOL if tol is None else tol
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


FP32_TOL = 1e-4  # max relative error per activation map, FP32 path
# A whole network run free (each layer fed its own previous output) accumulates the FP32
# reordering differences of every layer before it; with random He-init weights the YOLOv3
# activations grow to ~1e5 through 23 residual adds.  End-to-end outputs are held to this bound.
E2E_TOL = 1e-3


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
