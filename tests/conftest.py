import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs the CUDA kernels through the C ABI)")


def max_rel_err(a, b, floor_frac=1e-3):
    """max |a-b| / max(|b|, floor_frac * rms(b)) over one activation map.  The floor (0.1% of the
    map's rms) keeps entries of the reference that are near zero by cancellation from
    dominating; this is the tolerance definition used by every FP32 parity test."""
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    if b.size == 0:
        return 0.0
    assert np.all(np.isfinite(a)), "non-finite values in the result"
    rms = float(np.sqrt(np.mean(b * b)))
    den = np.maximum(np.abs(b), floor_frac * rms + 1e-30)
    return float(np.max(np.abs(a - b) / den))


def worst_map_err(a, b, maps):
    """Worst max_rel_err over `maps` equal slices (activation maps) of a and b."""
    a = np.asarray(a).reshape(maps, -1)
    b = np.asarray(b).reshape(maps, -1)
    return max(max_rel_err(a[i], b[i]) for i in range(maps))


FP32_TOL = 1e-4  # max relative error per activation map, FP32 path


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
