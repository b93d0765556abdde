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
