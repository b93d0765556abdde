"""tensorium_b200 -- B200 (sm_100a) backend for Tensorium's darknet-style conv inference path.

The compute lives in the C-ABI library ``libtensorium_b200.so`` (include/tensorium_b200.h);
this package is the host-side mirror of the reference's layer / network API over it.
"""
from ._lib import ACT, MATH_FP32, MATH_TF32, TBError, lib  # noqa: F401
from .context import Context, device_count, ptr  # noqa: F401
