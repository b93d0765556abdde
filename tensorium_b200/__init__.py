"""tensorium_b200 -- B200 (sm_100a) backend for Tensorium's darknet-style conv inference path.

The compute lives in the C-ABI library ``libtensorium_b200.so`` (include/tensorium_b200.h);
this package is the host-side mirror of the reference's layer / network API over it.  The
library is loaded on first use of any of the names below (importing a submodule that needs it
raises ImportError when it has not been built: there is no CPU fallback).
"""
_EXPORTS = {"ACT": "_lib", "MATH_FP32": "_lib", "MATH_TF32": "_lib", "MATH_FP32_TILED": "_lib", "MATH_BF16_SPLIT": "_lib", "TBError": "_lib", "lib": "_lib",
            "Context": "context", "device_count": "context", "ptr": "context"}


def __getattr__(name):
    if name in _EXPORTS:
        import importlib
        mod = importlib.import_module(f".{_EXPORTS[name]}", __name__)
        return getattr(mod, name)
    raise AttributeError(name)
