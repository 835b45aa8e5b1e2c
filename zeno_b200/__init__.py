"""zeno_b200: Zeno's batched rigid-body step on NVIDIA B200 (sm_100a).

The physics step runs as one fused CUDA kernel per World.step behind Zeno's C ABI
(``zeno_b200/lib/libzeno.so``, declared in ``include/zeno.h``).  This package is the
Python side of that boundary: ``ZenoWorld`` and ``ZenoEnv``/``make`` keep the reference
package's interface.

There is no fallback without the library: when ``libzeno.so`` has not been built, the
package still imports (so that ``python -m zeno_b200.build`` and the pure-Python
``scenes`` module work), but every name that needs the library raises the ImportError
that says so.
"""
_LIB_NAMES = ("CONTACT_DTYPE", "CudaArray", "ZenoWorld", "ZeroCopyArray", "is_cuda_available", "is_metal_available",
              "version", "ZenoEnv", "make")

try:
    from ._ffi import (CONTACT_DTYPE, CudaArray, ZenoWorld, ZeroCopyArray, is_cuda_available, is_metal_available,
                       version)
    from .env import ZenoEnv, make
except ImportError as _e:
    if "libzeno.so not found" not in str(_e):
        raise
    _missing = _e

    def __getattr__(name):
        if name in _LIB_NAMES:
            raise ImportError(str(_missing)) from _missing
        raise AttributeError(f"module 'zeno_b200' has no attribute {name!r}")

__version__ = "0.1.0"
__all__ = list(_LIB_NAMES)
