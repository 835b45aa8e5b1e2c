"""zeno_b200: Zeno's batched rigid-body step on NVIDIA B200 (sm_100a).

The physics step runs as one fused CUDA kernel per World.step behind Zeno's C ABI
(``zeno_b200/lib/libzeno.so``, declared in ``include/zeno.h``).  This package is the
Python side of that boundary: ``ZenoWorld`` and ``ZenoEnv``/``make`` keep the reference
package's interface.

The library is loaded on first use of a name that needs it (``ZenoWorld``,
``is_cuda_available``, ...), not at import, so that the pure-Python modules (``scenes``,
``initial_state``, ``build``) import without touching it.  There is no fallback: when
``libzeno.so`` is missing or cannot be loaded, that first use raises the ImportError that
says so.
"""
import importlib

_FFI_NAMES = ("CONTACT_DTYPE", "CudaArray", "ZenoWorld", "ZeroCopyArray", "is_cuda_available", "is_metal_available",
              "version")
_ENV_NAMES = ("ZenoEnv", "make")


def __getattr__(name):
    if name in _FFI_NAMES:
        return getattr(importlib.import_module("._ffi", __name__), name)
    if name in _ENV_NAMES:
        return getattr(importlib.import_module(".env", __name__), name)
    raise AttributeError(f"module 'zeno_b200' has no attribute {name!r}")


__version__ = "0.1.0"
__all__ = list(_FFI_NAMES + _ENV_NAMES)
