"""zeno_b200: Zeno's batched rigid-body step on NVIDIA B200 (sm_100a).

The physics step runs as one fused CUDA kernel per World.step behind Zeno's C ABI
(``zeno_b200/lib/libzeno.so``, declared in ``include/zeno.h``).  This package is the
Python side of that boundary: ``ZenoWorld`` and ``ZenoEnv``/``make`` keep the reference
package's interface.
"""
from ._ffi import (CONTACT_DTYPE, CudaArray, ZenoWorld, ZeroCopyArray, is_cuda_available, is_metal_available,
                   version)
from .env import ZenoEnv, make

__version__ = "0.1.0"
__all__ = ["ZenoWorld", "ZenoEnv", "make", "ZeroCopyArray", "CudaArray", "CONTACT_DTYPE", "version",
           "is_metal_available", "is_cuda_available"]
