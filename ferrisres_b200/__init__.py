"""ferrisres_b200: B200-native (sm_100a) ternary matmul hot path of FerrisRes.

The compute lives in ``libferris_ternary.so`` (CUDA C++, built in-tree by
``python -m ferrisres_b200.build``) behind the C ABI of
``include/ferris_ternary.h``.  ``ferrisres_b200.gpu`` mirrors the reference's
GPU op / accelerator API on top of that ABI; ``ferrisres_b200.ternary``
mirrors the reference's host-side packing.
"""
from ._lib import (CommTimeoutError, DeviceError, FerrisResError, GpuError, OOMError, ShapeError,
                   UnsupportedError)

__all__ = ["FerrisResError", "ShapeError", "GpuError", "OOMError", "UnsupportedError",
           "CommTimeoutError", "DeviceError"]
__version__ = "0.1.0"
