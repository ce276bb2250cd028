"""raon_npu_b200 -- B200-native (sm_100a) ``cuda`` backend for raon-npu's
q4nx GEMV and MoE hot path.

The compute lives in ``libraon_cuda.so`` (hand-written CUDA behind the C ABI
of ``include/raon_cuda.h``); this package is the Python host side that mirrors
the reference's ``Backend`` interface.  There is no CPU fallback: using the
backend without the built library raises ``RaonCudaError``.
"""

from ._lib import RaonCudaError, DeviceTimeout, load  # noqa: F401

__all__ = ["RaonCudaError", "DeviceTimeout", "load", "CudaBackend", "Context", "Q4nxWeight"]


def __getattr__(name):
    if name == "CudaBackend":
        from .backend import CudaBackend
        return CudaBackend
    if name in ("Context", "Q4nxWeight"):
        from . import device
        return getattr(device, name)
    raise AttributeError(name)
