"""VectorCore's B200-native CUDA device.

The product is the sm_100a library behind include/vc_cuda.h; this package
builds it (``vectorcore_b200.build``), binds it (``_abi``) and mirrors the
reference's device-plugin interface on top (``backend.CudaBackend``, the
Python twin of csrc/host/cuda_backend.hpp). The reference's own Tensor API
reaches the device through its host with the `cuda` device added
(csrc/host/reference_cuda_device.patch). Importing fails if the library is
missing: there is no CPU fallback.
"""
from . import _abi
from ._abi import available as cuda_available  # noqa: F401
from ._abi import device_name as cuda_device_name  # noqa: F401


def synchronize() -> None:
    """Wait for all queued device work and surface asynchronous errors
    (vectorcore::synchronize, include/vectorcore/metal_backend.hpp:60-63).
    Reading values (item(), numpy(), to('cpu')) synchronises by itself."""
    if _abi.available():
        _abi.synchronize()
