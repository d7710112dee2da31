"""VectorCore's B200-native CUDA device.

The product is the sm_100a library behind include/vc_cuda.h; this package
builds it (``vectorcore_b200.build``), binds it (``_abi``) and mirrors the
reference's device-plugin interface on top (``backend.CudaBackend``).
"""
from ._abi import available as cuda_available  # noqa: F401  (fails loudly if the library is missing)
from ._abi import device_name as cuda_device_name  # noqa: F401
from ._abi import synchronize  # noqa: F401
