"""VectorCore's B200-native CUDA device.

The product is the sm_100a library behind include/vc_cuda.h; this package
builds it (``vectorcore_b200.build``), binds it (``_abi``), mirrors the
reference's device-plugin interface on top (``backend.CudaBackend``) and
exposes the reference's Python API for the cuda device (``Tensor``,
``cross_entropy``, ``softmax``, ``Linear``, ``sgd_step``, ``synchronize``...).
Importing fails if the library is missing: there is no CPU fallback.
"""
from . import _abi
from ._abi import available as cuda_available  # noqa: F401
from ._abi import device_name as cuda_device_name  # noqa: F401
from .nn import Linear, mse_loss, sgd_step, zero_grad  # noqa: F401
from .tensor import (NoGradGuard, Tensor, argmax_int64, bias_relu_sum, cross_entropy, grad_enabled,  # noqa: F401
                     log_softmax, no_grad, softmax)


def synchronize() -> None:
    """Wait for all queued device work and surface asynchronous errors
    (vectorcore::synchronize, include/vectorcore/metal_backend.hpp:60-63).
    Reading values (item(), numpy(), to('cpu')) synchronises by itself."""
    if _abi.available():
        _abi.synchronize()
