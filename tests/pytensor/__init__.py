"""Test helper: the reference's Python Tensor API over the CUDA device's C ABI
(tensor.py, nn.py). Product code never imports it."""
from vectorcore_b200 import cuda_available, cuda_device_name, synchronize  # noqa: F401

from .nn import Linear, mse_loss, sgd_step, zero_grad  # noqa: F401
from .tensor import (NoGradGuard, Tensor, argmax_int64, bias_relu_sum, cross_entropy, grad_enabled,  # noqa: F401
                     log_softmax, no_grad, softmax)
