"""Model utilities of the reference (include/vectorcore/nn.hpp, src/nn.cpp) on
the cuda device: Linear, mse_loss, sgd_step, zero_grad. cross_entropy is the
fused kernel in tensor.py."""
from __future__ import annotations

import math

from vectorcore_b200.backend import CudaBackend
from .tensor import NoGradGuard, Tensor, cross_entropy  # noqa: F401


class Linear:
    """y = x @ weight + bias with weight [in, out] ~ N(0, 1) / sqrt(in) and a
    zero bias (src/nn.cpp:14-29)."""

    def __init__(self, in_features: int, out_features: int, seed: int = 0, device: str = "cuda"):
        w = Tensor.randn((in_features, out_features), False, seed, "cpu").numpy() / math.sqrt(in_features)
        self.weight = Tensor(w.astype("float32"), True, device)
        self.bias = Tensor.zeros((out_features,), True, device)

    def __call__(self, x: Tensor) -> Tensor:
        return x.matmul(self.weight) + self.bias

    def parameters(self):
        return [self.weight, self.bias]


def mse_loss(prediction: Tensor, target: Tensor) -> Tensor:
    error = prediction - target
    return (error * error).mean()


def sgd_step(parameters, learning_rate: float) -> None:
    """parameter -= lr * grad in place, as one axpy kernel per parameter,
    bumping the storage version so stale saved tensors are detected
    (src/nn.cpp:55-76)."""
    be = CudaBackend.instance()
    with NoGradGuard():
        for p in parameters:
            if p is None or p.grad is None:
                continue
            g = p.grad
            if g.shape != p.shape or g.device != p.device:
                raise ValueError("parameter gradient shape or device does not match")
            if p.device != "cuda":
                raise RuntimeError("vectorcore_b200.sgd_step updates cuda parameters")
            storage = p._impl.storage
            be.axpy_inplace(storage, g._impl.storage, p.numel, -learning_rate)
            storage.bump_version()


def zero_grad(parameters) -> None:
    for p in parameters:
        if p is not None:
            p.zero_grad()
