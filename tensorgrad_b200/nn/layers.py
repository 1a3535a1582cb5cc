"""Standard layers on device tensors (API of the reference's nn/layers.py:42-341).

Trainable tensors are created straight from their initial values: each draw is taken on the
host from the global generator, in the order and with the NumPy call the reference's
initialiser makes (so a seeded model starts from the reference's weights), and uploaded once.
Layers without parameters are thin adaptors over a functional op.
"""

from __future__ import annotations

import math
from collections.abc import Callable, Iterator, Sequence
from typing import Any, Literal

import numpy as np

from tensorgrad_b200 import ops
from tensorgrad_b200._random import get_rng
from tensorgrad_b200.nn.module import Module, Parameter
from tensorgrad_b200.tensor import Tensor, get_default_dtype

__all__ = ["GELU", "MLP", "BatchNorm1d", "BatchNorm2d", "Conv2d", "Dropout", "Embedding",
           "Flatten", "Identity", "LayerNorm", "Linear", "MaxPool2d", "ReLU", "Sequential",
           "Sigmoid", "Tanh"]


def _param(values: np.ndarray) -> Parameter:
    return Parameter(np.asarray(values, dtype=get_default_dtype()))


def _uniform(shape: tuple[int, ...], bound: float) -> Parameter:
    """U(-bound, bound) in the default dtype (init.uniform_'s draw)."""
    return _param(get_rng().uniform(-bound, bound, size=shape))


def _constant(shape: tuple[int, ...], value: float) -> Parameter:
    return _param(np.full(shape, value))


class Linear(Module):
    """``y = x W^T + b`` with weight and bias from ``U(-1/sqrt(in), 1/sqrt(in))``."""

    def __init__(self, in_features: int, out_features: int, bias: bool = True) -> None:
        super().__init__()
        self.in_features, self.out_features = in_features, out_features
        bound = 1.0 / math.sqrt(in_features)
        self.weight = _uniform((out_features, in_features), bound)
        self.bias: Parameter | None = _uniform((out_features,), bound) if bias else None

    def forward(self, x: Tensor) -> Tensor:
        return ops.linear(x, self.weight, self.bias)

    def extra_repr(self) -> str:
        return f"{self.in_features}, {self.out_features}, bias={self.bias is not None}"


class Conv2d(Module):
    """Cross-correlation of ``(N, C, H, W)`` inputs with square kernels; weight and bias from
    ``U(-1/sqrt(fan_in), 1/sqrt(fan_in))``, ``fan_in = C k k``."""

    def __init__(self, in_channels: int, out_channels: int, kernel_size: int, stride: int = 1,
                 padding: int = 0, bias: bool = True) -> None:
        super().__init__()
        self.in_channels, self.out_channels = in_channels, out_channels
        self.kernel_size, self.stride, self.padding = kernel_size, stride, padding
        bound = 1.0 / math.sqrt(in_channels * kernel_size * kernel_size)
        self.weight = _uniform((out_channels, in_channels, kernel_size, kernel_size), bound)
        self.bias: Parameter | None = _uniform((out_channels,), bound) if bias else None

    def forward(self, x: Tensor) -> Tensor:
        from tensorgrad_b200.ops.conv import conv2d

        return conv2d(x, self.weight, self.bias, stride=self.stride, padding=self.padding)

    def extra_repr(self) -> str:
        return (f"{self.in_channels}, {self.out_channels}, kernel_size={self.kernel_size}, "
                f"stride={self.stride}, padding={self.padding}")


class MaxPool2d(Module):
    """Window maxima over ``(N, C, H, W)``; the stride defaults to the window."""

    def __init__(self, kernel_size: int, stride: int | None = None, padding: int = 0) -> None:
        super().__init__()
        self.kernel_size, self.stride, self.padding = kernel_size, stride, padding

    def forward(self, x: Tensor) -> Tensor:
        from tensorgrad_b200.ops.conv import max_pool2d

        return max_pool2d(x, self.kernel_size, self.stride, self.padding)

    def extra_repr(self) -> str:
        return f"kernel_size={self.kernel_size}, stride={self.stride or self.kernel_size}"


class Embedding(Module):
    """Rows of a ``(num, dim)`` table from ``N(0, 1)``, gathered by integer ids."""

    def __init__(self, num_embeddings: int, embedding_dim: int) -> None:
        super().__init__()
        self.num_embeddings, self.embedding_dim = num_embeddings, embedding_dim
        self.weight = _param(get_rng().normal(0.0, 1.0, size=(num_embeddings, embedding_dim)))

    def forward(self, indices: Any) -> Tensor:
        return ops.embedding(indices, self.weight)

    def extra_repr(self) -> str:
        return f"{self.num_embeddings}, {self.embedding_dim}"


class LayerNorm(Module):
    """Normalisation over the last axis with an optional affine map (scale 1, shift 0)."""

    def __init__(self, normalized_shape: int, eps: float = 1e-5,
                 elementwise_affine: bool = True) -> None:
        super().__init__()
        self.normalized_shape, self.eps = normalized_shape, eps
        self.weight: Parameter | None = (
            _constant((normalized_shape,), 1.0) if elementwise_affine else None)
        self.bias: Parameter | None = (
            _constant((normalized_shape,), 0.0) if elementwise_affine else None)

    def forward(self, x: Tensor) -> Tensor:
        if x.shape[-1] != self.normalized_shape:
            raise ValueError(f"expected last dimension {self.normalized_shape}, got {x.shape}")
        return ops.layer_norm(x, self.weight, self.bias, self.eps)

    def extra_repr(self) -> str:
        return f"{self.normalized_shape}, eps={self.eps}"


class _BatchNorm(Module):
    """Batch statistics over every axis but the channel axis 1 in training (running mean and
    unbiased variance updated with ``momentum``), running statistics in evaluation."""

    ranks: tuple[int, ...] = ()
    layout = ""

    def __init__(self, num_features: int, eps: float = 1e-5, momentum: float = 0.1,
                 affine: bool = True) -> None:
        super().__init__()
        self.num_features, self.eps, self.momentum = num_features, eps, momentum
        self.weight: Parameter | None = _constant((num_features,), 1.0) if affine else None
        self.bias: Parameter | None = _constant((num_features,), 0.0) if affine else None
        dt = get_default_dtype()
        self.register_buffer("running_mean", np.zeros(num_features, dtype=dt))
        self.register_buffer("running_var", np.ones(num_features, dtype=dt))

    def forward(self, x: Tensor) -> Tensor:
        if x.ndim not in self.ranks or x.shape[1] != self.num_features:
            raise ValueError(f"{type(self).__name__}({self.num_features}) expects {self.layout} "
                             f"input, got {x.shape}")
        return ops.batch_norm(x, self.running_mean, self.running_var, self.weight, self.bias,
                              training=self.training, momentum=self.momentum, eps=self.eps)

    def extra_repr(self) -> str:
        return f"{self.num_features}, eps={self.eps}, momentum={self.momentum}"


class BatchNorm1d(_BatchNorm):
    ranks, layout = (2, 3), "(N, C) or (N, C, L)"


class BatchNorm2d(_BatchNorm):
    ranks, layout = (4,), "(N, C, H, W)"


class Dropout(Module):
    """Inverted dropout with probability ``p`` in training; the identity in evaluation."""

    def __init__(self, p: float = 0.5) -> None:
        super().__init__()
        if not 0.0 <= p <= 1.0:
            raise ValueError(f"dropout probability must be in [0, 1], got {p}")
        self.p = p

    def forward(self, x: Tensor) -> Tensor:
        return ops.dropout(x, self.p, self.training)

    def extra_repr(self) -> str:
        return f"p={self.p}"


class _Pointwise(Module):
    """A parameter-free layer applying one functional op."""

    fn: Callable[[Tensor], Tensor]

    def forward(self, x: Tensor) -> Tensor:
        return type(self).fn(x)


class ReLU(_Pointwise):
    fn = staticmethod(ops.relu)


class GELU(_Pointwise):
    fn = staticmethod(ops.gelu)


class Tanh(_Pointwise):
    fn = staticmethod(ops.tanh)


class Sigmoid(_Pointwise):
    fn = staticmethod(ops.sigmoid)


class Identity(_Pointwise):
    fn = staticmethod(lambda x: x)


class Flatten(Module):
    """Merge every axis from ``start_axis`` on into one."""

    def __init__(self, start_axis: int = 1) -> None:
        super().__init__()
        self.start_axis = start_axis

    def forward(self, x: Tensor) -> Tensor:
        return ops.flatten(x, self.start_axis)


class Sequential(Module):
    """Layers applied in order; registered as children ``"0"``, ``"1"``, ..."""

    def __init__(self, *layers: Module) -> None:
        super().__init__()
        self._length = 0
        for layer in layers:
            self.append(layer)

    def append(self, layer: Module) -> Sequential:
        setattr(self, str(self._length), layer)
        self._length += 1
        return self

    def __len__(self) -> int:
        return self._length

    def __getitem__(self, index: int) -> Module:
        if index < -self._length or index >= self._length:
            raise IndexError(f"index {index} out of range for Sequential of length {len(self)}")
        return getattr(self, str(index % self._length))  # type: ignore[no-any-return]

    def __iter__(self) -> Iterator[Module]:
        return (getattr(self, str(i)) for i in range(self._length))

    def forward(self, x: Tensor) -> Tensor:
        for layer in self:
            x = layer(x)
        return x


_ACTIVATIONS: dict[str, type[Module]] = {"relu": ReLU, "gelu": GELU, "tanh": Tanh}


class MLP(Sequential):
    """``Linear`` layers of the given sizes with an activation after each hidden one (and
    after the last with ``final_activation``), dropout after hidden activations."""

    def __init__(self, sizes: Sequence[int], activation: Literal["relu", "gelu", "tanh"] = "relu",
                 dropout: float = 0.0, final_activation: bool = False) -> None:
        if len(sizes) < 2:
            raise ValueError("an MLP needs at least an input and an output size")
        layers: list[Module] = []
        last = len(sizes) - 2
        for i in range(last + 1):
            layers.append(Linear(sizes[i], sizes[i + 1]))
            hidden = i < last
            if hidden or final_activation:
                layers.append(_ACTIVATIONS[activation]())
            if hidden and dropout > 0:
                layers.append(Dropout(dropout))
        super().__init__(*layers)
