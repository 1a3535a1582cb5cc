"""In-place initialisers for device parameters (API of the reference's nn/init.py).

Random values come from the global host generator with the NumPy call the reference's
initialiser makes (``uniform(low, high, size)`` / ``normal(mean, std, size)``), so seeded
initialisation matches the reference draw for draw; they are uploaded into the parameter's
device storage in one copy. Constant fills run on the device.
"""

from __future__ import annotations

import math
from typing import TypeVar

from tensorgrad_b200._random import get_rng
from tensorgrad_b200.tensor import Tensor

T = TypeVar("T", bound=Tensor)

__all__ = ["calculate_fans", "kaiming_uniform_", "normal_", "ones_", "uniform_",
           "xavier_uniform_", "zeros_"]


def calculate_fans(t: Tensor) -> tuple[int, int]:
    """``(fan_in, fan_out)`` of a weight laid out ``(out, in, *kernel)``."""
    if t.ndim < 2:
        raise ValueError("fans are defined for tensors with at least 2 dimensions")
    kernel = math.prod(t.shape[2:])
    return t.shape[1] * kernel, t.shape[0] * kernel


def _fill(t: T, values) -> T:  # noqa: ANN001
    t.data[...] = values
    return t


def uniform_(t: T, low: float = 0.0, high: float = 1.0) -> T:
    return _fill(t, get_rng().uniform(low, high, size=t.shape))


def normal_(t: T, mean: float = 0.0, std: float = 1.0) -> T:
    return _fill(t, get_rng().normal(mean, std, size=t.shape))


def zeros_(t: T) -> T:
    t.data.fill_(0.0)
    return t


def ones_(t: T) -> T:
    t.data.fill_(1.0)
    return t


def xavier_uniform_(t: T, gain: float = 1.0) -> T:
    """``U(-a, a)``, ``a = gain sqrt(6 / (fan_in + fan_out))``."""
    fan_in, fan_out = calculate_fans(t)
    a = gain * math.sqrt(6.0 / (fan_in + fan_out))
    return uniform_(t, -a, a)


def kaiming_uniform_(t: T, nonlinearity_gain: float = math.sqrt(2.0)) -> T:
    """``U(-a, a)``, ``a = gain sqrt(3 / fan_in)``."""
    a = nonlinearity_gain * math.sqrt(3.0 / calculate_fans(t)[0])
    return uniform_(t, -a, a)
