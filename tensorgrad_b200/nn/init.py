"""In-place parameter initialisers (the reference's nn/init.py:16-59).

Values are drawn on the host from the global generator in the reference's order and
uploaded, so a seeded model starts from the same weights as the reference's.
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
    if t.ndim < 2:
        raise ValueError("fans are defined for tensors with at least 2 dimensions")
    receptive = math.prod(t.shape[2:])
    return t.shape[1] * receptive, t.shape[0] * receptive


def uniform_(t: T, low: float = 0.0, high: float = 1.0) -> T:
    t.data[...] = get_rng().uniform(low, high, size=t.shape)
    return t


def normal_(t: T, mean: float = 0.0, std: float = 1.0) -> T:
    t.data[...] = get_rng().normal(mean, std, size=t.shape)
    return t


def zeros_(t: T) -> T:
    t.data.fill_(0.0)
    return t


def ones_(t: T) -> T:
    t.data.fill_(1.0)
    return t


def xavier_uniform_(t: T, gain: float = 1.0) -> T:
    fan_in, fan_out = calculate_fans(t)
    bound = gain * math.sqrt(6.0 / (fan_in + fan_out))
    return uniform_(t, -bound, bound)


def kaiming_uniform_(t: T, nonlinearity_gain: float = math.sqrt(2.0)) -> T:
    fan_in, _ = calculate_fans(t)
    bound = nonlinearity_gain * math.sqrt(3.0 / fan_in)
    return uniform_(t, -bound, bound)

