"""The process-wide NumPy generator (the reference's _random.py:25-46).

Parameter initialisation and random factories draw on the host from this generator in the
reference's order, so ``manual_seed(s)`` followed by building a model gives the same initial
weights as the reference; the values are then uploaded to the device.
"""

from __future__ import annotations

import numpy as np


class _RngState:
    generator: np.random.Generator = np.random.default_rng()


def manual_seed(seed: int) -> None:
    """Re-seed the global generator used for initialisation and random factories."""
    _RngState.generator = np.random.default_rng(seed)


def get_rng() -> np.random.Generator:
    """Return the global generator."""
    return _RngState.generator


#: Bit generators whose raw words carry 64 uniform bits (four 16-bit uniforms each).
_WIDE = (np.random.PCG64, np.random.PCG64DXSM, np.random.Philox, np.random.SFC64)


def keep_mask(shape: tuple[int, ...], p: float, rng: np.random.Generator) -> tuple[np.ndarray, float]:
    """Dropout keep-mask and inverse keep probability, the reference's scheme (_random.py:53-70):
    the drop probability is quantised to ``t / 65536`` with ``t = round(p * 65536)``; an element
    is kept when its uniform 16-bit word is ``>= t``, and survivors scale by
    ``65536 / (65536 - t)``. Same generator state in, same mask out."""
    threshold = round(p * 65536)
    if threshold >= 65536:
        return np.zeros(shape, dtype=np.bool_), 0.0
    n = int(np.prod(shape)) if shape else 1
    if isinstance(rng.bit_generator, _WIDE):
        words = rng.bit_generator.random_raw((n + 3) // 4).view(np.uint16)[:n]
    else:
        words = np.frombuffer(rng.bytes(2 * n), dtype=np.uint16)
    return (words >= threshold).reshape(shape), 65536.0 / (65536 - threshold)
