"""The process-wide NumPy generator (the reference's _random.py:25-46).

Parameter initialisation and random factories draw on the host from this generator in the
reference's order, so ``manual_seed(s)`` followed by building a model gives the same initial
weights as the reference; the values are then uploaded to the device.

Dropout masks are drawn on the device instead: :func:`pcg64_take` hands the kernels the
generator's PCG64 state before the mask's draws and moves the host generator past them, so
the device mask equals the reference's ``keep_mask`` bit for bit and every later draw on the
host sees the same stream as in the reference.
"""

from __future__ import annotations

import contextlib
from collections.abc import Iterator

import numpy as np


class _RngState:
    generator: np.random.Generator = np.random.default_rng()


def manual_seed(seed: int) -> None:
    """Re-seed the global generator used for initialisation and random factories."""
    _RngState.generator = np.random.default_rng(seed)


def get_rng() -> np.random.Generator:
    """Return the global generator."""
    return _RngState.generator


@contextlib.contextmanager
def replaying(generator: np.random.Generator) -> Iterator[None]:
    """Install ``generator`` as the global generator for the block and put the previous one
    back afterwards (the reference's _random.py:35-46). Gradient checkpointing recomputes a
    function inside this with a copy of the generator taken before its forward pass, so the
    device dropout kernels, which take their PCG64 state from the global generator, draw the
    same keep-masks again."""
    previous = _RngState.generator
    _RngState.generator = generator
    try:
        yield
    finally:
        _RngState.generator = previous


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


_M64 = (1 << 64) - 1
_M128 = (1 << 128) - 1
#: PCG64's 128-bit LCG multiplier (NumPy's PCG64: state <- state * M + inc, then the XSL-RR
#: output of the new state; checked against ``random_raw`` in tests/test_cpu_boundary.py).
_PCG_MULT = 0x2360ED051FC65DA44385DF649FCCF645


def _lcg_jump(inc: int, n: int) -> tuple[int, int]:
    """``(a, c)`` with ``state_{k+n} = a state_k + c (mod 2^128)`` (jump by squaring)."""
    acc_a, acc_c, cur_a, cur_c = 1, 0, _PCG_MULT, inc
    while n:
        if n & 1:
            acc_a = acc_a * cur_a & _M128
            acc_c = (acc_c * cur_a + cur_c) & _M128
        cur_c = (cur_a + 1) * cur_c & _M128
        cur_a = cur_a * cur_a & _M128
        n >>= 1
    return acc_a, acc_c


def pcg64_take(rng: np.random.Generator, outputs: int) -> np.ndarray | None:
    """Reserve the next ``outputs`` raw 64-bit draws of ``rng`` for a device kernel.

    Returns ``[state_hi, state_lo, inc_hi, inc_lo]`` (uint64) of the state before them and
    advances ``rng`` past them, exactly as ``rng.bit_generator.random_raw(outputs)`` would
    (the buffered 32-bit half, which ``random_raw`` does not touch, is kept). ``None`` when the
    bit generator is not PCG64 (the caller then draws on the host)."""
    bg = rng.bit_generator
    if type(bg) is not np.random.PCG64:
        return None
    state = bg.state
    s, inc = int(state["state"]["state"]), int(state["state"]["inc"])
    a, c = _lcg_jump(inc, int(outputs))
    state["state"]["state"] = (a * s + c) & _M128
    bg.state = state
    return np.array([s >> 64, s & _M64, inc >> 64, inc & _M64], dtype=np.uint64)


def dropout_threshold(p: float) -> tuple[int, float]:
    """``keep_mask``'s quantisation: threshold ``round(p * 65536)`` and survivor scale."""
    threshold = round(p * 65536)
    if threshold >= 65536:
        return 65536, 0.0
    return threshold, 65536.0 / (65536 - threshold)
