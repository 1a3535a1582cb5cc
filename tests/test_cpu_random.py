"""The dropout keep-mask stream, checked on the CPU against the reference's own outputs.

``tests/golden/dropout_masks.npz`` holds the reference's ``keep_mask`` for seeded generators
and the draws that follow it. The oracle restatement must reproduce both; so must the device
path's host half (``pcg64_take`` hands the kernels a PCG64 state and moves the generator past
the mask) together with a pure-Python restatement of the kernels' arithmetic (the 128-bit LCG
jump, the XSL-RR output, 16-bit words in little-endian order).
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import ops as O
from tests.conftest import load_golden
from tests.golden.specs import DROPOUT_CASES

M64, M128 = (1 << 64) - 1, (1 << 128) - 1
MULT = 0x2360ED051FC65DA44385DF649FCCF645


def _outputs_from(state: np.ndarray, count: int) -> np.ndarray:
    """The kernels' arithmetic in Python: output w = XSL-RR of the state after w + 1 steps."""
    s = (int(state[0]) << 64) | int(state[1])
    inc = (int(state[2]) << 64) | int(state[3])
    out = []
    for _ in range(count):
        s = (s * MULT + inc) & M128
        hi, lo = s >> 64, s & M64
        v, r = hi ^ lo, hi >> 58
        out.append(((v >> r) | (v << ((64 - r) & 63))) & M64)
    return np.array(out, dtype=np.uint64)


def _generator(seed: int) -> np.random.Generator:
    rng = np.random.default_rng(seed)
    rng.integers(0, 2**32, size=3, dtype=np.uint32)  # as the fixture: a buffered 32-bit half
    return rng


@pytest.mark.parametrize("case", range(len(DROPOUT_CASES)))
def test_oracle_keep_mask_matches_reference(case):
    gold = load_golden("dropout_masks.npz")
    shape, p, seed = DROPOUT_CASES[case]
    rng = _generator(seed)
    keep, scale = O.keep_mask(shape, p, rng)
    np.testing.assert_array_equal(keep, gold[f"case{case}/keep"])
    assert scale == float(gold[f"case{case}/scale"])
    np.testing.assert_array_equal(rng.integers(0, 2**32, size=3, dtype=np.uint32),
                                  gold[f"case{case}/next_u32"])
    np.testing.assert_array_equal(rng.bit_generator.random_raw(2), gold[f"case{case}/next_raw"])


@pytest.mark.parametrize("case", range(len(DROPOUT_CASES)))
def test_device_stream_hand_off_matches_reference(case):
    from tensorgrad_b200._random import dropout_threshold, pcg64_take

    gold = load_golden("dropout_masks.npz")
    shape, p, seed = DROPOUT_CASES[case]
    n = int(np.prod(shape))
    threshold, scale = dropout_threshold(p)
    rng = _generator(seed)
    if threshold >= 65536:
        keep = np.zeros(shape, dtype=np.bool_)  # nothing is drawn
    else:
        state = pcg64_take(rng, (n + 3) // 4)
        words = _outputs_from(state, (n + 3) // 4).view(np.uint16)[:n]
        keep = (words >= threshold).reshape(shape)
    np.testing.assert_array_equal(keep, gold[f"case{case}/keep"])
    assert scale == float(gold[f"case{case}/scale"])
    # The host generator continues exactly where the reference's does.
    np.testing.assert_array_equal(rng.integers(0, 2**32, size=3, dtype=np.uint32),
                                  gold[f"case{case}/next_u32"])
    np.testing.assert_array_equal(rng.bit_generator.random_raw(2), gold[f"case{case}/next_raw"])


def test_pcg64_take_is_random_raw():
    from tensorgrad_b200._random import pcg64_take

    a, b = np.random.default_rng(99), np.random.default_rng(99)
    state = pcg64_take(a, 1000)
    np.testing.assert_array_equal(_outputs_from(state, 1000), b.bit_generator.random_raw(1000))
    assert a.bit_generator.state == b.bit_generator.state
    assert pcg64_take(np.random.Generator(np.random.MT19937(0)), 4) is None


def test_replaying_repeats_the_draws_and_restores_the_generator():
    """Gradient checkpointing's recomputation: a copy of the generator taken before a forward
    pass, installed with ``replaying``, hands the dropout kernels the same PCG64 states; the
    outer generator comes back afterwards, also when the block raises."""
    import copy

    from tensorgrad_b200 import _random as R

    R.manual_seed(5)
    R.get_rng().standard_normal(3)
    snapshot = copy.deepcopy(R.get_rng())
    first = [R.pcg64_take(R.get_rng(), n) for n in (10, 3)]
    outer = R.get_rng()
    after = copy.deepcopy(outer.bit_generator.state)
    with R.replaying(copy.deepcopy(snapshot)):
        assert R.get_rng() is not outer
        again = [R.pcg64_take(R.get_rng(), n) for n in (10, 3)]
    assert R.get_rng() is outer
    assert outer.bit_generator.state == after
    for a, b in zip(first, again, strict=True):
        np.testing.assert_array_equal(a, b)
    with pytest.raises(KeyError), R.replaying(copy.deepcopy(snapshot)):
        raise KeyError("inside")
    assert R.get_rng() is outer
