"""Seeds and shapes of the golden fixtures, shared by ``make_golden.py`` and the tests."""

from __future__ import annotations

import numpy as np

from oracle import gpt as ogpt

#: Small GPT used for the committed fixture (all code paths of the char-GPT config). Its
#: ``max_norm`` sits below the gradient norm so that clipping is exercised.
GPT_SMALL = dict(cfg=ogpt.Config(vocab_size=65, block_size=16, n_layer=2, n_head=2, n_embd=16),
                 batch=4, seq=16, seed=0, max_norm=0.5, steps=2)
#: ((B, H, T, d), causal, seed) of the attention fixtures.
ATTN_CASES = [((2, 2, 24, 8), True, 1), ((1, 3, 17, 16), False, 2), ((2, 1, 33, 32), True, 3)]


def attention_inputs(shape: tuple[int, int, int, int], seed: int) -> list[np.ndarray]:
    """``q, k, v, dO`` ~ N(0, 1) from ``seed`` (the MHA-alone config's distribution)."""
    rng = np.random.default_rng(seed)
    return [rng.standard_normal(shape) for _ in range(4)]
