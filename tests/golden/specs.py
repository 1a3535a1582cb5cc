"""Seeds and shapes of the golden fixtures, shared by ``make_golden.py`` and the tests."""

from __future__ import annotations

import numpy as np

from oracle import cnn as ocnn
from oracle import gpt as ogpt

#: Small GPT used for the committed fixture (all code paths of the char-GPT config). Its
#: ``max_norm`` sits below the gradient norm so that clipping is exercised.
GPT_SMALL = dict(cfg=ogpt.Config(vocab_size=65, block_size=16, n_layer=2, n_head=2, n_embd=16),
                 batch=4, seq=16, seed=0, max_norm=0.5, steps=2)
#: The same GPT trained with dropout 0.1 everywhere the reference applies it (embeddings,
#: attention weights, the attention projection and the MLP output), the global generator
#: re-seeded right after the weights are loaded so the masks start from a known state.
GPT_DROPOUT = dict(GPT_SMALL, dropout=0.1, reseed=4321)
#: (shape, p, seed) of the keep-mask fixtures: odd sizes (a partial last 64-bit draw), a
#: common rate, and a rate that rounds to "drop everything" (no draw at all).
DROPOUT_CASES = [((7, 13), 0.1, 1), ((3, 5, 4), 0.5, 2), ((10,), 0.99999999, 3)]
#: ((B, H, T, d), causal, seed) of the attention fixtures.
ATTN_CASES = [((2, 2, 24, 8), True, 1), ((1, 3, 17, 16), False, 2), ((2, 1, 33, 32), True, 3)]


def attention_inputs(shape: tuple[int, int, int, int], seed: int) -> list[np.ndarray]:
    """``q, k, v, dO`` ~ N(0, 1) from ``seed`` (the MHA-alone config's distribution)."""
    rng = np.random.default_rng(seed)
    return [rng.standard_normal(shape) for _ in range(4)]


#: Small CNN (the CNN config's layer stack at 8x8 inputs) for the committed fixture.
CNN_SMALL = dict(cfg=ocnn.Config(in_channels=3, size=8, c1=4, c2=6, classes=4), batch=4, seed=5,
                 steps=2)

#: Op-level conv / pool cases: (x shape, (c_out, kh, kw), stride, padding, seed) and
#: (x shape, kernel, stride, padding, seed). The pool cases include overlapping windows and
#: -inf padding; ties and a NaN are planted by ``pool_input``.
CONV_CASES = [((2, 3, 9, 7), (4, 3, 2), (2, 1), (1, 0), 11), ((1, 2, 5, 5), (3, 1, 1), (1, 1), (0, 0), 12),
              ((2, 5, 6, 6), (2, 3, 3), (1, 1), (1, 1), 13)]
POOL_CASES = [((2, 3, 8, 8), (2, 2), (2, 2), (0, 0), 21), ((1, 2, 7, 9), (3, 3), (2, 2), (1, 1), 22),
              ((2, 1, 6, 5), (3, 2), (1, 1), (1, 1), 23)]


def conv_inputs(x_shape, wspec, seed):
    """``x, w, b`` ~ N(0, 1) for a conv case, and the generator that then draws the output
    gradient."""
    rng = np.random.default_rng(seed)
    c_out, kh, kw = wspec
    x = rng.standard_normal(x_shape)
    w = rng.standard_normal((c_out, x_shape[1], kh, kw))
    b = rng.standard_normal(c_out)
    return x, w, b, rng


def pool_input(x_shape, seed):
    """Values on a coarse grid (so windows hold ties) with one NaN."""
    rng = np.random.default_rng(seed)
    x = np.round(rng.standard_normal(x_shape) * 2) / 2
    x.reshape(-1)[x.size // 3] = np.nan
    return x, rng


#: Parameters of the CNN whose gradient is exactly zero: the convolution biases, each followed
#: by a batch norm.
CNN_ZERO_GRAD = {"0.bias": "0.weight", "4.bias": "4.weight"}


#: Op-level recurrent cases: (cell, T, B, I, H, seed).
RNN_CASES = [("lstm", 7, 3, 2, 5, 31), ("gru", 7, 3, 2, 5, 32), ("lstm", 4, 2, 3, 8, 33),
             ("gru", 5, 4, 6, 4, 34)]
#: The adding-problem regressors (LSTM and GRU, hidden 8, T = 12, batch 6), two AdamW steps.
RNN_SMALL = dict(hidden=8, seq=12, batch=6, seed=41, steps=2)


def rnn_inputs(cell, steps, batch, inputs, hidden, seed):
    """``x, h0, c0, w_ih, w_hh, b_ih, b_hh`` ~ N(0, 0.5) and the generator that then draws the
    output gradient (``c0`` is None for the GRU)."""
    rng = np.random.default_rng(seed)
    gates = 4 if cell == "lstm" else 3
    x = rng.standard_normal((steps, batch, inputs))
    h0 = 0.5 * rng.standard_normal((batch, hidden))
    c0 = 0.5 * rng.standard_normal((batch, hidden)) if cell == "lstm" else None
    w_ih = 0.5 * rng.standard_normal((gates * hidden, inputs))
    w_hh = 0.5 * rng.standard_normal((gates * hidden, hidden))
    b_ih = 0.5 * rng.standard_normal(gates * hidden)
    b_hh = 0.5 * rng.standard_normal(gates * hidden)
    return x, h0, c0, w_ih, w_hh, b_ih, b_hh, rng


def higher_order_inputs() -> dict[str, np.ndarray]:
    """Seeded float64 inputs of the differentiable-gradient fixture (higher_order.npz)."""
    rng = np.random.default_rng(61)
    return {
        "x": rng.standard_normal((3, 4)), "w": rng.standard_normal((4, 2)),
        "v": rng.standard_normal((3, 4)), "vw": rng.standard_normal((4, 2)),
        "c": rng.standard_normal((3, 4)),
        "xin": rng.standard_normal((5, 6)), "labels": rng.integers(0, 3, size=5),
        "w1": 0.5 * rng.standard_normal((7, 6)), "b1": 0.1 * rng.standard_normal(7),
        "w2": 0.5 * rng.standard_normal((3, 7)), "b2": 0.1 * rng.standard_normal(3),
    }
