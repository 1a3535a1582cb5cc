"""Finite-difference checks of every differentiable op on the device (the reference's
tests/test_gradcheck_ops.py strategy): ``gradcheck`` compares each op's VJP with central
differences of ``sum(op(inputs) * w)``, and ``gradgradcheck`` checks its differentiable VJP
(``create_graph``) against the plain one and its second derivatives against central
differences of the first. float64, seeded inputs of a few elements, broadcasting pairs
included.
"""

from __future__ import annotations

import zlib

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _leaf(rng, *shape, positive=False, distinct=False):
    import tensorgrad_b200 as tg

    if distinct:  # well-separated values: extrema and pooling winners stay put under eps
        n = int(np.prod(shape)) if shape else 1
        data = rng.permutation(n).reshape(shape).astype(np.float64) * 0.25 + rng.random(shape) * 0.01
    else:
        data = rng.standard_normal(shape)
    if positive:
        data = np.abs(data) + 0.5
    return tg.Tensor(np.asarray(data, dtype=np.float64), requires_grad=True)


def _case(name):
    """(function, inputs) of one case."""
    import tensorgrad_b200 as tg
    from tensorgrad_b200 import ops
    from tensorgrad_b200.ops.conv import conv2d_input_grad, conv2d_weight_grad
    from tensorgrad_b200.utils import checkpoint

    rng = np.random.default_rng(zlib.crc32(name.encode()))
    L = lambda *s, **k: _leaf(rng, *s, **k)  # noqa: E731
    cases = {
        "add_bcast": (lambda a, b: a + b, [L(2, 3), L(3)]),
        "sub_bcast": (lambda a, b: a - b, [L(2, 1), L(1, 3)]),
        "mul_scalar_bcast": (lambda a, b: a * b, [L(), L(2, 2)]),
        "div": (lambda a, b: a / b, [L(2, 3), L(2, 3, positive=True)]),
        "pow_tensor": (lambda a, b: a ** b, [L(2, 2, positive=True), L(2, 1)]),
        "pow_scalar": (lambda a: a ** 3.0, [L(5)]),
        "rpow": (lambda a: 2.0 ** a, [L(4)]),
        "unary": (lambda a: tg.exp(a) + tg.tanh(a) + tg.sigmoid(a) - a, [L(2, 3)]),
        "log_sqrt": (lambda a: tg.log(a) * tg.sqrt(a), [L(5, positive=True)]),
        "relu_gelu": (lambda a: tg.relu(a) + tg.gelu(a), [L(6)]),
        "sum_mean_var": (lambda a: a.sum(axis=1) + a.mean(axis=1) + a.var(axis=1)
                         + ops.var(a, 1, correction=0), [L(3, 4)]),
        "max_min": (lambda a: a.max(axis=0) * 2.0 + a.min(axis=1, keepdims=True).sum(),
                    [L(3, 4, distinct=True)]),
        "softmax_family": (lambda a: tg.softmax(a, 0) + tg.log_softmax(a, -1)
                           + tg.logsumexp(a, 1, keepdims=True), [L(3, 4)]),
        "shape_ops": (lambda a: ops.permute(a, (2, 0, 1)).reshape(4, 6)[1:3, ::2]
                      .unsqueeze(0).squeeze(0), [L(2, 3, 4)]),
        "broadcast_sum_to": (lambda a: ops.sum_to(ops.broadcast_to(a, (2, 3, 4)), (3, 1)),
                             [L(3, 1)]),
        "advanced_index": (lambda a: a[np.array([2, 0, 2])]
                           + a[np.array([[True, False, True, True]] * 3)].sum(), [L(3, 4)]),
        "stack_concat": (lambda a, b: tg.concat([tg.stack([a, b], 1).reshape(2, 6), a], 1),
                         [L(2, 3), L(2, 3)]),
        "where_masked": (lambda a, b: tg.where(np.array([[True, False, True]]), a, b)
                         + a.masked_fill(np.array([False, True, False]), 0.5), [L(2, 3), L(3)]),
        "matmul": (lambda a, b: a @ b, [L(2, 1, 3, 4), L(3, 4, 2)]),
        "matvec_dot": (lambda a, b: (a @ b) * (b @ b), [L(3, 4), L(4)]),
        "linear": (lambda x, w, b: tg.linear(x, w, b), [L(2, 3, 4), L(5, 4), L(5)]),
        "layer_norm": (lambda x, w, b: tg.layer_norm(x, w, b), [L(3, 5), L(5), L(5)]),
        "batch_norm": (lambda x, w, b: ops.batch_norm(x, None, None, w, b, training=True),
                       [L(3, 2, 2, 2), L(2), L(2)]),
        "conv2d": (lambda x, w, b: tg.conv2d(x, w, b, stride=2, padding=1),
                   [L(1, 2, 5, 5), L(3, 2, 3, 3), L(3)]),
        "conv2d_grads": (lambda g, w, x: conv2d_input_grad(g, w, (1, 2, 4, 4), 1, 1).sum()
                         + conv2d_weight_grad(x, g, (3, 2, 3, 3), 1, 1),
                         [L(1, 3, 4, 4), L(3, 2, 3, 3), L(1, 2, 4, 4)]),
        "max_pool": (lambda x: tg.max_pool2d(x, 3, 2, 1) + tg.max_pool2d(x, 2).sum(),
                     [L(1, 2, 4, 4, distinct=True)]),
        "embedding": (lambda w: tg.embedding(np.array([[1, 3, 1], [0, 2, 3]]), w), [L(4, 3)]),
        "dropout": (lambda x: tg.dropout(x, 0.3, True, np.random.default_rng(3)), [L(4, 5)]),
        "attention": (lambda q, k, v: ops.scaled_dot_product_attention(q, k, v, causal=True),
                      [L(1, 2, 3, 4), L(1, 2, 3, 4), L(1, 2, 3, 4)]),
        "attention_bcast_kv": (lambda q, k, v: ops.scaled_dot_product_attention(q, k, v),
                               [L(2, 3, 4), L(1, 5, 4), L(1, 5, 4)]),
        "attention_dropout": (lambda q, k, v: ops.scaled_dot_product_attention(
            q, k, v, causal=True, dropout_p=0.3, training=True, rng=np.random.default_rng(4)),
            [L(1, 1, 4, 8), L(1, 1, 4, 8), L(1, 1, 4, 8)]),
        "packed_attention": (lambda qkv: ops.packed_self_attention(qkv, 2), [L(1, 3, 12)]),
        "cross_entropy": (lambda z: tg.cross_entropy(z, np.array([0, 2, 1])), [L(3, 4)]),
        "mse_bce": (lambda z, y: tg.mse_loss(z, y) + tg.binary_cross_entropy_with_logits(z, y),
                    [L(2, 3), L(2, 3)]),
        "lstm": (lambda x, h, c, wi, wh, bi, bh: ops.lstm(x, h, c, wi, wh, bi, bh),
                 [L(3, 2, 2), L(2, 3), L(2, 3), L(12, 2), L(12, 3), L(12), L(12)]),
        "gru": (lambda x, h, wi, wh, bi, bh: ops.gru(x, h, wi, wh, bi, bh),
                [L(3, 2, 2), L(2, 3), L(9, 2), L(9, 3), L(9), L(9)]),
        "rnn_tanh": (lambda x, h, wi, wh: ops.rnn(x, h, wi, wh), [L(3, 2, 2), L(2, 3), L(3, 2),
                                                                   L(3, 3)]),
        "rnn_relu": (lambda x, h, wi, wh, bi, bh: ops.rnn(x, h, wi, wh, bi, bh,
                                                          nonlinearity="relu"),
                     [L(3, 2, 2), L(2, 3), L(3, 2), L(3, 3), L(3), L(3)]),
        "checkpoint": (lambda x, w: checkpoint(lambda t: tg.tanh(t @ w) * t, x, params=[w]),
                       [L(2, 3), L(3, 3)]),
    }
    return cases[name]


NAMES = [
    "add_bcast", "sub_bcast", "mul_scalar_bcast", "div", "pow_tensor", "pow_scalar", "rpow",
    "unary", "log_sqrt", "relu_gelu", "sum_mean_var", "max_min", "softmax_family", "shape_ops",
    "broadcast_sum_to", "advanced_index", "stack_concat", "where_masked", "matmul",
    "matvec_dot", "linear", "layer_norm", "batch_norm", "conv2d", "conv2d_grads", "max_pool",
    "embedding", "dropout", "attention", "attention_bcast_kv", "attention_dropout",
    "packed_attention", "cross_entropy", "mse_bce", "lstm", "gru", "rnn_tanh", "rnn_relu",
    "checkpoint",
]


@pytest.mark.parametrize("name", NAMES)
def test_first_derivatives(name):
    from tensorgrad_b200.utils import gradcheck

    fn, inputs = _case(name)
    assert gradcheck(fn, inputs)


# Second derivatives: the graph VJPs; a leaner set of inputs per case keeps the double loop
# (central differences of the first derivative) small.
@pytest.mark.parametrize("name", [n for n in NAMES if n not in (
    "lstm", "gru", "conv2d_grads", "packed_attention", "attention_bcast_kv")])
def test_second_derivatives(name):
    from tensorgrad_b200.utils import gradgradcheck

    fn, inputs = _case(name)
    assert gradgradcheck(fn, inputs)


@pytest.mark.parametrize("name", ["lstm", "gru", "conv2d_grads", "packed_attention",
                                  "attention_bcast_kv"])
def test_second_derivatives_of_the_larger_cases(name):
    """The same check with only the first input differentiated (the others held fixed)."""
    from tensorgrad_b200.utils import gradgradcheck

    fn, inputs = _case(name)
    for t in inputs[1:]:
        t.requires_grad = False
    assert gradgradcheck(fn, inputs)
