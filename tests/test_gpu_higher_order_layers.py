"""Second derivatives through the fused device layers against the reference's own results
(``tests/golden/higher_order_layers.npz``, float64; the programs are shared with the fixture
generator, ``specs.higher_order_layer_program`` and ``specs.gpt_penalty_program``):

* Hessian-vector products of scalar functions of layer norm, attention (causal, full, with
  dropout on the weights, the packed form with dropout), embedding + layer norm + cross
  entropy, LSTM, GRU and dropout, and the Hessian of a function of ``var``;
* gradient penalties through conv2d -> batch norm -> ReLU -> max pooling (3 x 3 windows of
  stride 2 with padding, and 2 x 2), differentiated to the input and every parameter;
* one GPT step with dropout 0.1 on ``loss + 0.01 * sum(grad ** 2)``.

float64 at 1e-10 (1e-9 for the GPT penalty: three passes through twelve kernels); fp32 at 1e-3
(second derivatives through 3xTF32 products and fp32 reductions).
"""

from __future__ import annotations

import types

import numpy as np
import pytest

from tests.conftest import assert_parity, assert_zero_gradient, load_golden
from tests.golden.specs import (
    GPT_PENALTY, gpt_penalty_program, higher_order_layer_inputs, higher_order_layer_program,
)

pytestmark = pytest.mark.gpu


def _ops(tg):
    from tensorgrad_b200 import ops

    return types.SimpleNamespace(
        tanh=tg.tanh, relu=tg.relu, layer_norm=tg.layer_norm, var=ops.var,
        sdpa=ops.scaled_dot_product_attention, packed=ops.packed_self_attention,
        conv2d=tg.conv2d, batch_norm=ops.batch_norm, max_pool2d=tg.max_pool2d,
        embedding=tg.embedding, linear=tg.linear, cross_entropy=tg.cross_entropy,
        lstm=ops.lstm, gru=ops.gru, dropout=tg.dropout)


def _host(t):
    return t.numpy()


@pytest.mark.parametrize("dtype,rel", [(np.float64, 1e-10), (np.float32, 1e-3)],
                         ids=["fp64", "fp32"])
def test_layer_second_derivatives_match_reference(dtype, rel):
    import tensorgrad_b200 as tg
    from tensorgrad_b200 import func

    gold = load_golden("higher_order_layers.npz")
    d = {k: (v.astype(dtype) if v.dtype.kind == "f" else v)
         for k, v in higher_order_layer_inputs().items()}
    tg.set_default_dtype(dtype)
    try:
        ours = higher_order_layer_program(tg, _ops(tg), func, _host, d)
    finally:
        tg.set_default_dtype(np.float32)
    assert set(ours) == {k for k in gold if not k.startswith("gpt_")}
    for k, v in ours.items():
        if k.endswith("_grad_b"):
            # The conv bias ahead of a batch norm: zero in exact arithmetic.
            scale = float(np.abs(gold[k.replace("_grad_b", "_grad_w")]).max())
            assert_zero_gradient(v, scale, rel, k)
        else:
            assert_parity(v, gold[k], rel, k)


@pytest.mark.parametrize("dtype,rel", [(np.float64, 1e-9), (np.float32, 1e-3)],
                         ids=["fp64", "fp32"])
def test_gpt_gradient_penalty_matches_reference(dtype, rel):
    import tensorgrad_b200 as tg

    gold = load_golden("higher_order_layers.npz")
    tg.set_default_dtype(dtype)
    try:
        ours = gpt_penalty_program(tg, tg.nn, _host, GPT_PENALTY)
    finally:
        tg.set_default_dtype(np.float32)
    assert set(ours) == {k for k in gold if k.startswith("gpt_")}
    for k in ("gpt_loss", "gpt_total"):
        assert np.shape(ours[k]) == np.shape(gold[k]), (k, np.shape(ours[k]))
        assert float(ours[k]) == pytest.approx(float(gold[k]), rel=rel), k
    for k, v in ours.items():
        if k.startswith("gpt_grad/"):
            assert_parity(v, gold[k], rel, k)
