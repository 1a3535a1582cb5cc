"""Differentiable gradients on the device (``create_graph=True`` and ``func``) against the
reference's own results (``tests/golden/higher_order.npz``, float64): gradients, a Hessian, a
Hessian-vector product, a Jacobian and a Jacobian-vector product of small functions of
elementwise, matrix and reduction ops (tanh, sigmoid, exp, log, sqrt, gelu, mean, division,
broadcasting), and a gradient penalty on an MLP with cross entropy: backward through an input
gradient that was itself built with ``create_graph``. float64 at 1e-10, fp32 at 1e-4.
"""

from __future__ import annotations

import numpy as np
import pytest

from tests.conftest import assert_parity, load_golden
from tests.golden.specs import higher_order_inputs

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype,rel", [(np.float64, 1e-10), (np.float32, 1e-4)],
                         ids=["fp64", "fp32"])
def test_function_transforms_match_reference(dtype, rel):
    import tensorgrad_b200 as tg
    from tensorgrad_b200 import func

    gold = load_golden("higher_order.npz")
    d = {k: (v.astype(dtype) if v.dtype.kind == "f" else v) for k, v in higher_order_inputs().items()}
    x, w, v, vw = (tg.Tensor(d[k]) for k in ("x", "w", "v", "vw"))

    def f(x_, w_):
        return (tg.tanh(x_ @ w_) ** 2).sum()

    def g(x_):
        return tg.sigmoid(x_ @ tg.Tensor(d["w"])).reshape(-1)

    def h(x_):
        return (tg.mean(tg.exp(x_) / (x_ * x_ + 1.0)) + tg.log(x_ * x_ + 1.0).sum()
                + (tg.gelu(x_) * tg.Tensor(d["c"])).sum() + tg.sqrt(x_ * x_ + 2.0).sum())

    gx, gw = func.grad(f, argnums=(0, 1))(x, w)
    assert_parity(gx.numpy(), gold["grad_x"], rel, "grad x")
    assert_parity(gw.numpy(), gold["grad_w"], rel, "grad w")
    assert_parity(func.hessian(f)(x, w).numpy(), gold["hess_x"], rel, "hessian")
    _, (hx, hw) = func.hvp(f, (x, w), (v, vw))
    assert_parity(hx.numpy(), gold["hvp_x"], rel, "hvp x")
    assert_parity(hw.numpy(), gold["hvp_w"], rel, "hvp w")
    _, jv = func.jvp(g, (x,), (v,))
    assert_parity(jv.numpy(), gold["jvp"], rel, "jvp")
    assert_parity(func.jacobian(g)(x).numpy(), gold["jac"], rel, "jacobian")
    assert_parity(func.hessian(h)(x).numpy(), gold["hess_h"], rel, "hessian (h)")


@pytest.mark.parametrize("dtype,rel", [(np.float64, 1e-10), (np.float32, 1e-4)],
                         ids=["fp64", "fp32"])
def test_gradient_penalty_backward_matches_reference(dtype, rel):
    import tensorgrad_b200 as tg

    gold = load_golden("higher_order.npz")
    d = higher_order_inputs()
    w1, b1, w2, b2, xin = (tg.Tensor(d[k].astype(dtype), requires_grad=True)
                           for k in ("w1", "b1", "w2", "b2", "xin"))
    loss = tg.cross_entropy(tg.linear(tg.relu(tg.linear(xin, w1, b1)), w2, b2), d["labels"])
    (gin,) = tg.autograd.grad(loss, [xin], create_graph=True)
    assert gin.requires_grad
    total = loss + (gin * gin).sum()
    total.backward()
    assert float(total.item()) == pytest.approx(float(gold["penalty_total"]), rel=rel)
    for k, t in (("w1", w1), ("b1", b1), ("w2", w2), ("b2", b2), ("xin", xin)):
        assert_parity(t.grad.numpy(), gold[f"penalty_grad_{k}"], rel, f"penalty grad {k}")


def test_a_node_without_a_differentiable_vjp_raises():
    """Every op of the package has a graph VJP; a node made without one (a user's own op)
    is refused by ``create_graph`` with its name, and still works to first order."""
    import tensorgrad_b200 as tg
    from tensorgrad_b200.ops._util import make_result

    x = tg.Tensor(np.random.default_rng(0).standard_normal((2, 8)).astype(np.float32),
                  requires_grad=True)
    y = make_result(x.data, (x,), lambda g, need: (g,), "user_identity").sum()
    with pytest.raises(NotImplementedError, match="user_identity"):
        tg.autograd.grad(y, [x], create_graph=True, retain_graph=True)
    (g,) = tg.autograd.grad(y, [x])
    np.testing.assert_array_equal(g.numpy(), np.ones((2, 8), np.float32))
