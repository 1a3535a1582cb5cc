"""Gradient checkpointing on the device (the reference's tests/test_checkpoint.py): the same
values and derivatives as without it, less device memory.

* a Linear -> GELU -> Dropout -> Linear block: loss, parameter and input gradients equal to
  the plain forward pass (the recomputation replays the dropout masks), float64 and fp32;
* Hessian-vector products through a checkpointed MLP (``create_graph`` over the recomputed
  graph), ``autograd.grad`` leaving ``.grad`` alone, a retained graph replaying the same masks,
  ``func.grad`` seeing through a checkpoint, and the reference's error cases;
* eight checkpointed MLP blocks: peak pool memory under half of the plain pass;
* two GPT training steps with dropout 0.1 and every block checkpointed against the
  reference's own run of the same steps without checkpointing (the float64 fixture
  ``gpt_dropout.npz``) is in ``test_gpu_dropout.py``.
"""

from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture
def f64():
    import tensorgrad_b200 as tg

    tg.set_default_dtype(np.float64)
    yield
    tg.set_default_dtype(np.float32)


def _block(tg, width=16, p=0.3):
    return tg.nn.Sequential(tg.nn.Linear(4, width), tg.nn.GELU(), tg.nn.Dropout(p),
                            tg.nn.Linear(width, 4))


def _gradients(tg, model, x, forward):
    model.zero_grad()
    x.zero_grad()
    tg.manual_seed(7)  # the same dropout masks for both variants
    loss = (forward(x) ** 2).sum()
    loss.backward()
    grads = [p.grad.numpy() for p in model.parameters() if p.grad is not None]
    return float(loss.item()), grads + [x.grad.numpy()]


@pytest.mark.parametrize("dtype,rel", [(np.float64, 1e-12), (np.float32, 1e-6)],
                         ids=["fp64", "fp32"])
def test_values_and_gradients_match_the_plain_pass(dtype, rel):
    import tensorgrad_b200 as tg
    from tensorgrad_b200.utils import checkpoint

    tg.set_default_dtype(dtype)
    try:
        tg.manual_seed(0)
        model = _block(tg)
        x = tg.Tensor(np.random.default_rng(1).standard_normal((5, 4)).astype(dtype),
                      requires_grad=True)
        loss_plain, plain = _gradients(tg, model, x, model)
        loss_ckpt, ckpt = _gradients(tg, model, x, lambda t: checkpoint(model, t))
    finally:
        tg.set_default_dtype(np.float32)
    assert len(plain) == len(ckpt) == 5
    assert loss_ckpt == pytest.approx(loss_plain, rel=rel)
    for a, b in zip(plain, ckpt, strict=True):
        np.testing.assert_allclose(b, a, rtol=rel, atol=rel * np.abs(a).max())
    tg.manual_seed(7)
    expected = model(x).numpy()
    tg.manual_seed(7)
    np.testing.assert_allclose(checkpoint(model, x).numpy(), expected, rtol=rel,
                               atol=rel * np.abs(expected).max())


def test_hessian_vector_products_match(f64):
    import tensorgrad_b200 as tg
    from tensorgrad_b200.utils import checkpoint

    tg.manual_seed(0)
    model = tg.nn.Sequential(tg.nn.Linear(3, 8), tg.nn.Tanh(), tg.nn.Linear(8, 1))
    x = tg.Tensor(np.random.default_rng(2).standard_normal((4, 3)))
    params = list(model.parameters())
    rng = np.random.default_rng(1)
    v = [tg.Tensor(rng.standard_normal(p.shape)) for p in params]

    def hvp(forward):
        grads = tg.autograd.grad(forward(x).sum(), params, create_graph=True)
        dot = (grads[0] * v[0]).sum()
        for g, u in zip(grads[1:], v[1:], strict=True):
            dot = dot + (g * u).sum()
        hs = tg.autograd.grad(dot, params, allow_unused=True)  # the last bias: no curvature
        return [np.zeros(p.shape) if h is None else h.numpy()
                for h, p in zip(hs, params, strict=True)]

    for a, b in zip(hvp(model), hvp(lambda t: checkpoint(model, t)), strict=True):
        np.testing.assert_allclose(b, a, rtol=1e-10, atol=1e-12)


def test_autograd_grad_through_a_checkpoint_leaves_dot_grad_alone(f64):
    import tensorgrad_b200 as tg
    from tensorgrad_b200.utils import checkpoint

    tg.manual_seed(0)
    model = tg.nn.Sequential(tg.nn.Linear(3, 4), tg.nn.ReLU())
    x = tg.Tensor(np.random.default_rng(3).standard_normal((2, 3)), requires_grad=True)
    params = list(model.parameters())
    expected = tg.autograd.grad(model(x).sum(), [x, *params])
    got = tg.autograd.grad(checkpoint(model, x).sum(), [x, *params])
    for a, b in zip(expected, got, strict=True):
        np.testing.assert_allclose(b.numpy(), a.numpy(), rtol=1e-12)
    assert all(p.grad is None for p in params)
    assert x.grad is None


def test_retained_graph_replays_the_same_dropout_masks(f64):
    import tensorgrad_b200 as tg
    from tensorgrad_b200.utils import checkpoint

    tg.manual_seed(0)
    model = _block(tg)
    x = tg.Tensor(np.random.default_rng(4).standard_normal((5, 4)), requires_grad=True)
    loss = checkpoint(model, x).sum()
    loss.backward(retain_graph=True)
    first = x.grad.numpy()
    tg.manual_seed(123)  # draws after the forward pass do not change the replayed masks
    loss.backward()
    np.testing.assert_allclose(x.grad.numpy(), 2 * first, rtol=1e-12)


def test_func_transforms_see_through_checkpoints(f64):
    import tensorgrad_b200 as tg
    from tensorgrad_b200 import func
    from tensorgrad_b200.utils import checkpoint

    def f(x):
        return checkpoint(lambda y: tg.tanh(y) ** 3, x).sum()

    x = tg.Tensor(np.array([0.3, -0.7]))
    t = np.tanh(x.numpy())
    np.testing.assert_allclose(func.grad(f)(x).numpy(), 3 * t**2 * (1 - t**2), rtol=1e-12)


def test_tensors_used_but_not_declared_are_an_error(f64):
    import tensorgrad_b200 as tg
    from tensorgrad_b200.utils import checkpoint

    w = tg.Tensor(np.eye(3), requires_grad=True)
    out = checkpoint(lambda x: x @ w, tg.Tensor(np.ones((2, 3)), requires_grad=True))
    with pytest.raises(RuntimeError, match="neither an argument nor in params"):
        out.sum().backward()
    # Declared, the same function is fine and w gets its gradient through the checkpoint.
    x = tg.Tensor(np.ones((2, 3)), requires_grad=True)
    checkpoint(lambda x_: x_ @ w, x, params=[w]).sum().backward()
    np.testing.assert_allclose(w.grad.numpy(), np.full((3, 3), 2.0))
    np.testing.assert_allclose(x.grad.numpy(), np.ones((2, 3)))


def test_argument_validation(f64):
    import tensorgrad_b200 as tg
    from tensorgrad_b200.utils import checkpoint

    w = tg.Tensor(np.ones((3, 3)), requires_grad=True)
    with pytest.raises(ValueError, match="leaf"):
        checkpoint(lambda x: x, tg.Tensor(np.ones(3)), params=[w * 2])
    with pytest.raises(TypeError, match="must return a Tensor"):
        checkpoint(lambda x: x.numpy(), tg.Tensor(np.ones(3)))


def test_checkpointing_every_block_lowers_peak_memory():
    """Eight MLP blocks on (4096, 256) fp32: the plain pass keeps every block's hidden
    activations (two (4096, 2048) buffers each) until the backward pass reaches it; the
    checkpointed pass keeps only the block boundaries and one block's recomputation."""
    import tensorgrad_b200 as tg
    from tensorgrad_b200 import device
    from tensorgrad_b200.utils import checkpoint

    tg.manual_seed(0)
    blocks = [tg.nn.MLP([256, 2048, 256], activation="gelu") for _ in range(8)]
    x = tg.Tensor(np.random.default_rng(5).standard_normal((4096, 256)).astype(np.float32),
                  requires_grad=True)

    def peak(use_checkpoint: bool) -> tuple[int, np.ndarray]:
        for b in blocks:
            b.zero_grad()
        x.zero_grad()
        device.synchronize()
        base = device.memory_stats(reset_peak=True)["used"]
        h = x
        for b in blocks:
            h = checkpoint(b, h) if use_checkpoint else b(h)
        h.sum().backward()
        device.synchronize()
        return device.memory_stats()["peak"] - base, x.grad.numpy()

    peak(False)  # warm the pool and the library's workspaces
    plain, g_plain = peak(False)
    ckpt, g_ckpt = peak(True)
    assert ckpt < 0.5 * plain, (ckpt, plain)
    np.testing.assert_allclose(g_ckpt, g_plain, rtol=1e-5, atol=1e-6 * np.abs(g_plain).max())
