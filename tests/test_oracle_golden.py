"""The oracle against the reference's own outputs (fixtures) and known answers (CPU only)."""

from __future__ import annotations

import math

import numpy as np
import pytest

from oracle import cnn as ocnn
from oracle import gpt as ogpt
from oracle import ops
from oracle import rnn as ornn
from tests.conftest import assert_parity, assert_zero_gradient, load_golden
from tests.golden.specs import (
    ATTN_CASES, CNN_SMALL, CNN_ZERO_GRAD, CONV_CASES, GPT_SMALL, POOL_CASES, RNN_CASES, RNN_SMALL,
    attention_inputs, conv_inputs, pool_input, rnn_inputs,
)

REL64 = 1e-10  # float64 restatement vs float64 reference


def test_gpt_two_steps_match_reference_fixture() -> None:
    gold = load_golden("gpt_small.npz")
    cfg = GPT_SMALL["cfg"]
    params = ogpt.init_params(cfg, GPT_SMALL["seed"])
    state = None
    for step in range(1, GPT_SMALL["steps"] + 1):
        ids, targets = ogpt.synthetic_batch(cfg, GPT_SMALL["batch"], GPT_SMALL["seq"],
                                            GPT_SMALL["seed"] + step)
        out = ogpt.train_step(params, ids, targets, cfg, state, max_norm=GPT_SMALL["max_norm"])
        assert out["loss"] == pytest.approx(float(gold[f"step{step}/loss"]), rel=REL64)
        assert out["total_norm"] == pytest.approx(float(gold[f"step{step}/total_norm"]), rel=REL64)
        for name, g in out["grads"].items():
            assert_parity(g, gold[f"step{step}/grad/{name}"], REL64, f"step{step} grad {name}")
        for name, p in out["params"].items():
            assert_parity(p, gold[f"step{step}/param/{name}"], REL64, f"step{step} param {name}")
        params, state = out["params"], out["state"]


def test_gpt_fixture_clips() -> None:
    # The fixture's max_norm is below the gradient norm, so clipping is exercised.
    gold = load_golden("gpt_small.npz")
    assert float(gold["step1/total_norm"]) > GPT_SMALL["max_norm"]


@pytest.mark.parametrize("shape,causal,seed", ATTN_CASES)
def test_attention_matches_reference_fixture(shape, causal, seed) -> None:
    gold = load_golden("attention.npz")
    key = "x".join(map(str, shape)) + ("_causal" if causal else "")
    q, k, v, do = attention_inputs(shape, seed)
    o, p = ops.attention_forward(q, k, v, causal)
    dq, dk, dv = ops.attention_backward(do, q, k, v, p)
    for name, ours in (("out", o), ("dq", dq), ("dk", dk), ("dv", dv)):
        assert_parity(ours, gold[f"{key}/{name}"], REL64, f"{key} {name}")


def test_gelu_known_value() -> None:
    # The reference's own value check (tests/test_ops_values.py:235-240).
    out, _ = ops.gelu_forward(np.array(1.0))
    assert float(out) == pytest.approx(0.841192, abs=1e-6)


def test_cross_entropy_manual_and_ignore_index(rng) -> None:
    # tests/test_ops_values.py:149-172 of the reference.
    logits = rng.standard_normal((5, 4))
    target = np.array([0, 3, 1, 1, 2])
    logp = logits - np.log(np.exp(logits).sum(axis=1, keepdims=True))
    expected = -logp[np.arange(5), target]
    loss, _ = ops.cross_entropy_forward(logits, target)
    assert float(loss) == pytest.approx(expected.mean())
    loss, logp2 = ops.cross_entropy_forward(np.zeros((3, 4)), np.array([1, -100, 2]))
    assert float(loss) == pytest.approx(math.log(4.0))
    g = ops.cross_entropy_backward(1.0, logp2, np.array([1, -100, 2]), (3, 4))
    np.testing.assert_array_equal(g[1], 0.0)
    with pytest.raises(IndexError):
        ops.cross_entropy_forward(np.zeros((2, 3)), np.array([0, 3]))


def test_adamw_known_answers() -> None:
    # tests/test_optim.py:58-63 (first step = lr * sign(g)) and :79-87 (decoupled decay).
    p, m, v = ops.adamw_update(np.array([1.0, 2.0, 3.0]), np.array([0.5, -2.0, 1e-3]),
                               np.zeros(3), np.zeros(3), 1, 0.01, (0.9, 0.999), 1e-8, 0.0)
    np.testing.assert_allclose(p, [0.99, 2.01, 2.99], rtol=1e-6)
    p, _, _ = ops.adamw_update(np.array([1.0, -2.0]), np.zeros(2), np.zeros(2), np.zeros(2), 1,
                               0.1, (0.9, 0.999), 1e-8, 0.5)
    np.testing.assert_allclose(p, [0.95, -1.9])


def test_clip_known_answers() -> None:
    # tests/test_optim.py:139-153.
    total, g = ops.clip_grad_norm([np.array([3.0]), np.array([4.0])], 1.0)
    assert total == pytest.approx(5.0)
    np.testing.assert_allclose([g[0][0], g[1][0]], [0.6, 0.8], rtol=1e-5)
    total, g = ops.clip_grad_norm([np.array([0.5])], 1.0)
    assert total == pytest.approx(0.5)
    np.testing.assert_array_equal(g[0], [0.5])


def test_embedding_backward_is_add_at() -> None:
    # tests/test_ops_values.py:304-315.
    rng = np.random.default_rng(5)
    ids = rng.integers(0, 5, size=(7, 11))
    g = rng.standard_normal((7, 11, 3))
    expected = np.zeros((5, 3))
    for i, row in zip(ids.reshape(-1), g.reshape(-1, 3), strict=True):
        expected[i] += row
    np.testing.assert_allclose(ops.embedding_backward(ids, g, 5), expected, rtol=1e-12)
    with pytest.raises(IndexError):
        ops.embedding_forward(np.array([-1]), np.zeros((4, 3)))


# ---------------------------------------------------------------------------- CNN path
def test_cnn_two_steps_match_reference_fixture() -> None:
    gold = load_golden("cnn_small.npz")
    cfg = CNN_SMALL["cfg"]
    params, buffers, state = ocnn.init_params(cfg, CNN_SMALL["seed"]), ocnn.init_buffers(cfg), None
    for step in range(1, CNN_SMALL["steps"] + 1):
        x, labels = ocnn.synthetic_batch(cfg, CNN_SMALL["batch"], CNN_SMALL["seed"] + step)
        out = ocnn.train_step(params, buffers, x, labels, state)
        assert out["loss"] == pytest.approx(float(gold[f"step{step}/loss"]), rel=REL64)
        for name, g in out["grads"].items():
            ref = gold[f"step{step}/grad/{name}"]
            if name in CNN_ZERO_GRAD:
                scale = float(np.abs(gold[f"step{step}/grad/{CNN_ZERO_GRAD[name]}"]).max())
                assert_zero_gradient(g, scale, REL64, f"step{step} grad {name}")
                assert_zero_gradient(ref, scale, REL64, f"reference step{step} grad {name}")
            else:
                assert_parity(g, ref, REL64, f"step{step} grad {name}")
        for name, p in out["params"].items():
            assert_parity(p, gold[f"step{step}/param/{name}"], REL64, f"step{step} param {name}")
        for name, b in out["buffers"].items():
            assert_parity(b, gold[f"step{step}/buffer/{name}"], REL64, f"step{step} {name}")
        params, state = out["params"], out["state"]


@pytest.mark.parametrize("case", range(len(CONV_CASES)))
def test_conv2d_matches_reference_fixture(case) -> None:
    gold = load_golden("conv_pool.npz")
    x_shape, wspec, stride, padding, seed = CONV_CASES[case]
    x, w, b, rng = conv_inputs(x_shape, wspec, seed)
    y, cols = ocnn.conv2d_forward(x, w, b, stride, padding)
    g = rng.standard_normal(y.shape)
    gx, gw, gb = ocnn.conv2d_backward(g, x.shape, w, cols, stride, padding)
    for name, ours in (("y", y), ("gx", gx), ("gw", gw), ("gb", gb)):
        assert_parity(ours, gold[f"conv{case}/{name}"], REL64, f"conv{case} {name}")


@pytest.mark.parametrize("case", range(len(POOL_CASES)))
def test_max_pool2d_matches_reference_fixture(case) -> None:
    gold = load_golden("conv_pool.npz")
    x_shape, kernel, stride, padding, seed = POOL_CASES[case]
    x, rng = pool_input(x_shape, seed)
    y, winner = ocnn.max_pool2d_forward(x, kernel, stride, padding)
    g = rng.standard_normal(y.shape)
    gx = ocnn.max_pool2d_backward(g, winner, x.shape, kernel, stride, padding)
    np.testing.assert_array_equal(y, gold[f"pool{case}/y"])
    np.testing.assert_array_equal(gx, gold[f"pool{case}/gx"])


def naive_conv2d(x, w, b, stride, pad):
    """Direct loops over output positions (the reference's tests/test_ops_values.py:14-27)."""
    xp = np.pad(x, ((0, 0), (0, 0), (pad, pad), (pad, pad)))
    n, _, h, wd = xp.shape
    c_out, _, k, _ = w.shape
    oh, ow = (h - k) // stride + 1, (wd - k) // stride + 1
    out = np.zeros((n, c_out, oh, ow))
    for i in range(oh):
        for j in range(ow):
            patch = xp[:, :, i * stride:i * stride + k, j * stride:j * stride + k]
            out[:, :, i, j] = np.tensordot(patch, w, axes=([1, 2, 3], [1, 2, 3])) + b
    return out


@pytest.mark.parametrize(("stride", "pad"), [(1, 0), (1, 1), (2, 1), (3, 0)])
def test_conv2d_matches_naive_loops(rng, stride, pad) -> None:
    x = rng.standard_normal((2, 3, 7, 6))
    w = rng.standard_normal((4, 3, 3, 3))
    b = rng.standard_normal(4)
    y, _ = ocnn.conv2d_forward(x, w, b, (stride, stride), (pad, pad))
    np.testing.assert_allclose(y, naive_conv2d(x, w, b, stride, pad), atol=1e-12)


def argmax_pool(x, g, k, stride, pad):
    """Output and input gradient where each window's gradient goes to the cell numpy.argmax
    picks (the first maximum, or the first NaN): the rule of tests/test_ops_values.py:56-74."""
    xp = np.pad(x, ((0, 0), (0, 0), (pad, pad), (pad, pad)), constant_values=-np.inf)
    n, c, hp, wp = xp.shape
    oh, ow = (hp - k) // stride + 1, (wp - k) // stride + 1
    out = np.empty((n, c, oh, ow))
    dxp = np.zeros_like(xp)
    for bi, ch, i, j in np.ndindex(n, c, oh, ow):
        window = xp[bi, ch, i * stride:i * stride + k, j * stride:j * stride + k]
        r, q = divmod(int(np.argmax(window)), k)
        out[bi, ch, i, j] = window[r, q]
        dxp[bi, ch, i * stride + r, j * stride + q] += g[bi, ch, i, j]
    return out, dxp[:, :, pad:pad + x.shape[2], pad:pad + x.shape[3]]


@pytest.mark.parametrize(("k", "stride", "pad"), [(2, 2, 0), (3, 1, 1), (3, 2, 1), (2, 1, 0)])
def test_max_pool2d_ties_and_nans_follow_argmax(k, stride, pad) -> None:
    rng = np.random.default_rng(k * 10 + stride)
    x = np.round(rng.standard_normal((2, 3, 7, 6)))
    x.reshape(-1)[::13] = np.nan
    y, winner = ocnn.max_pool2d_forward(x, (k, k), (stride, stride), (pad, pad))
    g = rng.standard_normal(y.shape)
    gx = ocnn.max_pool2d_backward(g, winner, x.shape, (k, k), (stride, stride), (pad, pad))
    ey, egx = argmax_pool(x, g, k, stride, pad)
    np.testing.assert_array_equal(y, ey)
    np.testing.assert_allclose(gx, egx)


# ---------------------------------------------------------------------------- LSTM / GRU
def rnn_oracle(cell, x, h0, c0, w_ih, w_hh, b_ih, b_hh, g):
    """Output and gradients of one recurrent op in the fixture's order."""
    if cell == "lstm":
        out, cache = ornn.lstm_forward(x, h0, c0, w_ih, w_hh, b_ih, b_hh)
        grads = ornn.lstm_backward(g, x, h0, c0, w_ih, w_hh, True, out, cache)
        names = ["dx", "dh0", "dc0", "dw_ih", "dw_hh", "db_ih", "db_hh"]
    else:
        out, cache = ornn.gru_forward(x, h0, w_ih, w_hh, b_ih, b_hh)
        grads = ornn.gru_backward(g, x, h0, w_ih, w_hh, True, out, cache)
        names = ["dx", "dh0", "dw_ih", "dw_hh", "db_ih", "db_hh"]
    return out, dict(zip(names, grads, strict=True))


@pytest.mark.parametrize("case", range(len(RNN_CASES)))
def test_recurrent_ops_match_reference_fixture(case) -> None:
    gold = load_golden("rnn_ops.npz")
    cell, steps, batch, inputs, hidden, seed = RNN_CASES[case]
    x, h0, c0, w_ih, w_hh, b_ih, b_hh, rng = rnn_inputs(cell, steps, batch, inputs, hidden, seed)
    shape = (steps, batch, 2, hidden) if cell == "lstm" else (steps, batch, hidden)
    g = rng.standard_normal(shape)
    out, grads = rnn_oracle(cell, x, h0, c0, w_ih, w_hh, b_ih, b_hh, g)
    assert_parity(out, gold[f"{cell}{case}/out"], REL64, f"{cell}{case} out")
    for name, ours in grads.items():
        assert_parity(ours, gold[f"{cell}{case}/{name}"], REL64, f"{cell}{case} {name}")


@pytest.mark.parametrize("cell", ["lstm", "gru"])
def test_recurrent_regressor_two_steps_match_reference_fixture(cell) -> None:
    gold = load_golden("rnn_small.npz")
    s = RNN_SMALL
    cfg = ornn.Config(cell=cell, hidden=s["hidden"], seq=s["seq"])
    params, state = ornn.init_params(cfg, s["seed"]), None
    for step in range(1, s["steps"] + 1):
        x, y = ornn.synthetic_batch(cfg, s["batch"], s["seed"] + step)
        out = ornn.train_step(params, cfg, x, y, state)
        assert out["loss"] == pytest.approx(float(gold[f"{cell}/step{step}/loss"]), rel=REL64)
        for name, g in out["grads"].items():
            assert_parity(g, gold[f"{cell}/step{step}/grad/{name}"], REL64, f"step{step} {name}")
        for name, p in out["params"].items():
            assert_parity(p, gold[f"{cell}/step{step}/param/{name}"], REL64, f"step{step} {name}")
        params, state = out["params"], out["state"]


def test_extra_ops_oracle_matches_reference_fixture() -> None:
    """The oracle's softmax family, tie-sharing max / min, binary cross entropy and Elman RNN
    against the reference's own outputs (ops_extra.npz), float64 at 1e-10."""
    from tests.golden.specs import ops_extra_inputs

    gold = load_golden("ops_extra.npz")
    d = ops_extra_inputs()
    x, g = d["s_x"], d["s_g"]
    s = ops.softmax_forward(x, -1)
    assert_parity(s, gold["softmax/y"], 1e-10, "softmax")
    assert_parity(ops.softmax_backward(g, s, -1), gold["softmax/g0"], 1e-10, "softmax vjp")
    s1 = ops.softmax_forward(x, 1)
    assert_parity(ops.softmax_backward(g, s1, 1), gold["softmax_ax1/g0"], 1e-10, "softmax ax1")
    ls = ops.log_softmax(x, -1)
    assert_parity(ls, gold["log_softmax/y"], 1e-10, "log_softmax")
    assert_parity(g - np.exp(ls) * g.sum(-1, keepdims=True), gold["log_softmax/g0"], 1e-10,
                  "log_softmax vjp")
    lse = ops.logsumexp_forward(x, 1)
    assert_parity(lse[:, 0], gold["logsumexp/y"], 1e-10, "logsumexp")
    assert_parity(d["s_g1"][:, None] * np.exp(x - lse), gold["logsumexp/g0"], 1e-10,
                  "logsumexp vjp")
    sm = ops.softmax_forward(d["masked"])
    assert_parity(sm, gold["softmax_masked/y"], 1e-10, "masked softmax")
    m = d["m_x"]
    for name, fn in (("max_ax1", np.max), ("min_ax1", np.min)):
        kept = fn(m, axis=1, keepdims=True)
        np.testing.assert_array_equal(kept[:, 0], gold[f"{name}/y"])
        gx = ops.extremum_backward(d["m_g1"][:, None], m, kept, (1,))
        assert_parity(gx, gold[f"{name}/g0"], 1e-10, name)
    z, y = d["b_z"], d["b_y"]
    losses = ops.bce_with_logits_forward(z, y)
    assert_parity(losses, gold["bce_none/y"], 1e-10, "bce")
    assert float(losses.mean()) == pytest.approx(float(gold["bce_mean/y"]), rel=1e-12)
    gz, gy = ops.bce_with_logits_backward(d["b_g"], z, y)
    assert_parity(gz, gold["bce_none/g0"], 1e-10, "bce dz")
    assert_parity(gy, gold["bce_none/g1"], 1e-10, "bce dy")
    args = [d[k] for k in ("rx", "rh0", "r_wih", "r_whh", "r_bih", "r_bhh")]
    for act in ("tanh", "relu"):
        relu = act == "relu"
        out = ornn.rnn_forward(*args, relu=relu)
        assert_parity(out, gold[f"rnn_{act}/y"], 1e-10, f"rnn {act}")
        grads = ornn.rnn_backward(d["r_g"], args[0], args[1], args[2], args[3], True, out,
                               relu=relu)
        for i, gr in enumerate(grads):
            assert_parity(gr, gold[f"rnn_{act}/g{i}"], 1e-10, f"rnn {act} grad {i}")
