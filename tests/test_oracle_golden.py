"""The oracle against the reference's own outputs (fixtures) and known answers (CPU only)."""

from __future__ import annotations

import math

import numpy as np
import pytest

from oracle import gpt as ogpt
from oracle import ops
from tests.conftest import assert_parity, load_golden
from tests.golden.specs import ATTN_CASES, GPT_SMALL, attention_inputs

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
