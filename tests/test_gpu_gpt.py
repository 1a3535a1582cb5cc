"""Whole training steps of the GPT path on the device against the reference.

* the committed fixture (the reference itself, float64, two steps with clipping active);
* the char-GPT configuration (4 layers, d=128, 4 heads, T=128, vocab 65, batch 32) against
  the float64 oracle;
* the float64 build mode against the fixture at 1e-10.
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import gpt as ogpt
from oracle import ops as O
from tests.conftest import assert_parity, assert_update_parity, ill_conditioned, load_golden
from tests.golden.specs import GPT_SMALL

pytestmark = pytest.mark.gpu


def build(cfg: ogpt.Config, params: dict[str, np.ndarray], dtype):
    import tensorgrad_b200 as tg

    tg.set_default_dtype(dtype)
    tg.manual_seed(0)
    model = tg.nn.GPT(tg.nn.GPTConfig(vocab_size=cfg.vocab_size, block_size=cfg.block_size,
                                      n_layer=cfg.n_layer, n_head=cfg.n_head,
                                      n_embd=cfg.n_embd, dropout=0.0))
    state = dict(params)
    state["head.weight"] = params["tok_emb.weight"]
    model.load_state_dict(state)
    names = [n for n, _ in model.named_parameters()]
    assert names == [n for n, _ in ogpt.param_shapes(cfg)]
    return model, names


def run_steps(cfg, spec_batch, spec_seq, seed, steps, max_norm, dtype, device_ids=False):
    """``device_ids``: token ids and targets as device tensors (checked and sorted on the
    device) and the clip norm returned as a device scalar, the no-round-trip step."""
    import tensorgrad_b200 as tg

    model, names = build(cfg, ogpt.init_params(cfg, seed), dtype)
    params = list(model.parameters())
    opt = tg.optim.AdamW(params, lr=3e-4, betas=(0.9, 0.999), eps=1e-8, weight_decay=1e-4)
    out = []
    for step in range(1, steps + 1):
        ids, targets = ogpt.synthetic_batch(cfg, spec_batch, spec_seq, seed + step)
        if device_ids:
            ids, targets = tg.Tensor(ids), tg.Tensor(targets)
        loss = tg.cross_entropy(model(ids), targets)
        opt.zero_grad()
        loss.backward()
        total = tg.optim.clip_grad_norm_(params, max_norm, sync=not device_ids)
        total = float(total.item()) if device_ids else total
        rec = {"loss": float(loss.item()), "total_norm": total,
               "grads": {n: p.grad.numpy() for n, p in zip(names, params, strict=True)},
               "before": {n: p.numpy() for n, p in zip(names, params, strict=True)}}
        opt.step()
        rec["params"] = {n: p.numpy() for n, p in zip(names, params, strict=True)}
        out.append(rec)
    tg.set_default_dtype(np.float32)
    return out


def check_against(recs, refs, rel):
    """Loss, clip norm and every gradient with the parity metric; post-AdamW parameters with
    it too, the max criterion restricted to entries whose gradients are determined at the
    tolerance so far (``ill_conditioned``); and the first update against the float64 AdamW
    applied to our own gradients, which checks the optimizer kernel exactly."""
    ill: dict[str, np.ndarray] = {}
    for step, (rec, ref) in enumerate(zip(recs, refs, strict=True), start=1):
        assert rec["loss"] == pytest.approx(ref["loss"], rel=rel)
        assert rec["total_norm"] == pytest.approx(ref["total_norm"], rel=rel)
        for n, g in rec["grads"].items():
            assert_parity(g, ref["grads"][n], rel, f"step{step} grad {n}")
            mask = ill_conditioned(ref["grads"][n], rel)
            ill[n] = mask if n not in ill else (ill[n] | mask)
        for n, p in rec["params"].items():
            assert_update_parity(p, ref["params"][n], ill[n], rel, f"step{step} param {n}")
        if step == 1:
            for n, p in rec["params"].items():
                mine, _, _ = O.adamw_update(rec["before"][n].astype(np.float64),
                                            rec["grads"][n].astype(np.float64),
                                            np.zeros(p.shape), np.zeros(p.shape), 1, 3e-4,
                                            (0.9, 0.999), 1e-8, 1e-4)
                assert_parity(p, mine, max(rel, 1e-6), f"AdamW kernel on our grads {n}")


def golden_steps(gold, steps, names):
    return [{"loss": float(gold[f"step{k}/loss"]), "total_norm": float(gold[f"step{k}/total_norm"]),
             "grads": {n: gold[f"step{k}/grad/{n}"] for n in names},
             "params": {n: gold[f"step{k}/param/{n}"] for n in names}}
            for k in range(1, steps + 1)]


@pytest.mark.parametrize("dtype,rel", [(np.float32, 1e-4), (np.float64, 1e-10)],
                         ids=["fp32", "fp64"])
def test_gpt_small_two_steps_match_reference_fixture(dtype, rel):
    gold = load_golden("gpt_small.npz")
    s = GPT_SMALL
    recs = run_steps(s["cfg"], s["batch"], s["seq"], s["seed"], s["steps"], s["max_norm"], dtype)
    check_against(recs, golden_steps(gold, s["steps"], list(recs[0]["grads"])), rel)


@pytest.mark.parametrize("device_ids", [False, True], ids=["host_ids", "device_ids"])
def test_char_gpt_config_matches_oracle(device_ids):
    cfg = ogpt.Config(vocab_size=65, block_size=128, n_layer=4, n_head=4, n_embd=128)
    seed, batch = 7, 32
    recs = run_steps(cfg, batch, 128, seed, 1, 1.0, np.float32, device_ids)
    ref = ogpt.train_step(ogpt.init_params(cfg, seed),
                          *ogpt.synthetic_batch(cfg, batch, 128, seed + 1), cfg, max_norm=1.0)
    check_against(recs, [ref], 1e-4)


def test_first_loss_is_near_log_vocab_and_training_reduces_it():
    # The reference's training sanity check (tests/test_training.py:124-127).
    import tensorgrad_b200 as tg

    tg.manual_seed(0)
    cfg = tg.nn.GPTConfig(vocab_size=65, block_size=32, n_layer=2, n_head=4, n_embd=64)
    model = tg.nn.GPT(cfg)
    params = list(model.parameters())
    opt = tg.optim.AdamW(params, lr=3e-3, weight_decay=1e-4)
    rng = np.random.default_rng(0)
    ids = rng.integers(0, 65, size=(8, 32))
    targets = np.roll(ids, -1, axis=1)
    losses = []
    for _ in range(30):
        loss = tg.cross_entropy(model(ids), targets)
        opt.zero_grad()
        loss.backward()
        tg.optim.clip_grad_norm_(params, 1.0)
        opt.step()
        losses.append(loss.item())
    assert losses[0] == pytest.approx(np.log(65), rel=0.05)
    assert losses[-1] < 0.6 * losses[0]
