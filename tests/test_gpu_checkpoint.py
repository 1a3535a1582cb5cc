"""Checkpoint files: the reference's ``.npz`` format both ways, and AdamW state resume.

``tests/golden/gpt_checkpoint.npz`` is the reference's own ``tensorgrad.utils.save`` of a
freshly initialised GPT (``manual_seed(7)``): the same seed must give the same weights here
(the initialisation draws in the reference's order), a model saved here must write the same
file contents, and the file must load here. The optimizer state (moments, step counts;
missing from the reference) must resume a run exactly.
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import gpt as ogpt
from tests.conftest import load_golden
from tests.golden.specs import GPT_SMALL

pytestmark = pytest.mark.gpu


def _gpt(tg, dropout=0.0):
    cfg = GPT_SMALL["cfg"]
    return tg.nn.GPT(tg.nn.GPTConfig(vocab_size=cfg.vocab_size, block_size=cfg.block_size,
                                     n_layer=cfg.n_layer, n_head=cfg.n_head, n_embd=cfg.n_embd,
                                     dropout=dropout))


def test_checkpoint_round_trips_the_reference_file(tmp_path):
    import tensorgrad_b200 as tg

    gold = load_golden("gpt_checkpoint.npz")
    tg.set_default_dtype(np.float64)
    try:
        tg.manual_seed(7)
        model = _gpt(tg)
        mine = tmp_path / "mine.ckpt"  # written to exactly this path (no suffix added)
        tg.utils.save(model, mine)
        assert mine.exists()
        saved = tg.utils.load(mine)
        assert sorted(saved) == sorted(gold)
        for name, ref in gold.items():
            np.testing.assert_array_equal(saved[name], ref, err_msg=name)
        other = _gpt(tg)
        other.load_state_dict(tg.utils.load(mine))
        for (n, p), (_, q) in zip(model.named_parameters(), other.named_parameters(), strict=True):
            np.testing.assert_array_equal(p.numpy(), q.numpy(), err_msg=n)
    finally:
        tg.set_default_dtype(np.float32)


def test_adamw_state_save_and_resume_is_exact(tmp_path):
    import tensorgrad_b200 as tg

    cfg = GPT_SMALL["cfg"]

    def run(model, opt, steps):
        params = list(model.parameters())
        for step in steps:
            ids, targets = ogpt.synthetic_batch(cfg, 4, 16, 100 + step)
            loss = tg.cross_entropy(model(ids), targets)
            opt.zero_grad()
            loss.backward()
            tg.optim.clip_grad_norm_(params, 0.5)
            opt.step()

    tg.manual_seed(3)
    a = _gpt(tg)
    opt_a = tg.optim.AdamW(list(a.parameters()), lr=1e-3, weight_decay=1e-2)
    run(a, opt_a, [1, 2])
    tg.utils.save(a, tmp_path / "model.npz")
    tg.utils.save(opt_a.state_dict(), tmp_path / "opt.npz")
    run(a, opt_a, [3, 4])

    tg.manual_seed(11)  # different initial weights: everything must come from the files
    b = _gpt(tg)
    b.load_state_dict(tg.utils.load(tmp_path / "model.npz"))
    opt_b = tg.optim.AdamW(list(b.parameters()), lr=5.0, weight_decay=0.5)
    opt_b.load_state_dict(tg.utils.load(tmp_path / "opt.npz"))
    assert opt_b.param_groups[0].lr == 1e-3
    run(b, opt_b, [3, 4])
    for (n, p), (_, q) in zip(a.named_parameters(), b.named_parameters(), strict=True):
        np.testing.assert_array_equal(p.numpy(), q.numpy(), err_msg=n)
    state = opt_b.state_dict()
    assert int(state["state.0.step"]) == 4
