"""KV-cache generation on the device against the reference's own ``GPT.generate``.

``tests/golden/gpt_generate.npz``: the reference's freshly initialised GPT (manual_seed(7),
block 16) extends a prompt by 20 tokens greedily and by seeded sampling, the window sliding
past the block on the way (both the cached and the re-encoded path run). In float64 the
tokens must be the reference's exactly; in fp32 the greedy tokens too, and every cached
decode step's logits must match a full forward of the same prefix.
"""

from __future__ import annotations

import numpy as np
import pytest

from tests.conftest import assert_parity, load_golden
from tests.golden.specs import GPT_SMALL

pytestmark = pytest.mark.gpu


def _model(tg, dtype):
    cfg = GPT_SMALL["cfg"]
    tg.set_default_dtype(dtype)
    tg.manual_seed(7)
    return tg.nn.GPT(tg.nn.GPTConfig(vocab_size=cfg.vocab_size, block_size=cfg.block_size,
                                     n_layer=cfg.n_layer, n_head=cfg.n_head, n_embd=cfg.n_embd))


def test_generation_matches_reference_in_float64():
    import tensorgrad_b200 as tg

    gold = load_golden("gpt_generate.npz")
    try:
        model = _model(tg, np.float64)
        greedy = model.generate(gold["prompt"], 20, top_k=1, rng=np.random.default_rng(1))
        sampled = model.generate(gold["prompt"], 20, temperature=0.8,
                                 rng=np.random.default_rng(2))
        model.eval()
        logits = model(gold["greedy"][:, :16]).numpy()
    finally:
        tg.set_default_dtype(np.float32)
    np.testing.assert_array_equal(greedy, gold["greedy"])
    np.testing.assert_array_equal(sampled, gold["sampled"])
    assert_parity(logits, gold["logits"], 1e-10, "logits")


def test_cached_decoding_matches_full_forward_fp32():
    import tensorgrad_b200 as tg

    gold = load_golden("gpt_generate.npz")
    model = _model(tg, np.float32)
    model.eval()
    seq = gold["sampled"][:, :16]
    full = model(seq).numpy()
    cache = model.make_cache(2)
    steps = [model(seq[:, :6], cache=cache).numpy()[:, -1]]
    for t in range(6, 16):
        steps.append(model(seq[:, t:t + 1], cache=cache).numpy()[:, -1])
    assert cache.length == 16
    for i, got in enumerate(steps):
        assert_parity(got, full[:, 5 + i], 1e-4, f"position {5 + i}")
    assert_parity(model(gold["greedy"][:, :16]).numpy(), gold["logits"], 1e-4, "logits")
    with pytest.raises(ValueError, match="exceeds block_size 16"):
        model(seq[:, :1], cache=cache)
    greedy = model.generate(gold["prompt"], 20, top_k=1, rng=np.random.default_rng(1))
    np.testing.assert_array_equal(greedy, gold["greedy"])
    no_cache = model.generate(gold["prompt"], 20, top_k=1, rng=np.random.default_rng(1),
                              use_cache=False)
    np.testing.assert_array_equal(no_cache, greedy)
    model.train()
    with pytest.raises(ValueError, match="call eval"):
        model(seq[:, :2], cache=model.make_cache(2))
