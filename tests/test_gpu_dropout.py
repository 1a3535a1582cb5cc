"""Dropout on the device with the reference's keep-masks (generated from the PCG64 state).

* the dropout op against the reference's keep_mask fixtures, bit for bit (output, VJP, and
  where the generator continues);
* attention dropout (scaled_dot_product_attention and the packed self-attention) against the
  float64 oracle driven with the same mask;
* two GPT training steps with dropout 0.1 everywhere against the reference's own run, with
  and without gradient checkpointing of every block.
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import gpt as ogpt
from oracle import ops as O
from tests.conftest import assert_parity, load_golden
from tests.golden.specs import DROPOUT_CASES, GPT_DROPOUT
from tests.test_gpu_gpt import check_against, golden_steps

pytestmark = pytest.mark.gpu


def _generator(seed: int) -> np.random.Generator:
    rng = np.random.default_rng(seed)
    rng.integers(0, 2**32, size=3, dtype=np.uint32)
    return rng


@pytest.mark.parametrize("dtype", [np.float32, np.float64], ids=["fp32", "fp64"])
@pytest.mark.parametrize("case", range(len(DROPOUT_CASES)))
def test_dropout_matches_reference_mask_bitwise(dtype, case):
    import tensorgrad_b200 as tg

    gold = load_golden("dropout_masks.npz")
    shape, p, seed = DROPOUT_CASES[case]
    keep, scale = gold[f"case{case}/keep"], float(gold[f"case{case}/scale"])
    mask = keep * np.asarray(scale, dtype=dtype)
    x = np.random.default_rng(case).standard_normal(shape).astype(dtype)
    g = np.random.default_rng(case + 10).standard_normal(shape).astype(dtype)
    rng = _generator(seed)
    tx = tg.Tensor(x, requires_grad=True)
    y = tg.dropout(tx, p, training=True, rng=rng)
    y.backward(g)
    np.testing.assert_array_equal(y.numpy(), x * mask)
    np.testing.assert_array_equal(tx.grad.numpy(), g * mask)
    np.testing.assert_array_equal(rng.integers(0, 2**32, size=3, dtype=np.uint32),
                                  gold[f"case{case}/next_u32"])


@pytest.mark.parametrize("dtype,rel", [(np.float32, 1e-4), (np.float64, 1e-10)],
                         ids=["fp32", "fp64"])
@pytest.mark.parametrize("shape,causal", [((2, 3, 37, 16), False), ((1, 2, 64, 32), True),
                                          ((1, 2, 130, 64), True), ((2, 2, 33, 8), True)])
def test_attention_dropout_matches_oracle(dtype, rel, shape, causal):
    import tensorgrad_b200 as tg

    rng = np.random.default_rng(sum(shape))
    q, k, v, do = (rng.standard_normal(shape) for _ in range(4))
    tq, tk, tv = (tg.Tensor(a.astype(dtype), requires_grad=True) for a in (q, k, v))
    o = tg.nn.functional.scaled_dot_product_attention(
        tq, tk, tv, causal=causal, dropout_p=0.1, training=True, rng=np.random.default_rng(5))
    dq, dk, dv = tg.autograd.grad(o, [tq, tk, tv], grad_outputs=do.astype(dtype))
    keep, ks = O.keep_mask(shape[:-1] + (shape[-2],), 0.1, np.random.default_rng(5))
    ref_o, p = O.attention_forward(q, k, v, causal, keep, ks)
    refs = (ref_o, *O.attention_backward(do, q, k, v, p, keep, ks))
    for got, ref, name in zip((o, dq, dk, dv), refs, ("out", "dq", "dk", "dv"), strict=True):
        assert_parity(got.numpy(), ref, rel, name)


def test_packed_attention_dropout_matches_oracle():
    import tensorgrad_b200 as tg

    b, t, h, hd = 2, 48, 2, 32
    rng = np.random.default_rng(3)
    qkv, g = rng.standard_normal((b, t, 3 * h * hd)), rng.standard_normal((b, t, h * hd))
    x = tg.Tensor(qkv.astype(np.float32), requires_grad=True)
    y = tg.nn.functional.packed_self_attention(x, h, dropout_p=0.2, training=True,
                                               rng=np.random.default_rng(8))
    y.backward(g.astype(np.float32))
    keep, ks = O.keep_mask((b, h, t, t), 0.2, np.random.default_rng(8))
    q, k, v = O.split_heads(qkv, h)
    out, p = O.attention_forward(q, k, v, True, keep, ks)
    assert_parity(y.numpy(), out.transpose(0, 2, 1, 3).reshape(b, t, h * hd), 1e-4, "y")
    gy = g.reshape(b, t, h, hd).transpose(0, 2, 1, 3)
    dq, dk, dv = O.attention_backward(gy, q, k, v, p, keep, ks)
    ref = np.stack([a.transpose(0, 2, 1, 3) for a in (dq, dk, dv)], 2).reshape(b, t, 3 * h * hd)
    assert_parity(x.grad.numpy(), ref, 1e-4, "dqkv")


@pytest.mark.parametrize("recompute", [False, True], ids=["plain", "checkpointed"])
@pytest.mark.parametrize("dtype,rel", [(np.float32, 1e-4), (np.float64, 1e-10)],
                         ids=["fp32", "fp64"])
def test_gpt_with_dropout_matches_reference_fixture(dtype, rel, recompute):
    """With ``recompute`` every block is checkpointed (``GPT.gradient_checkpointing``): the
    backward pass recomputes each block under the generator state of its forward pass, so
    losses, gradients and updates still match the reference's run without checkpointing."""
    import tensorgrad_b200 as tg

    gold = load_golden("gpt_dropout.npz")
    s = GPT_DROPOUT
    cfg = s["cfg"]
    tg.set_default_dtype(dtype)
    try:
        model = tg.nn.GPT(tg.nn.GPTConfig(vocab_size=cfg.vocab_size, block_size=cfg.block_size,
                                          n_layer=cfg.n_layer, n_head=cfg.n_head,
                                          n_embd=cfg.n_embd, dropout=s["dropout"]))
        model.gradient_checkpointing = recompute
        init = ogpt.init_params(cfg, s["seed"])
        model.load_state_dict({**init, "head.weight": init["tok_emb.weight"]})
        tg.manual_seed(s["reseed"])
        names = [n for n, _ in model.named_parameters()]
        params = list(model.parameters())
        opt = tg.optim.AdamW(params, lr=3e-4, betas=(0.9, 0.999), eps=1e-8, weight_decay=1e-4)
        recs = []
        for step in range(1, s["steps"] + 1):
            ids, targets = ogpt.synthetic_batch(cfg, s["batch"], s["seq"], s["seed"] + step)
            loss = tg.cross_entropy(model(ids), targets)
            opt.zero_grad()
            loss.backward()
            total = tg.optim.clip_grad_norm_(params, s["max_norm"])
            rec = {"loss": float(loss.item()), "total_norm": total,
                   "grads": {n: p.grad.numpy() for n, p in zip(names, params, strict=True)},
                   "before": {n: p.numpy() for n, p in zip(names, params, strict=True)}}
            opt.step()
            rec["params"] = {n: p.numpy() for n, p in zip(names, params, strict=True)}
            recs.append(rec)
    finally:
        tg.set_default_dtype(np.float32)
    check_against(recs, golden_steps(gold, s["steps"], names), rel)
