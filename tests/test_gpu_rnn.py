"""LSTM / GRU on the device: the fused sequence ops and the adding-problem training step.

* op level: the reference's own outputs and every gradient (``rnn_ops.npz``), fp32 at 1e-4
  and float64 at 1e-10;
* model level: two AdamW steps of the adding-problem regressors against the reference
  fixture, and one step at the LSTM/GRU configuration (T = 100, batch 512, hidden 512)
  against the float64 oracle.
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import ops as O
from oracle import rnn as ornn
from tests.conftest import assert_parity, assert_update_parity, ill_conditioned, load_golden
from tests.golden.specs import RNN_CASES, RNN_SMALL, rnn_inputs

pytestmark = pytest.mark.gpu

REL = {np.float32: 1e-4, np.float64: 1e-10}


@pytest.mark.parametrize("dtype", [np.float32, np.float64], ids=["fp32", "fp64"])
@pytest.mark.parametrize("case", range(len(RNN_CASES)))
def test_recurrent_ops_match_reference_fixture(case, dtype):
    import tensorgrad_b200 as tg

    gold = load_golden("rnn_ops.npz")
    cell, steps, batch, inputs, hidden, seed = RNN_CASES[case]
    x, h0, c0, w_ih, w_hh, b_ih, b_hh, rng = rnn_inputs(cell, steps, batch, inputs, hidden, seed)
    arrays = [x, h0] + ([c0] if cell == "lstm" else []) + [w_ih, w_hh, b_ih, b_hh]
    ts = [tg.Tensor(a.astype(dtype), requires_grad=True) for a in arrays]
    y = (tg.ops.lstm if cell == "lstm" else tg.ops.gru)(*ts)
    g = rng.standard_normal(y.shape)
    grads = tg.autograd.grad(y, ts, grad_outputs=g.astype(dtype))
    rel = REL[dtype]
    assert_parity(y.numpy(), gold[f"{cell}{case}/out"], rel, f"{cell}{case} out")
    names = ["dx", "dh0"] + (["dc0"] if cell == "lstm" else []) + [
        "dw_ih", "dw_hh", "db_ih", "db_hh"]
    for name, gr in zip(names, grads, strict=True):
        assert_parity(gr.numpy(), gold[f"{cell}{case}/{name}"], rel, f"{cell}{case} {name}")


def regressor(cell: str, hidden: int):
    """The adding-problem model (examples/adding_problem.py:71-81 of the reference)."""
    import tensorgrad_b200 as tg

    class Regressor(tg.nn.Module):
        def __init__(self) -> None:
            super().__init__()
            self.rnn = (tg.nn.LSTM if cell == "lstm" else tg.nn.GRU)(2, hidden)
            self.head = tg.nn.Linear(hidden, 1)

        def forward(self, x):
            output, _ = self.rnn(x)
            return self.head(output[-1])

    return Regressor()


def run_regressor(cfg: ornn.Config, batch: int, seed: int, steps: int, dtype):
    import tensorgrad_b200 as tg

    tg.set_default_dtype(dtype)
    try:
        tg.manual_seed(0)
        model = regressor(cfg.cell, cfg.hidden)
        model.load_state_dict(ornn.init_params(cfg, seed))
        names = [n for n, _ in model.named_parameters()]
        assert names == [n for n, _ in ornn.param_shapes(cfg)]
        params = list(model.parameters())
        opt = tg.optim.AdamW(params, lr=3e-4, betas=(0.9, 0.999), eps=1e-8, weight_decay=1e-4)
        recs = []
        for step in range(1, steps + 1):
            x, y = ornn.synthetic_batch(cfg, batch, seed + step)
            loss = tg.mse_loss(model(tg.Tensor(x.astype(dtype))), y.astype(dtype))
            opt.zero_grad()
            loss.backward()
            rec = {"loss": float(loss.item()),
                   "grads": {n: p.grad.numpy() for n, p in zip(names, params, strict=True)},
                   "before": {n: p.numpy() for n, p in zip(names, params, strict=True)}}
            opt.step()
            rec["params"] = {n: p.numpy() for n, p in zip(names, params, strict=True)}
            recs.append(rec)
        return recs
    finally:
        tg.set_default_dtype(np.float32)


def check_steps(recs, refs, rel):
    ill: dict[str, np.ndarray] = {}
    for step, (rec, ref) in enumerate(zip(recs, refs, strict=True), start=1):
        assert rec["loss"] == pytest.approx(ref["loss"], rel=rel)
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


@pytest.mark.parametrize("dtype", [np.float32, np.float64], ids=["fp32", "fp64"])
@pytest.mark.parametrize("cell", ["lstm", "gru"])
def test_regressor_two_steps_match_reference_fixture(cell, dtype):
    gold = load_golden("rnn_small.npz")
    s = RNN_SMALL
    cfg = ornn.Config(cell=cell, hidden=s["hidden"], seq=s["seq"])
    recs = run_regressor(cfg, s["batch"], s["seed"], s["steps"], dtype)
    names = list(recs[0]["grads"])
    refs = [{"loss": float(gold[f"{cell}/step{k}/loss"]),
             "grads": {n: gold[f"{cell}/step{k}/grad/{n}"] for n in names},
             "params": {n: gold[f"{cell}/step{k}/param/{n}"] for n in names}}
            for k in range(1, s["steps"] + 1)]
    check_steps(recs, refs, REL[dtype])


@pytest.mark.parametrize("cell", ["lstm", "gru"])
def test_recurrent_config_step_matches_oracle(cell):
    # The LSTM / GRU configuration: 100 steps, batch 512, hidden 512, input 2.
    # Every fp32 product of the step runs on the tensor cores, or (the input projection from
    # 2 inputs) on the small-k kernel: none falls back to the CUDA-core GEMM.
    from tensorgrad_b200._lib import lib

    cfg = ornn.Config(cell=cell)
    seed, batch = 9, 512
    before = lib.tg_gemm_fallback_count()
    recs = run_regressor(cfg, batch, seed, 1, np.float32)
    assert lib.tg_gemm_fallback_count() == before
    x, y = ornn.synthetic_batch(cfg, batch, seed + 1)
    ref = ornn.train_step(ornn.init_params(cfg, seed), cfg, x, y)
    check_steps(recs, [ref], 1e-4)
