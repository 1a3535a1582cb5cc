"""Generate the golden fixtures of ``tests/golden/`` by running the reference tensorgrad itself.

    PYTHONPATH=/root/reference/src python tests/golden/make_golden.py

Run in the build container, where the reference is importable (it is pure Python + NumPy).
Everything runs in float64. Inputs are regenerated in the tests from the same seeds
(``oracle.gpt.init_params``, ``oracle.gpt.synthetic_batch`` and ``specs.attention_inputs``),
so the fixtures hold only the reference's outputs. The reference is driven through its
public API exactly as a training script does: ``nn.GPT``, ``tg.cross_entropy``,
``loss.backward()``, ``optim.clip_grad_norm_``, ``optim.AdamW.step()``,
``nn.functional.scaled_dot_product_attention`` with ``autograd.grad``.
"""

from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))  # the repo root, for ``oracle``

import tensorgrad as tg  # noqa: E402  (the reference, from PYTHONPATH)
from tensorgrad import nn, optim  # noqa: E402

from oracle import cnn as ocnn  # noqa: E402
from oracle import rnn as ornn  # noqa: E402
from oracle import gpt as ogpt  # noqa: E402
from tests.golden.specs import (  # noqa: E402
    ATTN_CASES, CNN_SMALL, CONV_CASES, GPT_SMALL, POOL_CASES, RNN_CASES, RNN_SMALL,
    attention_inputs, conv_inputs, pool_input, rnn_inputs,
)

def run_gpt(spec: dict) -> dict[str, np.ndarray]:
    cfg: ogpt.Config = spec["cfg"]
    tg.set_default_dtype(np.float64)
    tg.manual_seed(0)
    model = nn.GPT(nn.GPTConfig(vocab_size=cfg.vocab_size, block_size=cfg.block_size,
                                n_layer=cfg.n_layer, n_head=cfg.n_head, n_embd=cfg.n_embd,
                                dropout=0.0))
    init = ogpt.init_params(cfg, spec["seed"])
    state = dict(init)
    state["head.weight"] = init["tok_emb.weight"]
    model.load_state_dict(state)
    params = list(model.parameters())
    names = [n for n, _ in model.named_parameters()]
    assert names == [n for n, _ in ogpt.param_shapes(cfg)], names
    opt = optim.AdamW(params, lr=3e-4, betas=(0.9, 0.999), eps=1e-8, weight_decay=1e-4)
    out: dict[str, np.ndarray] = {}
    for step in range(1, spec["steps"] + 1):
        ids, targets = ogpt.synthetic_batch(cfg, spec["batch"], spec["seq"], spec["seed"] + step)
        loss = tg.cross_entropy(model(ids), targets)
        opt.zero_grad()
        loss.backward()
        total = optim.clip_grad_norm_(params, spec["max_norm"])
        out[f"step{step}/loss"] = np.asarray(loss.item())
        out[f"step{step}/total_norm"] = np.asarray(total)
        for n, p in zip(names, params, strict=True):
            out[f"step{step}/grad/{n}"] = np.array(p.grad.data)
        opt.step()
        for n, p in zip(names, params, strict=True):
            out[f"step{step}/param/{n}"] = np.array(p.data)
    return out


def run_attention() -> dict[str, np.ndarray]:
    tg.set_default_dtype(np.float64)
    out: dict[str, np.ndarray] = {}
    for shape, causal, seed in ATTN_CASES:
        q, k, v, do = attention_inputs(shape, seed)
        tq, tk, tv = (tg.Tensor(a, requires_grad=True) for a in (q, k, v))
        o = nn.functional.scaled_dot_product_attention(tq, tk, tv, causal=causal)
        dq, dk, dv = tg.autograd.grad(o, [tq, tk, tv], grad_outputs=do)
        key = "x".join(map(str, shape)) + ("_causal" if causal else "")
        out[f"{key}/out"] = np.array(o.data)
        out[f"{key}/dq"], out[f"{key}/dk"], out[f"{key}/dv"] = (
            np.array(g.data) for g in (dq, dk, dv)
        )
    return out


def cnn_model(cfg: ocnn.Config) -> nn.Sequential:
    """The CNN configuration's layer stack (Conv-BN-ReLU-Pool twice, Flatten, Linear)."""
    return nn.Sequential(
        nn.Conv2d(cfg.in_channels, cfg.c1, 3, padding=1), nn.BatchNorm2d(cfg.c1), nn.ReLU(),
        nn.MaxPool2d(2), nn.Conv2d(cfg.c1, cfg.c2, 3, padding=1), nn.BatchNorm2d(cfg.c2),
        nn.ReLU(), nn.MaxPool2d(2), nn.Flatten(), nn.Linear(cfg.c2 * (cfg.size // 4) ** 2,
                                                            cfg.classes),
    )


def run_cnn(spec: dict) -> dict[str, np.ndarray]:
    cfg: ocnn.Config = spec["cfg"]
    tg.set_default_dtype(np.float64)
    tg.manual_seed(0)
    model = cnn_model(cfg)
    model.load_state_dict(ocnn.init_params(cfg, spec["seed"]) | ocnn.init_buffers(cfg))
    params = list(model.parameters())
    names = [n for n, _ in model.named_parameters()]
    assert names == [n for n, _ in ocnn.param_shapes(cfg)], names
    opt = optim.AdamW(params, lr=3e-4, betas=(0.9, 0.999), eps=1e-8, weight_decay=1e-4)
    out: dict[str, np.ndarray] = {}
    for step in range(1, spec["steps"] + 1):
        x, labels = ocnn.synthetic_batch(cfg, spec["batch"], spec["seed"] + step)
        loss = tg.cross_entropy(model(tg.Tensor(x)), labels)
        opt.zero_grad()
        loss.backward()
        out[f"step{step}/loss"] = np.asarray(loss.item())
        for n, p in zip(names, params, strict=True):
            out[f"step{step}/grad/{n}"] = np.array(p.grad.data)
        opt.step()
        for n, p in zip(names, params, strict=True):
            out[f"step{step}/param/{n}"] = np.array(p.data)
        for n, b in model.named_buffers():
            out[f"step{step}/buffer/{n}"] = np.array(b)
    return out


def run_conv_pool() -> dict[str, np.ndarray]:
    tg.set_default_dtype(np.float64)
    out: dict[str, np.ndarray] = {}
    for i, (x_shape, wspec, stride, padding, seed) in enumerate(CONV_CASES):
        x, w, b, rng = conv_inputs(x_shape, wspec, seed)
        tx, tw, tb = (tg.Tensor(a, requires_grad=True) for a in (x, w, b))
        y = tg.conv2d(tx, tw, tb, stride=stride, padding=padding)
        g = rng.standard_normal(y.shape)
        gx, gw, gb = tg.autograd.grad(y, [tx, tw, tb], grad_outputs=g)
        out[f"conv{i}/y"] = np.array(y.data)
        out[f"conv{i}/gx"], out[f"conv{i}/gw"], out[f"conv{i}/gb"] = (
            np.array(t.data) for t in (gx, gw, gb))
    for i, (x_shape, kernel, stride, padding, seed) in enumerate(POOL_CASES):
        x, rng = pool_input(x_shape, seed)
        tx = tg.Tensor(x, requires_grad=True)
        y = tg.max_pool2d(tx, kernel, stride, padding)
        g = rng.standard_normal(y.shape)
        (gx,) = tg.autograd.grad(y, [tx], grad_outputs=g)
        out[f"pool{i}/y"] = np.array(y.data)
        out[f"pool{i}/gx"] = np.array(gx.data)
    return out


def run_rnn_ops() -> dict[str, np.ndarray]:
    tg.set_default_dtype(np.float64)
    out: dict[str, np.ndarray] = {}
    for i, (cell, steps, batch, inputs, hidden, seed) in enumerate(RNN_CASES):
        x, h0, c0, w_ih, w_hh, b_ih, b_hh, rng = rnn_inputs(cell, steps, batch, inputs, hidden, seed)
        arrays = [x, h0] + ([c0] if cell == "lstm" else []) + [w_ih, w_hh, b_ih, b_hh]
        ts = [tg.Tensor(a, requires_grad=True) for a in arrays]
        y = (tg.ops.lstm if cell == "lstm" else tg.ops.gru)(*ts)
        g = rng.standard_normal(y.shape)
        grads = tg.autograd.grad(y, ts, grad_outputs=g)
        out[f"{cell}{i}/out"] = np.array(y.data)
        names = ["dx", "dh0"] + (["dc0"] if cell == "lstm" else []) + [
            "dw_ih", "dw_hh", "db_ih", "db_hh"]
        for name, gr in zip(names, grads, strict=True):
            out[f"{cell}{i}/{name}"] = np.array(gr.data)
    return out


class Regressor(nn.Module):
    """The adding-problem model: a recurrent layer read out by a linear map from its final
    hidden state (the reference's examples/adding_problem.py:71-81)."""

    def __init__(self, cell, hidden: int) -> None:
        super().__init__()
        self.rnn = cell(2, hidden)
        self.head = nn.Linear(hidden, 1)

    def forward(self, x):
        output, _ = self.rnn(x)
        return self.head(output[-1])


def run_rnn_models(spec: dict) -> dict[str, np.ndarray]:
    tg.set_default_dtype(np.float64)
    out: dict[str, np.ndarray] = {}
    for cell in ("lstm", "gru"):
        cfg = ornn.Config(cell=cell, hidden=spec["hidden"], seq=spec["seq"])
        tg.manual_seed(0)
        model = Regressor(nn.LSTM if cell == "lstm" else nn.GRU, spec["hidden"])
        model.load_state_dict(ornn.init_params(cfg, spec["seed"]))
        params = list(model.parameters())
        names = [n for n, _ in model.named_parameters()]
        assert names == [n for n, _ in ornn.param_shapes(cfg)], names
        opt = optim.AdamW(params, lr=3e-4, betas=(0.9, 0.999), eps=1e-8, weight_decay=1e-4)
        for step in range(1, spec["steps"] + 1):
            x, y = ornn.synthetic_batch(cfg, spec["batch"], spec["seed"] + step)
            loss = tg.mse_loss(model(tg.Tensor(x)), y)
            opt.zero_grad()
            loss.backward()
            out[f"{cell}/step{step}/loss"] = np.asarray(loss.item())
            for n, p in zip(names, params, strict=True):
                out[f"{cell}/step{step}/grad/{n}"] = np.array(p.grad.data)
            opt.step()
            for n, p in zip(names, params, strict=True):
                out[f"{cell}/step{step}/param/{n}"] = np.array(p.data)
    return out


def main() -> None:
    np.savez_compressed(os.path.join(HERE, "gpt_small.npz"), **run_gpt(GPT_SMALL))
    np.savez_compressed(os.path.join(HERE, "attention.npz"), **run_attention())
    np.savez_compressed(os.path.join(HERE, "cnn_small.npz"), **run_cnn(CNN_SMALL))
    np.savez_compressed(os.path.join(HERE, "conv_pool.npz"), **run_conv_pool())
    np.savez_compressed(os.path.join(HERE, "rnn_ops.npz"), **run_rnn_ops())
    np.savez_compressed(os.path.join(HERE, "rnn_small.npz"), **run_rnn_models(RNN_SMALL))
    print("wrote", sorted(f for f in os.listdir(HERE) if f.endswith(".npz")))


if __name__ == "__main__":
    main()
