"""Generate the golden fixtures of ``tests/golden/`` by running the reference tensorgrad itself.

    PYTHONPATH=<the reference's src/ directory> python tests/golden/make_golden.py [name ...]

(with names, only those fixtures are rewritten, e.g. ``gpt_dropout dropout_masks``).

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
    ATTN_CASES, CNN_SMALL, CONV_CASES, DROPOUT_CASES, GPT_DROPOUT, GPT_SMALL, POOL_CASES,
    RNN_CASES, RNN_SMALL,
    attention_inputs, conv_inputs, pool_input, rnn_inputs,
)

def run_gpt(spec: dict) -> dict[str, np.ndarray]:
    cfg: ogpt.Config = spec["cfg"]
    tg.set_default_dtype(np.float64)
    tg.manual_seed(0)
    model = nn.GPT(nn.GPTConfig(vocab_size=cfg.vocab_size, block_size=cfg.block_size,
                                n_layer=cfg.n_layer, n_head=cfg.n_head, n_embd=cfg.n_embd,
                                dropout=spec.get("dropout", 0.0)))
    init = ogpt.init_params(cfg, spec["seed"])
    state = dict(init)
    state["head.weight"] = init["tok_emb.weight"]
    model.load_state_dict(state)
    if "reseed" in spec:  # the dropout masks then start from a known generator state
        tg.manual_seed(spec["reseed"])
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


def run_dropout_masks() -> dict[str, np.ndarray]:
    """The reference's keep_mask for seeded generators, and the generator's next raw draws
    after it (so the stream position after a mask is pinned too)."""
    from tensorgrad._random import keep_mask

    out: dict[str, np.ndarray] = {}
    for i, (shape, p, seed) in enumerate(DROPOUT_CASES):
        rng = np.random.default_rng(seed)
        rng.integers(0, 2**32, size=3, dtype=np.uint32)  # leaves a buffered 32-bit half
        keep, scale = keep_mask(shape, p, rng)
        out[f"case{i}/keep"] = keep
        out[f"case{i}/scale"] = np.asarray(scale)
        out[f"case{i}/next_u32"] = rng.integers(0, 2**32, size=3, dtype=np.uint32)
        out[f"case{i}/next_raw"] = rng.bit_generator.random_raw(2)
    return out


def write_checkpoint(path: str) -> None:
    """The reference's own checkpoint file: a freshly initialised GPT (manual_seed(7), so the
    weights also pin the initialisation order) saved with tensorgrad.utils.save."""
    cfg = GPT_SMALL["cfg"]
    tg.set_default_dtype(np.float64)
    tg.manual_seed(7)
    model = nn.GPT(nn.GPTConfig(vocab_size=cfg.vocab_size, block_size=cfg.block_size,
                                n_layer=cfg.n_layer, n_head=cfg.n_head, n_embd=cfg.n_embd))
    tg.utils.save(model, path)


def run_generate() -> dict[str, np.ndarray]:
    """KV-cache generation by the reference: a freshly initialised GPT (manual_seed(7), block
    16) extends a 5-token prompt by 20 tokens, greedily (top_k = 1) and by sampling at
    temperature 0.8 from a seeded generator; the window slides past the block after 11 new
    tokens, so both the cached and the re-encoded paths run. Also the logits of one
    full-window forward in evaluation mode."""
    cfg = GPT_SMALL["cfg"]
    tg.set_default_dtype(np.float64)
    tg.manual_seed(7)
    model = nn.GPT(nn.GPTConfig(vocab_size=cfg.vocab_size, block_size=cfg.block_size,
                                n_layer=cfg.n_layer, n_head=cfg.n_head, n_embd=cfg.n_embd))
    prompt = np.random.default_rng(17).integers(0, cfg.vocab_size, size=(2, 5))
    greedy = model.generate(prompt, 20, top_k=1, rng=np.random.default_rng(1))
    sampled = model.generate(prompt, 20, temperature=0.8, rng=np.random.default_rng(2))
    model.eval()
    logits = np.array(model(greedy[:, :cfg.block_size]).data)
    return {"prompt": prompt, "greedy": greedy, "sampled": sampled, "logits": logits}


def run_higher_order() -> dict[str, np.ndarray]:
    """Differentiable gradients by the reference (float64): func.grad / hessian / hvp / jvp /
    jacobian of small functions of elementwise, matrix and reduction ops, and a gradient
    penalty (backward through an input gradient built with create_graph) on a small MLP with
    cross entropy. Inputs regenerate from specs.higher_order_inputs."""
    from tensorgrad import func
    from tests.golden.specs import higher_order_inputs

    tg.set_default_dtype(np.float64)
    d = higher_order_inputs()
    x, w, v, vw = (tg.Tensor(d[k]) for k in ("x", "w", "v", "vw"))

    def f(x_, w_):
        return (tg.tanh(x_ @ w_) ** 2).sum()

    def g(x_):
        return tg.sigmoid(x_ @ tg.Tensor(d["w"])).reshape(-1)

    def h(x_):
        return tg.mean(tg.exp(x_) / (x_ * x_ + 1.0)) + tg.log(x_ * x_ + 1.0).sum() \
            + (tg.gelu(x_) * tg.Tensor(d["c"])).sum() + tg.sqrt(x_ * x_ + 2.0).sum()

    out: dict[str, np.ndarray] = {}
    gx, gw = func.grad(f, argnums=(0, 1))(x, w)
    out["grad_x"], out["grad_w"] = np.array(gx.data), np.array(gw.data)
    out["hess_x"] = np.array(func.hessian(f)(x, w).data)
    _, (hx, hw) = func.hvp(f, (x, w), (v, vw))
    out["hvp_x"], out["hvp_w"] = np.array(hx.data), np.array(hw.data)
    _, jv = func.jvp(g, (x,), (v,))
    out["jvp"] = np.array(jv.data)
    out["jac"] = np.array(func.jacobian(g)(x).data)
    out["hess_h"] = np.array(func.hessian(h)(x).data)
    # Gradient penalty on an MLP: loss + sum(d loss / d input)^2, backward to the weights.
    w1, b1, w2, b2 = (tg.Tensor(d[k], requires_grad=True) for k in ("w1", "b1", "w2", "b2"))
    xin = tg.Tensor(d["xin"], requires_grad=True)
    loss = tg.cross_entropy(tg.linear(tg.relu(tg.linear(xin, w1, b1)), w2, b2), d["labels"])
    (gin,) = tg.autograd.grad(loss, [xin], create_graph=True)
    total = loss + (gin * gin).sum()
    total.backward()
    out["penalty_total"] = np.asarray(total.item())
    for k, t in (("w1", w1), ("b1", b1), ("w2", w2), ("b2", b2), ("xin", xin)):
        out[f"penalty_grad_{k}"] = np.array(t.grad.data)
    return out


def run_higher_order_layers() -> dict[str, np.ndarray]:
    """Second derivatives through the fused layers by the reference (float64): Hessian-vector
    products of small functions of layer norm, variance, attention (with and without the
    causal mask and dropout, and the packed form), embedding + layer norm + cross entropy,
    LSTM, GRU and dropout; gradient penalties through conv2d, batch norm, ReLU and max
    pooling (overlapping 3 x 3 windows, and 2 x 2); and one GPT step on a gradient penalty
    with dropout 0.1. The programs are shared with the tests (specs.py)."""
    import types

    from tensorgrad import func
    from tensorgrad.ops import attention as ref_attention
    from tensorgrad.ops import layers as ref_layers
    from tensorgrad.ops import recurrent as ref_recurrent
    from tests.golden.specs import (
        GPT_PENALTY, gpt_penalty_program, higher_order_layer_inputs, higher_order_layer_program,
    )

    tg.set_default_dtype(np.float64)
    O = types.SimpleNamespace(
        tanh=tg.tanh, relu=tg.relu, layer_norm=tg.layer_norm, var=tg.var,
        sdpa=ref_attention.scaled_dot_product_attention,
        packed=ref_attention.packed_self_attention, conv2d=tg.conv2d,
        batch_norm=ref_layers.batch_norm, max_pool2d=tg.max_pool2d, embedding=tg.embedding,
        linear=tg.linear, cross_entropy=tg.cross_entropy, lstm=ref_recurrent.lstm,
        gru=ref_recurrent.gru, dropout=tg.dropout)

    def host(t):
        return np.array(t.data)

    out = higher_order_layer_program(tg, O, func, host, higher_order_layer_inputs())
    out.update(gpt_penalty_program(tg, nn, host, GPT_PENALTY))
    return out


def run_ops_extra() -> dict[str, np.ndarray]:
    """The remaining ops by the reference (float64): softmax family, max / min with ties,
    where / masked_fill, concat, binary cross entropy, Elman RNN, vector matmuls,
    comparisons, all / any / argmax (the program is shared with the tests, specs.py); and the
    batch order of a shuffled DataLoader."""
    import types

    from tensorgrad import ops as ref_ops
    from tensorgrad.utils import DataLoader
    from tests.golden.specs import ops_extra_inputs, ops_extra_program

    tg.set_default_dtype(np.float64)

    def host(t):
        return np.array(t.data)

    from tensorgrad.ops.attention import scaled_dot_product_attention

    O = types.SimpleNamespace(rnn=ref_ops.rnn, sdpa=scaled_dot_product_attention)
    out = ops_extra_program(tg, O, host, ops_extra_inputs())
    loader = DataLoader(np.arange(10), batch_size=4, shuffle=True, seed=5)
    for epoch in range(2):
        out[f"loader_epoch{epoch}"] = np.concatenate([np.array(b.data) for (b,) in loader])
    return out


def run_profiler_table() -> dict[str, np.ndarray]:
    """The reference profiler's table for fixed statistics (the text format users parse)."""
    from tensorgrad import profiler
    from tests.golden.specs import PROFILE_ROWS

    prof = profiler.Profile()
    for name, fc, fs, bc, bs in PROFILE_ROWS:
        prof.ops[name] = profiler.OpStats(fc, fs, bc, bs)
    prof.wall_seconds = 0.125
    return {"table": np.array(prof.table()), "table_limit2": np.array(prof.table(limit=2))}


def run_viz() -> dict[str, np.ndarray]:
    """The reference's graph drawings of two small graphs (the text format users render):
    ``sum((tanh(w @ x))**2)`` with named leaves, and a named intermediate under a quoted
    name."""
    from tensorgrad import viz

    tg.set_default_dtype(np.float64)
    w = tg.Tensor(np.ones((2, 3)), requires_grad=True)
    x = tg.Tensor(np.ones(3))
    y = tg.tanh(w @ x)
    loss = (y * y).sum()
    a = tg.Tensor([1.0, 2.0], requires_grad=True)
    hidden = tg.relu(a)
    out = hidden.sum()
    named = {'say "a"': a, "hidden": hidden}
    return {"mermaid_lr": np.array(viz.to_mermaid(loss, names={"w": w, "x": x}, direction="LR")),
            "dot_tb": np.array(viz.to_dot(loss, names={"w": w, "x": x})),
            "mermaid_named": np.array(viz.to_mermaid(out, names=named)),
            "dot_named": np.array(viz.to_dot(out, names=named))}


def main() -> None:
    jobs = {
        "gpt_small": lambda: run_gpt(GPT_SMALL),
        "attention": run_attention,
        "cnn_small": lambda: run_cnn(CNN_SMALL),
        "conv_pool": run_conv_pool,
        "rnn_ops": run_rnn_ops,
        "rnn_small": lambda: run_rnn_models(RNN_SMALL),
        "gpt_dropout": lambda: run_gpt(GPT_DROPOUT),
        "dropout_masks": run_dropout_masks,
        "gpt_generate": run_generate,
        "higher_order": run_higher_order,
        "higher_order_layers": run_higher_order_layers,
        "ops_extra": run_ops_extra,
        "profiler_table": run_profiler_table,
        "viz": run_viz,
    }
    names = sys.argv[1:] or [*jobs, "gpt_checkpoint"]
    for name in names:
        path = os.path.join(HERE, f"{name}.npz")
        if name == "gpt_checkpoint":
            write_checkpoint(path)
        else:
            np.savez_compressed(path, **jobs[name]())
    print("wrote", names)


if __name__ == "__main__":
    main()
