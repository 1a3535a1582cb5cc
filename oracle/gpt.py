"""Float64 NumPy restatement of one reference GPT training step (test infrastructure only).

The step is what the reference's ``benchmarks/train_step.py:86-104`` runs, with dropout 0:
``loss = cross_entropy(GPT(ids), targets)``; ``loss.backward()``; ``clip_grad_norm_``;
``AdamW.step()``. The model wiring follows ``nn/transformer.py:24-48, 97-167`` and
``nn/attention.py:84-91``; the op arithmetic is :mod:`oracle.ops`.

Parameters are a ``dict`` keyed by the reference's ``parameters()`` names in its order
(``nn/module.py:138-147``): the tied head weight is ``tok_emb.weight`` and appears once.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np

from oracle import ops


@dataclass(frozen=True)
class Config:
    """GPT hyper-parameters (``nn/transformer.py:68-78``; dropout 0, tied head)."""

    vocab_size: int
    block_size: int
    n_layer: int
    n_head: int
    n_embd: int


def param_shapes(cfg: Config) -> list[tuple[str, tuple[int, ...]]]:
    """``(name, shape)`` in ``GPT.parameters()`` order (tied head deduplicated)."""
    d, v = cfg.n_embd, cfg.vocab_size
    out: list[tuple[str, tuple[int, ...]]] = [
        ("tok_emb.weight", (v, d)),
        ("pos_emb.weight", (cfg.block_size, d)),
    ]
    for i in range(cfg.n_layer):
        p = f"blocks.{i}."
        out += [
            (p + "ln1.weight", (d,)),
            (p + "ln1.bias", (d,)),
            (p + "attn.qkv.weight", (3 * d, d)),
            (p + "attn.qkv.bias", (3 * d,)),
            (p + "attn.proj.weight", (d, d)),
            (p + "attn.proj.bias", (d,)),
            (p + "ln2.weight", (d,)),
            (p + "ln2.bias", (d,)),
            (p + "mlp.0.weight", (4 * d, d)),
            (p + "mlp.0.bias", (4 * d,)),
            (p + "mlp.2.weight", (d, 4 * d)),
            (p + "mlp.2.bias", (d,)),
        ]
    out += [("ln_f.weight", (d,)), ("ln_f.bias", (d,))]
    return out


def init_params(cfg: Config, seed: int) -> dict[str, np.ndarray]:
    """Seeded float64 weights with the reference's GPT-2 distributions
    (``nn/transformer.py:116-127``): N(0, 0.02), residual projections N(0, 0.02/sqrt(2L)),
    zero biases. LayerNorm scales are drawn near 1 and shifts near 0 (instead of exactly 1 and
    0) so that their gradients and updates are exercised by a parity check."""
    rng = np.random.default_rng(seed)
    resid = 0.02 / math.sqrt(2 * cfg.n_layer)
    params: dict[str, np.ndarray] = {}
    for name, shape in param_shapes(cfg):
        if name.endswith(("ln1.weight", "ln2.weight", "ln_f.weight")):
            params[name] = 1.0 + 0.1 * rng.standard_normal(shape)
        elif name.endswith(("ln1.bias", "ln2.bias", "ln_f.bias")):
            params[name] = 0.1 * rng.standard_normal(shape)
        elif name.endswith(".bias"):
            params[name] = 0.01 * rng.standard_normal(shape)
        elif name.endswith(("attn.proj.weight", "mlp.2.weight")):
            params[name] = resid * rng.standard_normal(shape)
        else:
            params[name] = 0.02 * rng.standard_normal(shape)
    return params


def forward_backward(
    params: dict[str, np.ndarray], ids: np.ndarray, targets: np.ndarray, cfg: Config
) -> tuple[float, dict[str, np.ndarray]]:
    """Loss and every parameter gradient of ``cross_entropy(GPT(ids), targets)``.

    Forward: ``nn/transformer.py:156-160``; blocks ``:45-47``; attention ``nn/attention.py:84-91``.
    Backward visits the ops in reverse, summing fan-out contributions (residual stream and
    the tied embedding) as the engine does (``autograd.py:315-324``).
    """
    b, t = ids.shape
    h = cfg.n_head
    p = params
    tok = ops.embedding_forward(ids, p["tok_emb.weight"])
    pos = ops.embedding_forward(np.arange(t), p["pos_emb.weight"])
    x = tok + pos
    saved = []
    for i in range(cfg.n_layer):
        q = f"blocks.{i}."
        a_in, xh1, r1 = ops.layer_norm_forward(x, p[q + "ln1.weight"], p[q + "ln1.bias"])
        qkv = ops.linear_forward(a_in, p[q + "attn.qkv.weight"], p[q + "attn.qkv.bias"])
        y, probs = ops.packed_self_attention_forward(qkv, h, causal=True)
        a_out = ops.linear_forward(y, p[q + "attn.proj.weight"], p[q + "attn.proj.bias"])
        x1 = x + a_out
        m_in, xh2, r2 = ops.layer_norm_forward(x1, p[q + "ln2.weight"], p[q + "ln2.bias"])
        f1 = ops.linear_forward(m_in, p[q + "mlp.0.weight"], p[q + "mlp.0.bias"])
        gl, tg = ops.gelu_forward(f1)
        f2 = ops.linear_forward(gl, p[q + "mlp.2.weight"], p[q + "mlp.2.bias"])
        saved.append((x, a_in, xh1, r1, qkv, y, probs, x1, m_in, xh2, r2, f1, gl, tg))
        x = x1 + f2
    lf, xhf, rf = ops.layer_norm_forward(x, p["ln_f.weight"], p["ln_f.bias"])
    logits = ops.linear_forward(lf, p["tok_emb.weight"], None)
    loss, logp = ops.cross_entropy_forward(logits, targets)

    grads: dict[str, np.ndarray] = {}
    dlogits = ops.cross_entropy_backward(1.0, logp, targets, logits.shape)
    dlf, dhead, _ = ops.linear_backward(dlogits, lf, p["tok_emb.weight"], False)
    dx, grads["ln_f.weight"], grads["ln_f.bias"] = ops.layer_norm_backward(
        dlf, xhf, rf, p["ln_f.weight"]
    )
    for i in reversed(range(cfg.n_layer)):
        q = f"blocks.{i}."
        (x0, a_in, xh1, r1, qkv, y, probs, x1, m_in, xh2, r2, f1, gl, tg) = saved[i]
        dgl, grads[q + "mlp.2.weight"], grads[q + "mlp.2.bias"] = ops.linear_backward(
            dx, gl, p[q + "mlp.2.weight"], True
        )
        df1 = ops.gelu_backward(dgl, f1, tg)
        dm_in, grads[q + "mlp.0.weight"], grads[q + "mlp.0.bias"] = ops.linear_backward(
            df1, m_in, p[q + "mlp.0.weight"], True
        )
        dx1_ln, grads[q + "ln2.weight"], grads[q + "ln2.bias"] = ops.layer_norm_backward(
            dm_in, xh2, r2, p[q + "ln2.weight"]
        )
        dx1 = dx + dx1_ln
        dy, grads[q + "attn.proj.weight"], grads[q + "attn.proj.bias"] = ops.linear_backward(
            dx1, y, p[q + "attn.proj.weight"], True
        )
        dqkv = ops.packed_self_attention_backward(dy, qkv, probs, h)
        da_in, grads[q + "attn.qkv.weight"], grads[q + "attn.qkv.bias"] = ops.linear_backward(
            dqkv, a_in, p[q + "attn.qkv.weight"], True
        )
        dx0_ln, grads[q + "ln1.weight"], grads[q + "ln1.bias"] = ops.layer_norm_backward(
            da_in, xh1, r1, p[q + "ln1.weight"]
        )
        dx = dx1 + dx0_ln
    grads["pos_emb.weight"] = ops.embedding_backward(
        np.arange(t), ops.unbroadcast(dx, (t, cfg.n_embd)), cfg.block_size
    )
    grads["tok_emb.weight"] = dhead + ops.embedding_backward(ids, dx, cfg.vocab_size)
    ordered = {name: grads[name] for name, _ in param_shapes(cfg)}
    return float(loss), ordered


@dataclass
class AdamWState:
    """Per-parameter moments and step counts (``optim/adam.py:38-42``)."""

    m: dict[str, np.ndarray]
    v: dict[str, np.ndarray]
    step: dict[str, int]


def train_step(
    params: dict[str, np.ndarray],
    ids: np.ndarray,
    targets: np.ndarray,
    cfg: Config,
    state: AdamWState | None = None,
    *,
    lr: float = 3e-4,
    betas: tuple[float, float] = (0.9, 0.999),
    eps: float = 1e-8,
    weight_decay: float = 1e-4,
    max_norm: float = 1.0,
) -> dict[str, object]:
    """One full step; returns loss, pre-clip norm, clipped grads, new params and state."""
    loss, grads = forward_backward(params, ids, targets, cfg)
    names = list(grads)
    total, clipped = ops.clip_grad_norm([grads[n] for n in names], max_norm)
    grads = dict(zip(names, clipped, strict=True))
    if state is None:
        state = AdamWState(
            {n: np.zeros_like(params[n]) for n in names},
            {n: np.zeros_like(params[n]) for n in names},
            {n: 0 for n in names},
        )
    new_params = {}
    for n in names:
        state.step[n] += 1
        new_params[n], state.m[n], state.v[n] = ops.adamw_update(
            params[n], grads[n], state.m[n], state.v[n], state.step[n], lr, betas, eps,
            weight_decay,
        )
    return {"loss": loss, "total_norm": total, "grads": grads, "params": new_params,
            "state": state}


def synthetic_batch(cfg: Config, batch: int, seq: int, seed: int) -> tuple[np.ndarray, np.ndarray]:
    """Token ids and next-token targets, uniform in ``[0, vocab)`` from ``seed``."""
    rng = np.random.default_rng(seed)
    ids = rng.integers(0, cfg.vocab_size, size=(batch, seq), dtype=np.int64)
    targets = rng.integers(0, cfg.vocab_size, size=(batch, seq), dtype=np.int64)
    return ids, targets


def step_flops(cfg: Config, batch: int, seq: int) -> float:
    """Algorithmic FLOPs of one forward+backward step: ``6 N (12 L d^2 + d V)`` for the
    matmuls plus ``6 N L T d`` for causal attention (half the ``T x T`` scores)."""
    n = batch * seq
    d, L = cfg.n_embd, cfg.n_layer
    return float(n * (6 * (12 * L * d * d + d * cfg.vocab_size) + 6 * L * seq * d))
