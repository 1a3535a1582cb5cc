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

from oracle import gpt as ogpt  # noqa: E402
from tests.golden.specs import ATTN_CASES, GPT_SMALL, attention_inputs  # noqa: E402

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


def main() -> None:
    np.savez_compressed(os.path.join(HERE, "gpt_small.npz"), **run_gpt(GPT_SMALL))
    np.savez_compressed(os.path.join(HERE, "attention.npz"), **run_attention())
    print("wrote", sorted(f for f in os.listdir(HERE) if f.endswith(".npz")))


if __name__ == "__main__":
    main()
