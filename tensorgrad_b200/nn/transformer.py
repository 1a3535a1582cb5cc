"""Pre-LN transformer block and the GPT language model (the reference's nn/transformer.py)."""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Any

import numpy as np

from tensorgrad_b200 import device
from tensorgrad_b200.nn import init
from tensorgrad_b200.nn.attention import MultiHeadAttention
from tensorgrad_b200.nn.layers import GELU, Dropout, Embedding, LayerNorm, Linear, Sequential
from tensorgrad_b200.nn.module import Module
from tensorgrad_b200.tensor import Tensor

__all__ = ["GPT", "GPTConfig", "TransformerBlock"]


class TransformerBlock(Module):
    """``x + attn(ln1(x))`` then ``x + mlp(ln2(x))`` (nn/transformer.py:24-48)."""

    def __init__(self, embed_dim: int, num_heads: int, dropout: float = 0.0,
                 mlp_ratio: int = 4) -> None:
        super().__init__()
        self.ln1 = LayerNorm(embed_dim)
        self.attn = MultiHeadAttention(embed_dim, num_heads, dropout=dropout, causal=True)
        self.ln2 = LayerNorm(embed_dim)
        self.mlp = Sequential(
            Linear(embed_dim, mlp_ratio * embed_dim),
            GELU(),
            Linear(mlp_ratio * embed_dim, embed_dim),
            Dropout(dropout),
        )

    def forward(self, x: Tensor, cache: object = None) -> Tensor:
        x = x + self.attn(self.ln1(x), cache)
        return x + self.mlp(self.ln2(x))


@dataclass(frozen=True)
class GPTConfig:
    """Hyper-parameters of :class:`GPT` (nn/transformer.py:68-78)."""

    vocab_size: int
    block_size: int = 64
    n_layer: int = 4
    n_head: int = 4
    n_embd: int = 128
    dropout: float = 0.0
    tie_weights: bool = True


class GPT(Module):
    """Decoder-only transformer LM: token + position embeddings, pre-LN blocks, final LN and
    a (tied) linear head (nn/transformer.py:81-167). The head reuses the token-embedding
    parameter, so the engine sums both gradient contributions into it."""

    def __init__(self, config: GPTConfig) -> None:
        super().__init__()
        self.config = config
        self.tok_emb = Embedding(config.vocab_size, config.n_embd)
        self.pos_emb = Embedding(config.block_size, config.n_embd)
        self.drop = Dropout(config.dropout)
        self.blocks = Sequential(
            *(TransformerBlock(config.n_embd, config.n_head, config.dropout)
              for _ in range(config.n_layer))
        )
        self.ln_f = LayerNorm(config.n_embd)
        self.head = Linear(config.n_embd, config.vocab_size, bias=False)
        self._init_weights()
        if config.tie_weights:
            self.head.weight = self.tok_emb.weight
        self.gradient_checkpointing = False

    def _init_weights(self) -> None:
        # GPT-2 initialisation (nn/transformer.py:116-127): N(0, 0.02) everywhere, residual
        # output projections N(0, 0.02 / sqrt(2 n_layer)), zero biases.
        residual_std = 0.02 / math.sqrt(2 * self.config.n_layer)
        for name, module in self.named_modules():
            if isinstance(module, Linear):
                is_residual = name.endswith(("attn.proj", "mlp.2"))
                init.normal_(module.weight, 0.0, residual_std if is_residual else 0.02)
                if module.bias is not None:
                    init.zeros_(module.bias)
            elif isinstance(module, Embedding):
                init.normal_(module.weight, 0.0, 0.02)

    def forward(self, idx: Any, cache: object = None) -> Tensor:
        """Token ids ``(B, T)`` to logits ``(B, T, vocab_size)``. Host ids are checked on the
        host; ids in a device tensor stay on the device (checked there, see ``embedding``)."""
        if cache is not None:
            raise NotImplementedError("KV-cache inference is not on the device training path")
        tokens = idx if isinstance(idx, Tensor) else np.asarray(idx)
        if tokens.ndim != 2:
            raise ValueError(f"expected (B, T) token ids, got shape {tokens.shape}")
        t = tokens.shape[1]
        if t > self.config.block_size:
            raise ValueError(f"sequence length {t} exceeds block_size {self.config.block_size}")
        x = self.drop(self.tok_emb(tokens) + self.pos_emb(_positions(t)))
        for block in self.blocks:
            x = block(x)
        return self.head(self.ln_f(x))


_POSITIONS: dict[tuple[int, str], Tensor] = {}


def _positions(t: int) -> Tensor:
    """Positions 0..t-1 as a device tensor, uploaded once per length and device."""
    key = (t, str(device.current_device()))
    p = _POSITIONS.get(key)
    if p is None:
        p = _POSITIONS[key] = Tensor(np.arange(t, dtype=np.int64))
    return p
