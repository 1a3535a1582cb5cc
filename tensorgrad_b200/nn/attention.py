"""Multi-head self-attention (the reference's nn/attention.py:40-111, training path)."""

from __future__ import annotations

from tensorgrad_b200.nn.layers import Dropout, Linear
from tensorgrad_b200.nn.module import Module
from tensorgrad_b200.ops.attention import (
    causal_mask, packed_self_attention, scaled_dot_product_attention,
)
from tensorgrad_b200.tensor import Tensor

__all__ = ["MultiHeadAttention", "causal_mask", "scaled_dot_product_attention"]


class MultiHeadAttention(Module):
    """Fused QKV projection, packed attention, output projection (nn/attention.py:73-91)."""

    def __init__(self, embed_dim: int, num_heads: int, dropout: float = 0.0,
                 causal: bool = True, bias: bool = True) -> None:
        super().__init__()
        if embed_dim % num_heads:
            raise ValueError(f"embed_dim {embed_dim} is not divisible by num_heads {num_heads}")
        self.embed_dim = embed_dim
        self.num_heads = num_heads
        self.head_dim = embed_dim // num_heads
        self.causal = causal
        self.dropout = dropout
        self.qkv = Linear(embed_dim, 3 * embed_dim, bias=bias)
        self.proj = Linear(embed_dim, embed_dim, bias=bias)
        self.resid_dropout = Dropout(dropout)

    def forward(self, x: Tensor, cache: object = None) -> Tensor:
        if x.ndim != 3 or x.shape[-1] != self.embed_dim:
            raise ValueError(f"expected (B, T, {self.embed_dim}) input, got {x.shape}")
        if cache is not None:
            raise NotImplementedError("KV-cache inference is not on the device training path")
        y = packed_self_attention(self.qkv(x), self.num_heads, causal=self.causal,
                                  dropout_p=self.dropout, training=self.training)
        return self.resid_dropout(self.proj(y))

    def extra_repr(self) -> str:
        return f"embed_dim={self.embed_dim}, num_heads={self.num_heads}, causal={self.causal}"
