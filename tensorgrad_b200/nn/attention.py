"""Multi-head self-attention with a device KV cache (API of the reference's
nn/attention.py:27-111).

Training goes through the fused packed-QKV op (one graph node from the ``(B, T, 3D)``
projection to merged heads). Inference with a :class:`LayerCache` keeps every layer's keys
and values in preallocated device buffers ``(B, H, capacity, head_dim)``: a step copies the
new positions' keys and values out of the packed projection into the buffers (one strided
copy each) and runs the attention kernel on the cached prefix in place, the new queries
seeing every earlier key (``j <= i + start``).
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from tensorgrad_b200 import device
from tensorgrad_b200._lib import AttnShape, check, lib
from tensorgrad_b200.autograd import no_grad
from tensorgrad_b200.device import DeviceArray, dtype_code
from tensorgrad_b200.nn.layers import Dropout, Linear
from tensorgrad_b200.nn.module import Module
from tensorgrad_b200.ops.attention import (
    causal_mask, packed_self_attention, scaled_dot_product_attention,
)
from tensorgrad_b200.ops.shape import strided_copy
from tensorgrad_b200.tensor import Tensor

__all__ = ["LayerCache", "MultiHeadAttention", "causal_mask", "scaled_dot_product_attention"]


@dataclass
class LayerCache:
    """One layer's cached keys and values: ``(B, H, capacity, head_dim)`` device buffers of
    which the first ``length`` positions are filled (see ``GPT.make_cache``)."""

    keys: DeviceArray
    values: DeviceArray
    length: int = 0

    @classmethod
    def empty(cls, batch: int, heads: int, capacity: int, head_dim: int,
              dtype: np.dtype) -> LayerCache:
        shape = (batch, heads, capacity, head_dim)
        return cls(device.empty(shape, dtype), device.empty(shape, dtype))


class MultiHeadAttention(Module):
    """Self-attention over ``(B, T, D)`` with a fused QKV projection, ``num_heads`` heads of
    ``D / num_heads`` features, dropout on the weights and after the output projection."""

    def __init__(self, embed_dim: int, num_heads: int, dropout: float = 0.0,
                 causal: bool = True, bias: bool = True) -> None:
        super().__init__()
        if embed_dim % num_heads:
            raise ValueError(f"embed_dim {embed_dim} is not divisible by num_heads {num_heads}")
        self.embed_dim, self.num_heads = embed_dim, num_heads
        self.head_dim = embed_dim // num_heads
        self.causal, self.dropout = causal, dropout
        self.qkv = Linear(embed_dim, 3 * embed_dim, bias=bias)
        self.proj = Linear(embed_dim, embed_dim, bias=bias)
        self.resid_dropout = Dropout(dropout)

    def forward(self, x: Tensor, cache: LayerCache | None = None) -> Tensor:
        if x.ndim != 3 or x.shape[-1] != self.embed_dim:
            raise ValueError(f"expected (B, T, {self.embed_dim}) input, got {x.shape}")
        if cache is not None:
            return self._attend_cached(x, cache)
        y = packed_self_attention(self.qkv(x), self.num_heads, causal=self.causal,
                                  dropout_p=self.dropout, training=self.training)
        return self.resid_dropout(self.proj(y))

    def _attend_cached(self, x: Tensor, cache: LayerCache) -> Tensor:
        b, t, d = x.shape
        h, hd = self.num_heads, self.head_dim
        cap = cache.keys.shape[2]
        start, end = cache.length, cache.length + t
        if end > cap:
            raise ValueError(f"KV cache holds {cap} positions; {end} requested")
        with no_grad():
            qkv = self.qkv(x).data  # (B, t, 3D)
            es = qkv.itemsize
            packed = [t * 3 * d, hd, 3 * d, 1]    # (b, h, position, feature) in the projection
            cached = [h * cap * hd, cap * hd, hd, 1]
            for part, buf in ((1, cache.keys), (2, cache.values)):
                strided_copy(qkv.ptr + part * d * es, packed, buf.ptr + start * hd * es, cached,
                             (b, h, t, hd), es)
            cache.length = end
            out = device.empty((b, t, d), qkv.dtype)
            lse = device.empty((b * h * t,), qkv.dtype)
            shape = AttnShape(b, h, t, end, hd, *packed[:3], *cached[:3], *cached[:3],
                              t * d, hd, d, 1 if self.causal else 0)
            code = dtype_code(qkv.dtype)
            scratch = device.scratch(lib.tg_attention_forward_scratch_bytes(code, shape))
            check(lib.tg_attention_forward(code, shape, qkv.ptr, cache.keys.ptr,
                                           cache.values.ptr, out.ptr, lse.ptr, scratch.ptr,
                                           device.stream()), "attention (KV cache)")
            return self.resid_dropout(self.proj(Tensor._wrap(out)))

    def extra_repr(self) -> str:
        return f"embed_dim={self.embed_dim}, num_heads={self.num_heads}, causal={self.causal}"
