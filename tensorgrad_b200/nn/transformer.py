"""Pre-LN transformer blocks and the GPT language model on the device, with KV-cache
generation (API of the reference's nn/transformer.py:24-220).

The model is a stack of ``x + attn(ln1(x))``, ``x + mlp(ln2(x))`` blocks between token +
position embeddings and a final LayerNorm and vocabulary head, the head sharing the token
embedding's parameter (the engine then sums both gradient contributions into it).
Initialisation is GPT-2's, drawn from the global generator in the reference's order so a
seeded model starts from the reference's weights. Generation keeps per-layer keys and values
on the device (``nn.attention.LayerCache``), so a new token costs one position per layer;
only the last position's logits come back to the host for sampling.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Any

import numpy as np

from tensorgrad_b200 import device
from tensorgrad_b200._random import get_rng
from tensorgrad_b200.autograd import is_grad_enabled, no_grad
from tensorgrad_b200.nn.attention import LayerCache, MultiHeadAttention
from tensorgrad_b200.nn.layers import GELU, Dropout, Embedding, LayerNorm, Linear, Sequential
from tensorgrad_b200.nn.module import Module
from tensorgrad_b200.tensor import Tensor
from tensorgrad_b200.utils.grad_checkpoint import checkpoint

__all__ = ["GPT", "GPTConfig", "KVCache", "TransformerBlock"]


class TransformerBlock(Module):
    """Pre-LN block: ``x + attn(ln1(x))`` then ``x + mlp(ln2(x))``; the MLP is
    ``Linear(D, r D) -> GELU -> Linear(r D, D) -> Dropout``."""

    def __init__(self, embed_dim: int, num_heads: int, dropout: float = 0.0,
                 mlp_ratio: int = 4) -> None:
        super().__init__()
        hidden = mlp_ratio * embed_dim
        self.ln1 = LayerNorm(embed_dim)
        self.attn = MultiHeadAttention(embed_dim, num_heads, dropout=dropout, causal=True)
        self.ln2 = LayerNorm(embed_dim)
        self.mlp = Sequential(Linear(embed_dim, hidden), GELU(), Linear(hidden, embed_dim),
                              Dropout(dropout))

    def forward(self, x: Tensor, cache: LayerCache | None = None) -> Tensor:
        x = x + self.attn(self.ln1(x), cache)
        return x + self.mlp(self.ln2(x))


@dataclass
class KVCache:
    """Every layer's cached keys and values for the tokens a :class:`GPT` has processed."""

    layers: list[LayerCache]

    @property
    def length(self) -> int:
        """Positions already cached."""
        return self.layers[0].length if self.layers else 0


@dataclass(frozen=True)
class GPTConfig:
    """Hyper-parameters of :class:`GPT`."""

    vocab_size: int
    block_size: int = 64
    n_layer: int = 4
    n_head: int = 4
    n_embd: int = 128
    dropout: float = 0.0
    tie_weights: bool = True


_RESIDUAL_OUTPUTS = ("attn.proj", "mlp.2")


class GPT(Module):
    """Decoder-only transformer language model: ids ``(B, T)`` to logits ``(B, T, V)``.

    With :attr:`gradient_checkpointing` set, a training forward pass keeps only the residual
    stream between blocks and recomputes each block in the backward pass
    (``tensorgrad_b200.utils.checkpoint``; the reference's nn/transformer.py:155-159)."""

    gradient_checkpointing: bool

    def __init__(self, config: GPTConfig) -> None:
        super().__init__()
        self.config = config
        self.tok_emb = Embedding(config.vocab_size, config.n_embd)
        self.pos_emb = Embedding(config.block_size, config.n_embd)
        self.drop = Dropout(config.dropout)
        self.blocks = Sequential(*[TransformerBlock(config.n_embd, config.n_head, config.dropout)
                                   for _ in range(config.n_layer)])
        self.ln_f = LayerNorm(config.n_embd)
        self.head = Linear(config.n_embd, config.vocab_size, bias=False)
        self._gpt2_init()
        if config.tie_weights:
            self.head.weight = self.tok_emb.weight
        self.gradient_checkpointing = False

    def _gpt2_init(self) -> None:
        """N(0, 0.02) for every linear weight and embedding, N(0, 0.02 / sqrt(2 L)) for the
        projections that write into the residual stream, zero biases; drawn module by module
        in traversal order."""
        rng = get_rng()
        narrow = 0.02 / math.sqrt(2 * self.config.n_layer)
        for name, module in self.named_modules():
            if not isinstance(module, Linear | Embedding):
                continue
            std = narrow if (isinstance(module, Linear) and name.endswith(_RESIDUAL_OUTPUTS)) \
                else 0.02
            module.weight.data[...] = rng.normal(0.0, std, size=module.weight.shape)
            bias = getattr(module, "bias", None)
            if bias is not None:
                bias.data.fill_(0.0)

    # ------------------------------------------------------------------ forward
    def forward(self, idx: Any, cache: KVCache | None = None) -> Tensor:
        """Logits for token ids ``(B, T)``; with a ``cache``, ids continue the cached ones
        (positions from ``cache.length``; inference only, no graph). Host ids are checked
        on the host; ids in a device tensor stay on the device (checked there)."""
        tokens = idx if isinstance(idx, Tensor) else np.asarray(idx)
        if tokens.ndim != 2:
            raise ValueError(f"expected (B, T) token ids, got shape {tokens.shape}")
        start = cache.length if cache is not None else 0
        t = tokens.shape[1]
        if start + t > self.config.block_size:
            raise ValueError(f"sequence length {start + t} exceeds block_size "
                             f"{self.config.block_size}")
        if cache is None:
            x = self.drop(self.tok_emb(tokens) + self.pos_emb(_positions(0, t)))
            recompute = self.gradient_checkpointing and is_grad_enabled()
            for block in self.blocks:
                x = checkpoint(block, x) if recompute else block(x)
            return self.head(self.ln_f(x))
        if self.training:
            raise ValueError("a KV cache is for inference: call eval() first")
        with no_grad():
            x = self.tok_emb(tokens) + self.pos_emb(_positions(start, t))
            for block, layer in zip(self.blocks, cache.layers, strict=True):
                x = block(x, layer)
            return self.head(self.ln_f(x))

    # ------------------------------------------------------------------ generation
    def make_cache(self, batch_size: int) -> KVCache:
        """Empty per-layer device caches for ``batch_size`` sequences of ``block_size``."""
        dt = self.tok_emb.weight.dtype
        return KVCache([LayerCache.empty(batch_size, blk.attn.num_heads, self.config.block_size,
                                         blk.attn.head_dim, dt) for blk in self.blocks])

    def generate(self, idx: Any, max_new_tokens: int, *, temperature: float = 1.0,
                 top_k: int | None = None, rng: np.random.Generator | None = None,
                 use_cache: bool = True) -> np.ndarray:
        """Extend ids ``(B, T)`` by ``max_new_tokens`` sampled tokens (evaluation mode, no
        graph). The context is the last ``block_size`` tokens; ``top_k`` keeps the k most
        likely tokens; ``rng`` defaults to the global generator. With ``use_cache`` each new
        token is one position per layer against the device KV cache while the sequence fits
        in ``block_size``; once the window slides, the (absolute) positions shift and the
        window is encoded afresh, so both settings give the same tokens."""
        if temperature <= 0:
            raise ValueError("temperature must be positive")
        gen = rng or get_rng()
        was_training = self.training
        self.eval()
        out = np.asarray(idx, dtype=np.int64)
        window = self.config.block_size
        try:
            with no_grad():
                cache: KVCache | None = None
                for _ in range(max_new_tokens):
                    if not use_cache:
                        logits = self(out[:, -window:])
                    elif cache is not None and cache.length == out.shape[1] - 1:
                        logits = self(out[:, -1:], cache=cache)
                    else:
                        cache = self.make_cache(len(out))
                        logits = self(out[:, -window:], cache=cache)
                    if out.shape[1] >= window:
                        cache = None
                    last = _last_position(logits).astype(np.float64) / temperature
                    out = np.concatenate([out, _sample(last, top_k, gen)[:, None]], axis=1)
        finally:
            self.train(was_training)
        return out


def _last_position(logits: Tensor) -> np.ndarray:
    """The last position's logits ``(B, V)`` on the host (one small copy)."""
    b, t, v = logits.shape
    return logits.data.flat_view(0, b * t * v, (b, t, v)).numpy()[:, -1, :]


def _sample(logits: np.ndarray, top_k: int | None, gen: np.random.Generator) -> np.ndarray:
    """One token per row from ``softmax(logits)`` after an optional top-k cut, drawn as the
    reference does (a max-shifted softmax in float64, then ``Generator.choice``)."""
    if top_k is not None:
        kth = np.sort(logits, axis=-1)[:, -min(top_k, logits.shape[-1])]
        logits = np.where(logits < kth[:, None], -np.inf, logits)
    peak = logits.max(axis=-1, keepdims=True)
    e = np.exp(logits - np.where(np.isfinite(peak), peak, 0))
    probs = e / e.sum(axis=-1, keepdims=True)
    return np.array([gen.choice(probs.shape[-1], p=row) for row in probs])


_POSITIONS: dict[tuple[int, int, str], Tensor] = {}


def _positions(start: int, t: int) -> Tensor:
    """Positions ``start .. start + t - 1`` as a device tensor, uploaded once per range."""
    key = (start, t, str(device.current_device()))
    p = _POSITIONS.get(key)
    if p is None:
        if len(_POSITIONS) > 4096:
            _POSITIONS.clear()
        p = _POSITIONS[key] = Tensor(np.arange(start, start + t, dtype=np.int64))
    return p
