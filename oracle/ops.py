"""Float64 NumPy restatement of the reference's per-op forward and VJP arithmetic.

Test infrastructure only (the checker): imported by ``tests/``, ``__graft_entry__.smoke()``
and ``bench.py``'s CPU legs, never by the product package. Every function names the
reference function it restates (``file:line`` inside the tensorgrad 0.2.0 project). The
arithmetic follows the reference step by step so float64 results agree with it to rounding.
"""

from __future__ import annotations

import math

import numpy as np

GELU_C = math.sqrt(2.0 / math.pi)
GELU_A = 0.044715


# ---------------------------------------------------------------------------- linear
def linear_forward(x: np.ndarray, w: np.ndarray, b: np.ndarray | None) -> np.ndarray:
    """``x @ w.T + b`` over flattened leading axes (ops/layers.py:22-42)."""
    x2 = x.reshape(-1, w.shape[1])
    out = x2 @ w.T
    if b is not None:
        out = out + b
    return out.reshape(*x.shape[:-1], w.shape[0])


def linear_backward(
    g: np.ndarray, x: np.ndarray, w: np.ndarray, has_bias: bool
) -> tuple[np.ndarray, np.ndarray, np.ndarray | None]:
    """``(gx, gw, gb)`` = ``(G W, G^T X, sum_rows G)`` (ops/layers.py:43-49)."""
    g2 = g.reshape(-1, g.shape[-1])
    x2 = x.reshape(-1, w.shape[1])
    gx = (g2 @ w).reshape(x.shape)
    gw = g2.T @ x2
    gb = g2.sum(axis=0) if has_bias else None
    return gx, gw, gb


# ---------------------------------------------------------------------------- layer norm
def layer_norm_forward(
    x: np.ndarray, w: np.ndarray | None, b: np.ndarray | None, eps: float = 1e-5
) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """``(out, xhat, rstd)``: biased variance over the last axis (ops/layers.py:65-87)."""
    xc = x - x.mean(axis=-1, keepdims=True)
    rstd = 1.0 / np.sqrt((xc * xc).mean(axis=-1, keepdims=True) + eps)
    xhat = xc * rstd
    out = xhat if w is None else xhat * w
    if b is not None:
        out = out + b
    return out, xhat, rstd


def layer_norm_backward(
    g: np.ndarray, xhat: np.ndarray, rstd: np.ndarray, w: np.ndarray | None
) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """``(gx, gw, gb)`` with ``gx = rstd (gh - mean(gh) - xhat mean(gh xhat))``, ``gh = g w``
    (ops/layers.py:98-117)."""
    lead = tuple(range(g.ndim - 1))
    gw = (g * xhat).sum(axis=lead)
    gb = g.sum(axis=lead)
    gh = g * w if w is not None else g.copy()
    mean_ghx = (gh * xhat).mean(axis=-1, keepdims=True)
    gx = rstd * (gh - gh.mean(axis=-1, keepdims=True) - xhat * mean_ghx)
    return gx, gw, gb


# ---------------------------------------------------------------------------- pointwise
def gelu_forward(x: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """``(out, t)``: tanh-approximate GELU and its saved ``t = tanh(...)``
    (ops/elementwise.py:275-295)."""
    t = np.tanh(GELU_C * x * (1.0 + GELU_A * x * x))
    return 0.5 * x * (1.0 + t), t


def gelu_backward(g: np.ndarray, x: np.ndarray, t: np.ndarray) -> np.ndarray:
    """``g * (0.5 (1 + t) + 0.5 x (1 - t^2) c (1 + 3 a x^2))`` (ops/elementwise.py:297-312)."""
    d = GELU_C + 3 * GELU_A * GELU_C * x * x
    return g * (0.5 * ((1.0 - t * t) * d * x + t + 1.0))


def relu_forward(x: np.ndarray) -> np.ndarray:
    """``max(x, 0)`` (ops/elementwise.py:255-268)."""
    return np.maximum(x, 0)


def relu_backward(g: np.ndarray, x: np.ndarray) -> np.ndarray:
    """``g * (x > 0)``: the gradient is 0 at exactly 0 (ops/elementwise.py:261-262)."""
    return g * (x > 0)


def unbroadcast(grad: np.ndarray, shape: tuple[int, ...]) -> np.ndarray:
    """Sum ``grad`` down to ``shape``, the adjoint of broadcasting (ops/_util.py:49-63)."""
    if grad.shape == shape:
        return grad
    extra = grad.ndim - len(shape)
    if extra > 0:
        grad = grad.sum(axis=tuple(range(extra)))
    stretched = tuple(i for i, n in enumerate(shape) if n == 1 and grad.shape[i] != 1)
    if stretched:
        grad = grad.sum(axis=stretched, keepdims=True)
    return grad.reshape(shape)


# ---------------------------------------------------------------------------- embedding
def embedding_forward(ids: np.ndarray, w: np.ndarray) -> np.ndarray:
    """Row gather ``w[ids]`` after the range check (ops/layers.py:209-224)."""
    if ids.size and (ids.min() < 0 or ids.max() >= w.shape[0]):
        raise IndexError("embedding ids out of range")
    return w[ids]


def embedding_backward(ids: np.ndarray, g: np.ndarray, num: int) -> np.ndarray:
    """Scatter-add of gradient rows, ``numpy.add.at`` semantics (ops/layers.py:192-206, 226)."""
    out = np.zeros((num, g.shape[-1]), dtype=g.dtype)
    np.add.at(out, ids.reshape(-1), g.reshape(-1, g.shape[-1]))
    return out


# ---------------------------------------------------------------------------- attention
def causal_forbidden(q_len: int, k_len: int) -> np.ndarray:
    """``True`` where attention is forbidden: key ``j > i + (k_len - q_len)``
    (ops/attention.py:40-49)."""
    return np.triu(np.ones((q_len, k_len), dtype=np.bool_), k=1 + k_len - q_len)


def keep_mask(shape: tuple[int, ...], p: float,
              rng: np.random.Generator) -> tuple[np.ndarray, float]:
    """The reference's dropout keep-mask (_random.py:53-70): threshold ``t = round(p 2^16)``;
    16-bit words from ``random_raw(ceil(n / 4))`` viewed as uint16; keep where ``word >= t``;
    survivors scale by ``2^16 / (2^16 - t)``; all dropped (no draw) when ``t >= 2^16``."""
    t = round(p * 65536)
    if t >= 65536:
        return np.zeros(shape, dtype=np.bool_), 0.0
    n = int(np.prod(shape))
    words = rng.bit_generator.random_raw((n + 3) // 4).view(np.uint16)[:n]
    return (words >= t).reshape(shape), 65536.0 / (65536 - t)


def attention_forward(
    q: np.ndarray, k: np.ndarray, v: np.ndarray, causal: bool,
    keep: np.ndarray | None = None, keep_scale: float = 1.0,
) -> tuple[np.ndarray, np.ndarray]:
    """``(out, probs)`` of ``softmax(q k^T / sqrt(d) + mask) v`` (ops/attention.py:71-88);
    with a dropout ``keep`` mask the weights are ``probs * keep * keep_scale``."""
    scale = 1.0 / math.sqrt(q.shape[-1])
    s = (q @ np.swapaxes(k, -1, -2)) * scale
    if causal:
        s = np.where(causal_forbidden(q.shape[-2], k.shape[-2]), -np.inf, s)
    m = s.max(axis=-1, keepdims=True)
    m = np.where(np.isfinite(m), m, 0.0)
    p = np.exp(s - m)
    p /= p.sum(axis=-1, keepdims=True)
    w = p if keep is None else p * keep * keep_scale
    return w @ v, p


def attention_backward(
    g: np.ndarray, q: np.ndarray, k: np.ndarray, v: np.ndarray, p: np.ndarray,
    keep: np.ndarray | None = None, keep_scale: float = 1.0,
) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """``(dq, dk, dv)``: ``dV = W^T g`` (``W`` the dropped-out weights), ``dP' = g V^T``
    masked like ``W``, ``dS = P (dP' - rowsum(dP' P)) / sqrt(d)``, ``dQ = dS K``,
    ``dK = dS^T Q`` (ops/attention.py:91-116)."""
    scale = 1.0 / math.sqrt(q.shape[-1])
    w = p if keep is None else p * keep * keep_scale
    dv = np.swapaxes(w, -1, -2) @ g
    ds = g @ np.swapaxes(v, -1, -2)
    if keep is not None:
        ds = ds * keep * keep_scale
    ds = (ds - (ds * p).sum(axis=-1, keepdims=True)) * p * scale
    return ds @ k, np.swapaxes(ds, -1, -2) @ q, dv


def split_heads(qkv: np.ndarray, num_heads: int) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """``(B, H, T, hd)`` views of Q, K, V in a packed ``(B, T, 3 H hd)`` array
    (ops/attention.py:216-220)."""
    b, t, d3 = qkv.shape
    parts = qkv.reshape(b, t, 3, num_heads, d3 // (3 * num_heads))
    return tuple(parts[:, :, i].transpose(0, 2, 1, 3) for i in range(3))  # type: ignore[return-value]


def packed_self_attention_forward(
    qkv: np.ndarray, num_heads: int, causal: bool = True
) -> tuple[np.ndarray, np.ndarray]:
    """Merged-head output ``(B, T, D)`` and the probabilities (ops/attention.py:223-252)."""
    b, t, d3 = qkv.shape
    q, k, v = split_heads(qkv, num_heads)
    y, p = attention_forward(q, k, v, causal)
    return y.transpose(0, 2, 1, 3).reshape(b, t, d3 // 3), p


def packed_self_attention_backward(
    g: np.ndarray, qkv: np.ndarray, p: np.ndarray, num_heads: int
) -> np.ndarray:
    """Packed ``(B, T, 3D)`` gradient (ops/attention.py:254-260)."""
    b, t, d3 = qkv.shape
    hd = d3 // (3 * num_heads)
    q, k, v = split_heads(qkv, num_heads)
    gy = g.reshape(b, t, num_heads, hd).transpose(0, 2, 1, 3)
    grads = attention_backward(gy, q, k, v, p)
    out = np.empty((b, t, 3, num_heads, hd), dtype=g.dtype)
    for i, gr in enumerate(grads):
        out[:, :, i] = gr.transpose(0, 2, 1, 3)
    return out.reshape(b, t, d3)


# ---------------------------------------------------------------------------- losses
def log_softmax(x: np.ndarray, axis: int = -1) -> np.ndarray:
    """Shifted log-softmax (ops/activation.py:19-24, 48-52)."""
    m = x.max(axis=axis, keepdims=True)
    m = np.where(np.isfinite(m), m, 0.0)
    s = x - m
    return s - np.log(np.exp(s).sum(axis=axis, keepdims=True))


def cross_entropy_forward(
    logits: np.ndarray, target: np.ndarray, ignore_index: int = -100, reduction: str = "mean"
) -> tuple[np.ndarray, np.ndarray]:
    """``(loss, logp)``; class axis last, mean over non-ignored targets (ops/loss.py:23-66)."""
    c = logits.shape[-1]
    flat = logits.reshape(-1, c)
    t = target.reshape(-1)
    valid = t != ignore_index
    safe = np.where(valid, t, 0)
    if np.any((safe < 0) | (safe >= c)):
        raise IndexError(f"target out of range for {c} classes")
    logp = log_softmax(flat, axis=1)
    losses = np.where(valid, -logp[np.arange(t.size), safe], 0.0)
    n_valid = int(valid.sum())
    if reduction == "mean":
        return np.asarray(losses.sum() / max(n_valid, 1)), logp
    if reduction == "sum":
        return np.asarray(losses.sum()), logp
    return losses.reshape(target.shape), logp


def cross_entropy_backward(
    g: np.ndarray | float,
    logp: np.ndarray,
    target: np.ndarray,
    logits_shape: tuple[int, ...],
    ignore_index: int = -100,
    reduction: str = "mean",
) -> np.ndarray:
    """``(softmax - onehot) * valid * g / n_valid`` (ops/loss.py:70-80)."""
    t = target.reshape(-1)
    valid = t != ignore_index
    safe = np.where(valid, t, 0)
    grad = np.exp(logp)
    grad[np.arange(t.size), safe] -= 1.0
    grad *= valid[:, None]
    if reduction == "none":
        grad *= np.asarray(g).reshape(-1, 1)
    elif reduction == "mean":
        grad *= np.asarray(g) / max(int(valid.sum()), 1)
    else:
        grad *= np.asarray(g)
    return grad.reshape(logits_shape)


def mse_forward(pred: np.ndarray, target: np.ndarray) -> np.ndarray:
    """``mean((pred - target)**2)`` (ops/loss.py:148-161)."""
    return np.asarray(((pred - target) ** 2).mean())


def mse_backward(g: float, pred: np.ndarray, target: np.ndarray) -> np.ndarray:
    """Gradient of the composite ``mean(pow(sub(p, t), 2))`` with respect to ``pred``."""
    return g * 2.0 * (pred - target) / pred.size


# ---------------------------------------------------------------------------- optimiser
def clip_grad_norm(grads: list[np.ndarray], max_norm: float, eps: float = 1e-6) -> tuple[
    float, list[np.ndarray]
]:
    """Global L2 norm over all gradients (float64, ``math.fsum``) and the rescaled gradients
    when ``max_norm / (total + eps) < 1`` (optim/clip.py:15-31)."""
    total = math.sqrt(math.fsum(float(np.sum(np.square(g, dtype=np.float64))) for g in grads))
    scale = max_norm / (total + eps)
    if scale < 1.0:
        grads = [g * np.asarray(scale, dtype=g.dtype) for g in grads]
    return total, grads


def adamw_update(
    p: np.ndarray,
    g: np.ndarray,
    m: np.ndarray,
    v: np.ndarray,
    step: int,
    lr: float,
    betas: tuple[float, float],
    eps: float,
    weight_decay: float,
    decoupled: bool = True,
) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """One Adam/AdamW update in the reference's order of operations; returns ``(p, m, v)``
    for the ``step``-th update (1-based) (optim/adam.py:59-74, 77-94)."""
    b1, b2 = betas
    p, m, v = p.copy(), m.copy(), v.copy()
    if weight_decay:
        if decoupled:
            p *= 1.0 - lr * weight_decay
        else:
            g = g + weight_decay * p
    m *= b1
    m += (1.0 - b1) * g
    v *= b2
    v += (1.0 - b2) * g * g
    bc1 = 1.0 - b1**step
    bc2 = 1.0 - b2**step
    denom = np.sqrt(v) / math.sqrt(bc2) + eps
    p -= (lr / bc1) * m / denom
    return p, m, v


# ---------------------------------------------------------------------------- softmax family
def _row_shift(x: np.ndarray, axis: int) -> np.ndarray:
    m = x.max(axis=axis, keepdims=True)
    return np.where(np.isfinite(m), m, 0.0)


def softmax_forward(x: np.ndarray, axis: int = -1) -> np.ndarray:
    """``exp(x - m) / sum(exp(x - m))`` (ops/activation.py:27-45)."""
    e = np.exp(x - _row_shift(x, axis))
    return e / e.sum(axis=axis, keepdims=True)


def softmax_backward(g: np.ndarray, s: np.ndarray, axis: int = -1) -> np.ndarray:
    """``s (g - sum(g s))`` (ops/activation.py:36-37)."""
    return s * (g - (g * s).sum(axis=axis, keepdims=True))


def logsumexp_forward(x: np.ndarray, axis: int = -1) -> np.ndarray:
    """``log(sum(exp(x - m))) + m`` with the reduced axis kept (ops/activation.py:75-86)."""
    m = _row_shift(x, axis)
    return np.log(np.exp(x - m).sum(axis=axis, keepdims=True)) + m


def extremum_backward(g_kept: np.ndarray, x: np.ndarray, kept: np.ndarray,
                      axes: tuple[int, ...]) -> np.ndarray:
    """Tied extrema share the gradient equally (ops/reduce.py:78-85); ``g_kept`` and ``kept``
    have the reduced axes kept."""
    winners = (x == kept).astype(np.float64)
    return g_kept * winners / winners.sum(axis=axes, keepdims=True)


def bce_with_logits_forward(z: np.ndarray, y: np.ndarray) -> np.ndarray:
    """Per-element ``max(z, 0) - z y + log1p(exp(-|z|))`` (ops/loss.py:115-118)."""
    return np.maximum(z, 0.0) - z * y + np.log1p(np.exp(-np.abs(z)))


def bce_with_logits_backward(up: np.ndarray, z: np.ndarray,
                             y: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """``(sigmoid(z) - y) up`` and ``-z up`` (ops/loss.py:128-135)."""
    e = np.exp(-np.abs(z))
    sig = np.where(z >= 0, 1.0 / (1.0 + e), e / (1.0 + e))
    return (sig - y) * up, -z * up
