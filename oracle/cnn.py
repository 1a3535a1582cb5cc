"""Float64 NumPy restatement of the reference's CNN training step (test infrastructure only).

The model is ``nn.Sequential(Conv2d(3, c1, 3, padding=1), BatchNorm2d(c1), ReLU(),
MaxPool2d(2), Conv2d(c1, c2, 3, padding=1), BatchNorm2d(c2), ReLU(), MaxPool2d(2), Flatten(),
Linear(c2 * (s/4)^2, classes))`` in training mode; one step is ``cross_entropy`` ->
``loss.backward()`` -> ``AdamW.step()`` (no clipping). Op arithmetic:

* conv2d: im2col patch matrix, one GEMM each way, col2im scatter-add (ops/conv.py:53-177);
* batch_norm: the composite ``(x - mean) / sqrt(var + eps) * w + b`` with biased batch
  statistics, whose VJP the reference gets from the recorded primitives; restated here in
  closed form (ops/layers.py:144-189); running statistics with momentum and the unbiased
  variance (ops/layers.py:171-178);
* max_pool2d: running maximum over the window offsets, gradient to the first maximum in
  row-major order, NaN counting as the maximum (ops/conv.py:245-357);
* relu, linear, cross_entropy, AdamW: :mod:`oracle.ops`.

Parameter names follow ``Sequential``'s ``parameters()`` order (``nn/layers.py:279-308``):
``0.weight``, ``0.bias``, ``1.weight``, ... ``9.bias``; buffers ``1.running_mean`` etc.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from oracle import ops
from oracle.gpt import AdamWState


@dataclass(frozen=True)
class Config:
    """Input channels and side, the two conv widths and the class count."""

    in_channels: int = 3
    size: int = 64
    c1: int = 32
    c2: int = 64
    classes: int = 4


# ---------------------------------------------------------------------------- conv2d
def _pad(x: np.ndarray, ph: int, pw: int, value: float = 0.0) -> np.ndarray:
    if not (ph or pw):
        return x
    return np.pad(x, ((0, 0), (0, 0), (ph, ph), (pw, pw)), constant_values=value)


def im2col(x: np.ndarray, kh: int, kw: int, stride: tuple[int, int],
           padding: tuple[int, int]) -> tuple[np.ndarray, int, int]:
    """The ``(N*OH*OW, C*KH*KW)`` patch matrix of the zero-padded input (ops/conv.py:53-60,
    77-83): row = (image, oy, ox), column = (channel, i, j)."""
    xp = _pad(x, *padding)
    n, c, hp, wp = xp.shape
    sh, sw = stride
    oh, ow = (hp - kh) // sh + 1, (wp - kw) // sw + 1
    cols = np.empty((n, oh, ow, c, kh, kw), dtype=x.dtype)
    for i in range(kh):
        for j in range(kw):
            cols[:, :, :, :, i, j] = xp[:, :, i:i + sh * (oh - 1) + 1:sh,
                                        j:j + sw * (ow - 1) + 1:sw].transpose(0, 2, 3, 1)
    return cols.reshape(n * oh * ow, c * kh * kw), oh, ow


def conv2d_forward(x: np.ndarray, w: np.ndarray, b: np.ndarray | None,
                   stride: tuple[int, int] = (1, 1),
                   padding: tuple[int, int] = (0, 0)) -> tuple[np.ndarray, np.ndarray]:
    """``(y, cols)``: ``y = cols @ W^T (+ b)`` reshaped to NCHW (ops/conv.py:91-98)."""
    c_out = w.shape[0]
    cols, oh, ow = im2col(x, w.shape[2], w.shape[3], stride, padding)
    y = (cols @ w.reshape(c_out, -1).T).reshape(x.shape[0], oh, ow, c_out).transpose(0, 3, 1, 2)
    if b is not None:
        y = y + b.reshape(1, -1, 1, 1)
    return np.ascontiguousarray(y), cols


def conv2d_backward(g: np.ndarray, x_shape: tuple[int, ...], w: np.ndarray, cols: np.ndarray,
                    stride: tuple[int, int] = (1, 1), padding: tuple[int, int] = (0, 0),
                    has_bias: bool = True) -> tuple[np.ndarray, np.ndarray, np.ndarray | None]:
    """``(gx, gw, gb)``: ``gx`` = col2im of ``G W``, ``gw = G^T cols``, ``gb`` = sum of G
    over (N, H, W) (ops/conv.py:101-116, 159-168)."""
    n, c, h, width = x_shape
    c_out, _, kh, kw = w.shape
    (sh, sw), (ph, pw) = stride, padding
    oh, ow = g.shape[2], g.shape[3]
    g_mat = g.transpose(0, 2, 3, 1).reshape(-1, c_out)
    gw = (g_mat.T @ cols).reshape(w.shape)
    gb = g_mat.sum(axis=0) if has_bias else None
    d_cols = (g_mat @ w.reshape(c_out, -1)).reshape(n, oh, ow, c, kh, kw)
    dxp = np.zeros((n, c, h + 2 * ph, width + 2 * pw), dtype=g.dtype)
    for i in range(kh):
        for j in range(kw):
            dxp[:, :, i:i + sh * oh:sh, j:j + sw * ow:sw] += d_cols[..., i, j].transpose(0, 3, 1, 2)
    return dxp[:, :, ph:ph + h, pw:pw + width], gw, gb


# ---------------------------------------------------------------------------- batch norm
def batch_norm_forward(x: np.ndarray, w: np.ndarray | None, b: np.ndarray | None,
                       running_mean: np.ndarray | None, running_var: np.ndarray | None,
                       momentum: float = 0.1, eps: float = 1e-5) -> tuple[np.ndarray, tuple]:
    """Training-mode batch norm over ``(0, 2, 3, ...)``; returns ``(y, cache)`` and updates
    the running statistics in place (ops/layers.py:165-189)."""
    axes = (0, *range(2, x.ndim))
    view = (1, -1, *([1] * (x.ndim - 2)))
    mean = x.mean(axis=axes, keepdims=True)
    var = ((x - mean) ** 2).mean(axis=axes, keepdims=True)
    if running_mean is not None and running_var is not None:
        m = x.size // x.shape[1]
        unbiased = var.reshape(-1) * (m / max(m - 1, 1))
        running_mean *= 1 - momentum
        running_mean += momentum * mean.reshape(-1)
        running_var *= 1 - momentum
        running_var += momentum * unbiased
    rstd = 1.0 / np.sqrt(var + eps)
    xhat = (x - mean) * rstd
    y = xhat
    if w is not None:
        y = y * w.reshape(view)
    if b is not None:
        y = y + b.reshape(view)
    return y, (xhat, rstd)


def batch_norm_backward(g: np.ndarray, cache: tuple, w: np.ndarray | None) -> tuple[
    np.ndarray, np.ndarray | None, np.ndarray
]:
    """Closed form of the composite's VJP: ``gx = rstd w (g - mean(g) - xhat mean(g xhat))``,
    ``gw = sum(g xhat)``, ``gb = sum(g)`` over the statistics axes."""
    xhat, rstd = cache
    axes = (0, *range(2, g.ndim))
    view = (1, -1, *([1] * (g.ndim - 2)))
    gb = g.sum(axis=axes)
    gw = (g * xhat).sum(axis=axes)
    scale = rstd if w is None else rstd * w.reshape(view)
    gx = scale * (g - g.mean(axis=axes, keepdims=True)
                  - xhat * (g * xhat).mean(axis=axes, keepdims=True))
    return gx, (gw if w is not None else None), gb


# ---------------------------------------------------------------------------- max pool
def max_pool2d_forward(x: np.ndarray, kernel: tuple[int, int], stride: tuple[int, int],
                       padding: tuple[int, int] = (0, 0)) -> tuple[np.ndarray, np.ndarray]:
    """``(y, winner)``: window maxima over ``-inf`` padding and the row-major offset of each
    window's first maximum (NaN wins) (ops/conv.py:245-280, 330-335)."""
    (kh, kw), (sh, sw), (ph, pw) = kernel, stride, padding
    xp = _pad(x, ph, pw, -np.inf)
    oh = (xp.shape[2] - kh) // sh + 1
    ow = (xp.shape[3] - kw) // sw + 1
    views = [xp[:, :, i:i + sh * (oh - 1) + 1:sh, j:j + sw * (ow - 1) + 1:sw]
             for i in range(kh) for j in range(kw)]
    y = views[0].copy()
    for v in views[1:]:
        np.maximum(y, v, out=y)
    winner = np.zeros(y.shape, dtype=np.int64)
    open_ = np.ones(y.shape, dtype=bool)
    nan_y = np.isnan(y)
    for k, v in enumerate(views):
        hit = (v == y) | (np.isnan(v) & nan_y)
        hit &= open_
        open_ &= ~hit
        winner[hit] = k
    return y, winner


def max_pool2d_backward(g: np.ndarray, winner: np.ndarray, x_shape: tuple[int, ...],
                        kernel: tuple[int, int], stride: tuple[int, int],
                        padding: tuple[int, int] = (0, 0)) -> np.ndarray:
    """``g`` added into each window's winning cell (ops/conv.py:337-345)."""
    (kh, kw), (sh, sw), (ph, pw) = kernel, stride, padding
    n, c, h, w = x_shape
    dxp = np.zeros((n, c, h + 2 * ph, w + 2 * pw), dtype=g.dtype)
    oh, ow = g.shape[2], g.shape[3]
    for i in range(kh):
        for j in range(kw):
            dxp[:, :, i:i + sh * (oh - 1) + 1:sh, j:j + sw * (ow - 1) + 1:sw] += g * (
                winner == i * kw + j)
    return dxp[:, :, ph:ph + h, pw:pw + w]


# ---------------------------------------------------------------------------- model
def param_shapes(cfg: Config) -> list[tuple[str, tuple[int, ...]]]:
    feat = cfg.c2 * (cfg.size // 4) ** 2
    return [
        ("0.weight", (cfg.c1, cfg.in_channels, 3, 3)), ("0.bias", (cfg.c1,)),
        ("1.weight", (cfg.c1,)), ("1.bias", (cfg.c1,)),
        ("4.weight", (cfg.c2, cfg.c1, 3, 3)), ("4.bias", (cfg.c2,)),
        ("5.weight", (cfg.c2,)), ("5.bias", (cfg.c2,)),
        ("9.weight", (cfg.classes, feat)), ("9.bias", (cfg.classes,)),
    ]


def init_params(cfg: Config, seed: int) -> dict[str, np.ndarray]:
    """Seeded weights: conv and linear ``U(-1/sqrt(fan_in), 1/sqrt(fan_in))`` as the
    reference's modules draw them (nn/layers.py:42-98), batch-norm scale ``1 + 0.1 N(0,1)``
    and shift ``0.1 N(0,1)`` (not the 1/0 defaults, so that both enter the gradients)."""
    rng = np.random.default_rng(seed)
    out: dict[str, np.ndarray] = {}
    for name, shape in param_shapes(cfg):
        if name in ("1.weight", "5.weight"):
            out[name] = 1.0 + 0.1 * rng.standard_normal(shape)
        elif name in ("1.bias", "5.bias"):
            out[name] = 0.1 * rng.standard_normal(shape)
        else:
            wshape = dict(param_shapes(cfg))[name.replace("bias", "weight")]
            fan_in = int(np.prod(wshape[1:]))
            bound = 1.0 / np.sqrt(fan_in)
            out[name] = rng.uniform(-bound, bound, size=shape)
    return out


def init_buffers(cfg: Config) -> dict[str, np.ndarray]:
    return {"1.running_mean": np.zeros(cfg.c1), "1.running_var": np.ones(cfg.c1),
            "5.running_mean": np.zeros(cfg.c2), "5.running_var": np.ones(cfg.c2)}


def synthetic_batch(cfg: Config, batch: int, seed: int) -> tuple[np.ndarray, np.ndarray]:
    """Images ``N(0, 1)`` of ``(batch, in_channels, size, size)`` and labels uniform over the
    classes, from ``seed``."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((batch, cfg.in_channels, cfg.size, cfg.size))
    labels = rng.integers(0, cfg.classes, size=batch, dtype=np.int64)
    return x, labels


def max_pool2d_gather(x: np.ndarray, winner: np.ndarray, kernel: tuple[int, int],
                      stride: tuple[int, int]) -> np.ndarray:
    """Pooling output for given window winners (no padding): ``y = x`` at each winner."""
    (kh, kw), (sh, sw) = kernel, stride
    oh, ow = winner.shape[2], winner.shape[3]
    y = np.zeros(winner.shape, dtype=x.dtype)
    for i in range(kh):
        for j in range(kw):
            sel = winner == i * kw + j
            y[sel] = x[:, :, i:i + sh * (oh - 1) + 1:sh, j:j + sw * (ow - 1) + 1:sw][sel]
    return y


def forward_backward(params: dict[str, np.ndarray], buffers: dict[str, np.ndarray],
                     x: np.ndarray, labels: np.ndarray, decisions: dict | None = None,
                     acts: dict | None = None) -> tuple[float, dict[str, np.ndarray]]:
    """Loss and every parameter gradient; ``buffers`` (running statistics) are updated.

    ``decisions`` optionally fixes the discrete choices of the step -- the ReLU masks
    ``relu1``/``relu2`` and the pooling winners ``win1``/``win2`` -- to those of another
    evaluation, so that a float32 run can be compared with this float64 one where an input
    sits within rounding of a ReLU kink or a pooling tie (there the two precisions may
    legitimately choose differently). ``acts``, if given, receives the float64
    pre-activations ``b1``, ``b2`` and pooled inputs ``r1``, ``r2`` of this evaluation."""
    P = params
    d = decisions or {}
    same, k2 = (1, 1), (2, 2)
    y1, cols1 = conv2d_forward(x, P["0.weight"], P["0.bias"], same, same)
    b1, bn1 = batch_norm_forward(y1, P["1.weight"], P["1.bias"], buffers["1.running_mean"],
                                 buffers["1.running_var"])
    m1 = d.get("relu1", b1 > 0)
    r1 = b1 * m1
    if "win1" in d:
        win1 = d["win1"]
        p1 = max_pool2d_gather(r1, win1, k2, k2)
    else:
        p1, win1 = max_pool2d_forward(r1, k2, k2)
    y2, cols2 = conv2d_forward(p1, P["4.weight"], P["4.bias"], same, same)
    b2, bn2 = batch_norm_forward(y2, P["5.weight"], P["5.bias"], buffers["5.running_mean"],
                                 buffers["5.running_var"])
    m2 = d.get("relu2", b2 > 0)
    r2 = b2 * m2
    if "win2" in d:
        win2 = d["win2"]
        p2 = max_pool2d_gather(r2, win2, k2, k2)
    else:
        p2, win2 = max_pool2d_forward(r2, k2, k2)
    if acts is not None:
        acts.update(b1=b1, b2=b2, r1=r1, r2=r2)
    flat = p2.reshape(p2.shape[0], -1)
    logits = ops.linear_forward(flat, P["9.weight"], P["9.bias"])
    loss, logp = ops.cross_entropy_forward(logits, labels)

    G: dict[str, np.ndarray] = {}
    g = ops.cross_entropy_backward(1.0, logp, labels, logits.shape)
    gflat, G["9.weight"], G["9.bias"] = ops.linear_backward(g, flat, P["9.weight"], True)
    g = max_pool2d_backward(gflat.reshape(p2.shape), win2, r2.shape, k2, k2)
    g = g * m2
    g, G["5.weight"], G["5.bias"] = batch_norm_backward(g, bn2, P["5.weight"])
    g, G["4.weight"], G["4.bias"] = conv2d_backward(g, p1.shape, P["4.weight"], cols2, same,
                                                    same)
    g = max_pool2d_backward(g, win1, r1.shape, k2, k2)
    g = g * m1
    g, G["1.weight"], G["1.bias"] = batch_norm_backward(g, bn1, P["1.weight"])
    _, G["0.weight"], G["0.bias"] = conv2d_backward(g, x.shape, P["0.weight"], cols1, same, same)
    return float(loss), {name: G[name] for name in P}


def train_step(params: dict[str, np.ndarray], buffers: dict[str, np.ndarray], x: np.ndarray,
               labels: np.ndarray, state: AdamWState | None = None, *, lr: float = 3e-4,
               betas: tuple[float, float] = (0.9, 0.999), eps: float = 1e-8,
               weight_decay: float = 1e-4, decisions: dict | None = None,
               acts: dict | None = None) -> dict[str, object]:
    """Forward, backward and one AdamW update (no clipping)."""
    loss, grads = forward_backward(params, buffers, x, labels, decisions, acts)
    names = list(grads)
    if state is None:
        state = AdamWState({n: np.zeros_like(params[n]) for n in names},
                           {n: np.zeros_like(params[n]) for n in names}, {n: 0 for n in names})
    new_params = {}
    for n in names:
        state.step[n] += 1
        new_params[n], state.m[n], state.v[n] = ops.adamw_update(
            params[n], grads[n], state.m[n], state.v[n], state.step[n], lr, betas, eps,
            weight_decay)
    return {"loss": loss, "grads": grads, "params": new_params, "state": state,
            "buffers": {k: v.copy() for k, v in buffers.items()}}


def step_flops(cfg: Config, batch: int) -> float:
    """Convolution FLOPs of one step: forward of both convolutions, the weight gradients of
    both, the input gradient of the second (the images need none)."""
    s = cfg.size
    f1 = 2.0 * batch * s * s * cfg.c1 * cfg.in_channels * 9
    f2 = 2.0 * batch * (s // 2) ** 2 * cfg.c2 * cfg.c1 * 9
    return 2 * f1 + 3 * f2
