"""Float64 NumPy restatement of the reference's LSTM / GRU training step (test infrastructure
only).

The model is the adding-problem regressor of the reference's ``examples/adding_problem.py``
(lines 71-81): ``nn.LSTM(2, H)`` or ``nn.GRU(2, H)`` over a time-major ``(T, B, 2)`` sequence,
``Linear(H, 1)`` on the last hidden state, ``mse_loss`` against ``(B, 1)`` targets;
``loss.backward()`` (backpropagation through time); ``AdamW.step()`` (no clipping).

The recurrences and their VJPs restate ``ops/recurrent.py``: the input projection for all
steps as one product, the serial recurrence keeping the gate activations (LSTM 223-272,
GRU 336-385), the reverse-time loop carrying the hidden (and cell) gradients (LSTM 274-292,
GRU 387-403) and one product per weight at the end (``_parameter_grads`` 92-109). The
sigmoid is the reference's overflow-free form (ops/elementwise.py:230-237).
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from oracle import ops
from oracle.gpt import AdamWState


def sigmoid(x: np.ndarray) -> np.ndarray:
    z = np.exp(-np.abs(x))
    return np.where(x >= 0, 1 / (1 + z), z / (1 + z))


def _previous(h0: np.ndarray, hs: np.ndarray) -> np.ndarray:
    return np.concatenate((h0[None], hs[:-1])).reshape(-1, h0.shape[-1])


def _param_grads(dz, dz_hh, x, h_prev, w_ih, has_bias):
    rows = dz.shape[-1]
    dz2, dh2 = dz.reshape(-1, rows), dz_hh.reshape(-1, rows)
    dx = (dz2 @ w_ih).reshape(x.shape)
    dw_ih = dz2.T @ x.reshape(-1, x.shape[-1])
    dw_hh = dh2.T @ h_prev
    dbs = (dz2.sum(axis=0), dh2.sum(axis=0)) if has_bias else (None, None)
    return dx, dw_ih, dw_hh, *dbs


# ---------------------------------------------------------------------------- LSTM
def lstm_forward(x, h0, c0, w_ih, w_hh, b_ih=None, b_hh=None):
    """``(out, cache)``; ``out`` is ``(T, B, 2, H)``: hidden and cell state of every step."""
    steps, batch, hid = x.shape[0], x.shape[1], h0.shape[1]
    acts = (x.reshape(-1, x.shape[2]) @ w_ih.T).reshape(steps, batch, -1)
    if b_ih is not None:
        acts += b_ih + b_hh
    out = np.empty((steps, batch, 2, hid))
    tanh_c = np.empty((steps, batch, hid))
    h, c = h0, c0
    for t in range(steps):
        z = acts[t]
        z += h @ w_hh.T
        z[:, :2 * hid] = sigmoid(z[:, :2 * hid])
        z[:, 3 * hid:] = sigmoid(z[:, 3 * hid:])
        z[:, 2 * hid:3 * hid] = np.tanh(z[:, 2 * hid:3 * hid])
        c_new = z[:, hid:2 * hid] * c + z[:, :hid] * z[:, 2 * hid:3 * hid]
        out[t, :, 1] = c_new
        tanh_c[t] = np.tanh(c_new)
        out[t, :, 0] = z[:, 3 * hid:] * tanh_c[t]
        h, c = out[t, :, 0], out[t, :, 1]
    return out, (acts, tanh_c)


def lstm_backward(g, x, h0, c0, w_ih, w_hh, has_bias, out, cache):
    """``(dx, dh0, dc0, dw_ih, dw_hh, db_ih, db_hh)``."""
    acts, tanh_c = cache
    steps, hid = x.shape[0], h0.shape[1]
    dz = np.empty_like(acts)
    dh, dc = np.zeros_like(h0), np.zeros_like(c0)
    for t in range(steps - 1, -1, -1):
        dh = dh + g[t, :, 0]
        dc = dc + g[t, :, 1]
        a, tc = acts[t], tanh_c[t]
        i, f, gg, o = (a[:, k * hid:(k + 1) * hid] for k in range(4))
        c_prev = c0 if t == 0 else out[t - 1, :, 1]
        dc = dc + dh * o * (1.0 - tc * tc)
        dz[t, :, :hid] = dc * gg * (i * (1.0 - i))
        dz[t, :, hid:2 * hid] = dc * c_prev * (f * (1.0 - f))
        dz[t, :, 2 * hid:3 * hid] = dc * i * (1.0 - gg * gg)
        dz[t, :, 3 * hid:] = dh * tc * (o * (1.0 - o))
        dc = dc * f
        dh = dz[t] @ w_hh
    dx, dw_ih, dw_hh, db_ih, db_hh = _param_grads(dz, dz, x, _previous(h0, out[:, :, 0]), w_ih,
                                                  has_bias)
    return dx, dh, dc, dw_ih, dw_hh, db_ih, db_hh


# ---------------------------------------------------------------------------- GRU
def gru_forward(x, h0, w_ih, w_hh, b_ih=None, b_hh=None):
    """``(out, cache)``; ``out`` is ``(T, B, H)``."""
    steps, batch, hid = x.shape[0], x.shape[1], h0.shape[1]
    acts = (x.reshape(-1, x.shape[2]) @ w_ih.T).reshape(steps, batch, -1)
    if b_ih is not None:
        acts += b_ih
    hn = np.empty((steps, batch, hid))
    out = np.empty((steps, batch, hid))
    h = h0
    for t in range(steps):
        hw = h @ w_hh.T
        if b_hh is not None:
            hw = hw + b_hh
        a = acts[t]
        a[:, :2 * hid] = sigmoid(a[:, :2 * hid] + hw[:, :2 * hid])
        hn[t] = hw[:, 2 * hid:]
        a[:, 2 * hid:] = np.tanh(a[:, 2 * hid:] + a[:, :hid] * hn[t])
        n, u = a[:, 2 * hid:], a[:, hid:2 * hid]
        out[t] = (h - n) * u + n
        h = out[t]
    return out, (acts, hn)


def gru_backward(g, x, h0, w_ih, w_hh, has_bias, out, cache):
    """``(dx, dh0, dw_ih, dw_hh, db_ih, db_hh)``."""
    acts, hn = cache
    steps, hid = x.shape[0], h0.shape[1]
    dz_ih, dz_hh = np.empty_like(acts), np.empty_like(acts)
    dh = np.zeros_like(h0)
    for t in range(steps - 1, -1, -1):
        dh = dh + g[t]
        a = acts[t]
        r, u, n = (a[:, k * hid:(k + 1) * hid] for k in range(3))
        h_prev = h0 if t == 0 else out[t - 1]
        dn = dh * (1.0 - u) * (1.0 - n * n)
        du = dh * (h_prev - n) * (u * (1.0 - u))
        dr = dn * hn[t] * (r * (1.0 - r))
        dz_ih[t] = np.concatenate([dr, du, dn], axis=1)
        dz_hh[t] = np.concatenate([dr, du, dn * r], axis=1)
        dh = dh * u + dz_hh[t] @ w_hh
    dx, dw_ih, dw_hh, db_ih, db_hh = _param_grads(dz_ih, dz_hh, x, _previous(h0, out), w_ih,
                                                  has_bias)
    return dx, dh, dw_ih, dw_hh, db_ih, db_hh


# ---------------------------------------------------------------------------- Elman RNN
def rnn_forward(x, h0, w_ih, w_hh, b_ih=None, b_hh=None, relu=False):
    """``h_t = act(x_t W_ih^T + b_ih + h_{t-1} W_hh^T + b_hh)``, ``(T, B, H)``
    (ops/recurrent.py:140-181)."""
    steps, batch = x.shape[0], x.shape[1]
    out = (x.reshape(-1, x.shape[2]) @ w_ih.T).reshape(steps, batch, -1)
    if b_ih is not None:
        out = out + b_ih + b_hh
    h = h0
    for t in range(steps):
        a = out[t] + h @ w_hh.T
        out[t] = np.maximum(a, 0.0) if relu else np.tanh(a)
        h = out[t]
    return out


def rnn_backward(g, x, h0, w_ih, w_hh, has_bias, out, relu=False):
    """BPTT of :func:`rnn_forward`: ``(dx, dh0, dw_ih, dw_hh, db_ih, db_hh)``
    (ops/recurrent.py:183-193)."""
    dz = np.empty_like(out)
    dh = np.zeros_like(h0)
    for t in range(out.shape[0] - 1, -1, -1):
        dh = dh + g[t]
        dz[t] = dh * (out[t] > 0) if relu else dh * (1.0 - out[t] * out[t])
        dh = dz[t] @ w_hh
    dx, dw_ih, dw_hh, db_ih, db_hh = _param_grads(dz, dz, x, _previous(h0, out), w_ih, has_bias)
    return dx, dh, dw_ih, dw_hh, db_ih, db_hh


# ---------------------------------------------------------------------------- model
@dataclass(frozen=True)
class Config:
    """Cell kind (``"lstm"`` / ``"gru"``), hidden size, sequence length, input size 2."""

    cell: str = "lstm"
    hidden: int = 512
    seq: int = 100
    inputs: int = 2

    @property
    def gates(self) -> int:
        return 4 if self.cell == "lstm" else 3


def param_shapes(cfg: Config) -> list[tuple[str, tuple[int, ...]]]:
    rows = cfg.gates * cfg.hidden
    return [("rnn.weight_ih_l0", (rows, cfg.inputs)), ("rnn.weight_hh_l0", (rows, cfg.hidden)),
            ("rnn.bias_ih_l0", (rows,)), ("rnn.bias_hh_l0", (rows,)),
            ("head.weight", (1, cfg.hidden)), ("head.bias", (1,))]


def init_params(cfg: Config, seed: int) -> dict[str, np.ndarray]:
    """``U(-1/sqrt(H), 1/sqrt(H))`` for the recurrent layer (nn/recurrent.py:51-62) and the
    head (nn/layers.py:42-62: ``1/sqrt(in_features)``, the same bound here)."""
    rng = np.random.default_rng(seed)
    bound = 1.0 / np.sqrt(cfg.hidden)
    return {name: rng.uniform(-bound, bound, size=shape) for name, shape in param_shapes(cfg)}


def synthetic_batch(cfg: Config, batch: int, seed: int) -> tuple[np.ndarray, np.ndarray]:
    """The adding problem (examples/adding_problem.py:57-68): values ``U[0, 1]``, two markers
    per sequence (one in each half), target = the sum of the two marked values."""
    rng = np.random.default_rng(seed)
    length = cfg.seq
    values = rng.uniform(0.0, 1.0, size=(length, batch))
    half = length // 2
    first = rng.integers(0, half, size=batch)
    second = rng.integers(half, length, size=batch)
    markers = np.zeros((length, batch))
    markers[first, np.arange(batch)] = 1.0
    markers[second, np.arange(batch)] = 1.0
    x = np.stack([values, markers], axis=-1)
    y = (values * markers).sum(axis=0)[:, None]
    return x, y


def forward_backward(params: dict[str, np.ndarray], cfg: Config, x: np.ndarray,
                     y: np.ndarray) -> tuple[float, dict[str, np.ndarray]]:
    P = params
    batch = x.shape[1]
    h0 = np.zeros((batch, cfg.hidden))
    w_ih, w_hh, b_ih, b_hh = (P[f"rnn.{n}_l0"] for n in ("weight_ih", "weight_hh", "bias_ih",
                                                         "bias_hh"))
    if cfg.cell == "lstm":
        out, cache = lstm_forward(x, h0, h0, w_ih, w_hh, b_ih, b_hh)
        last = out[-1, :, 0]
    else:
        out, cache = gru_forward(x, h0, w_ih, w_hh, b_ih, b_hh)
        last = out[-1]
    pred = ops.linear_forward(last, P["head.weight"], P["head.bias"])
    loss = ops.mse_forward(pred, y)
    G: dict[str, np.ndarray] = {}
    gp = ops.mse_backward(1.0, pred, y)
    glast, G["head.weight"], G["head.bias"] = ops.linear_backward(gp, last, P["head.weight"], True)
    if cfg.cell == "lstm":
        g = np.zeros_like(out)
        g[-1, :, 0] = glast
        _, _, _, dw_ih, dw_hh, db_ih, db_hh = lstm_backward(g, x, h0, h0, w_ih, w_hh, True, out,
                                                            cache)
    else:
        g = np.zeros_like(out)
        g[-1] = glast
        _, _, dw_ih, dw_hh, db_ih, db_hh = gru_backward(g, x, h0, w_ih, w_hh, True, out, cache)
    G["rnn.weight_ih_l0"], G["rnn.weight_hh_l0"] = dw_ih, dw_hh
    G["rnn.bias_ih_l0"], G["rnn.bias_hh_l0"] = db_ih, db_hh
    return float(loss), {n: G[n] for n in P}


def train_step(params: dict[str, np.ndarray], cfg: Config, x: np.ndarray, y: np.ndarray,
               state: AdamWState | None = None, *, lr: float = 3e-4,
               betas: tuple[float, float] = (0.9, 0.999), eps: float = 1e-8,
               weight_decay: float = 1e-4) -> dict[str, object]:
    loss, grads = forward_backward(params, cfg, x, y)
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
    return {"loss": loss, "grads": grads, "params": new_params, "state": state}


def step_flops(cfg: Config, batch: int) -> float:
    """Recurrent-product FLOPs of one step: the forward recurrence, the backward
    ``dz W_hh`` per step and the ``dW_hh`` product, each ``2 T B H (G H)``."""
    return 3.0 * 2 * cfg.seq * batch * cfg.hidden * cfg.gates * cfg.hidden
