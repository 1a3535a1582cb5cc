"""Stacked Elman RNN, LSTM and GRU layers on the device (API of the reference's
nn/recurrent.py:24-205, PyTorch's parameter names and call signatures).

Each layer of the stack is one fused sequence op (``ops.recurrent.rnn`` / ``lstm`` / ``gru``: the input
projection for all steps, then the recurrence, and backpropagation through time, inside one
C call). Layers take the previous layer's hidden sequence (with dropout between layers in
training); the final states are the last step of each layer.
"""

from __future__ import annotations

import math

import numpy as np

from tensorgrad_b200 import ops
from tensorgrad_b200._random import get_rng
from tensorgrad_b200.nn.module import Module, Parameter
from tensorgrad_b200.ops.recurrent import gru, lstm, rnn
from tensorgrad_b200.ops.shape import stack
from tensorgrad_b200.tensor import Tensor, get_default_dtype

__all__ = ["GRU", "LSTM", "RNN"]


class _RecurrentStack(Module):
    """``num_layers`` recurrent layers of ``gates * hidden_size`` gate rows. Layer ``k`` owns
    ``weight_ih_lk``, ``weight_hh_lk`` and, with ``bias``, ``bias_ih_lk`` and ``bias_hh_lk``,
    drawn in that order from ``U(-1/sqrt(hidden), 1/sqrt(hidden))``."""

    gates = 1

    def __init__(self, input_size: int, hidden_size: int, num_layers: int = 1, bias: bool = True,
                 batch_first: bool = False, dropout: float = 0.0) -> None:
        super().__init__()
        if min(input_size, hidden_size, num_layers) < 1:
            raise ValueError("input_size, hidden_size and num_layers must be positive")
        if not 0.0 <= dropout <= 1.0:
            raise ValueError(f"dropout probability must be in [0, 1], got {dropout}")
        self.input_size, self.hidden_size, self.num_layers = input_size, hidden_size, num_layers
        self.bias, self.batch_first, self.dropout = bias, batch_first, dropout
        bound = 1.0 / math.sqrt(hidden_size)
        g = self.gates * hidden_size
        rng, dt = get_rng(), get_default_dtype()
        for k in range(num_layers):
            fan_in = input_size if k == 0 else hidden_size
            for name, shape in self._layer_shapes(g, fan_in):
                drawn = rng.uniform(-bound, bound, size=shape)
                setattr(self, f"{name}_l{k}", Parameter(np.asarray(drawn, dtype=dt)))

    def _layer_shapes(self, g: int, fan_in: int) -> list[tuple[str, tuple[int, ...]]]:
        shapes = [("weight_ih", (g, fan_in)), ("weight_hh", (g, self.hidden_size))]
        return shapes + ([("bias_ih", (g,)), ("bias_hh", (g,))] if self.bias else [])

    def layer_weights(self, layer: int) -> list[Tensor]:
        """``[weight_ih, weight_hh(, bias_ih, bias_hh)]`` of one layer."""
        names = ["weight_ih", "weight_hh", "bias_ih", "bias_hh"][:4 if self.bias else 2]
        return [getattr(self, f"{n}_l{layer}") for n in names]

    def _sequence(self, x: Tensor) -> Tensor:
        """The input as time-major ``(T, B, input_size)``."""
        if x.ndim != 3 or x.shape[-1] != self.input_size:
            layout = "(B, T, input_size)" if self.batch_first else "(T, B, input_size)"
            raise ValueError(f"{type(self).__name__} expects {layout} input with input_size "
                             f"{self.input_size}, got {x.shape}")
        return ops.transpose(x, 0, 1) if self.batch_first else x

    def _state(self, given: Tensor | None, batch: int, dtype: np.dtype) -> Tensor:
        want = (self.num_layers, batch, self.hidden_size)
        if given is None:
            return Tensor(np.zeros(want, dtype=dtype))
        if given.shape != want:
            raise ValueError(f"initial state should have shape {want}, got {given.shape}")
        return given

    def _between_layers(self, hs: Tensor, layer: int) -> Tensor:
        last = layer == self.num_layers - 1
        if self.dropout > 0 and self.training and not last:
            return ops.dropout(hs, self.dropout, True)
        return hs

    def _result(self, hs: Tensor) -> Tensor:
        return ops.transpose(hs, 0, 1) if self.batch_first else hs

    def extra_repr(self) -> str:
        return (f"{self.input_size}, {self.hidden_size}, num_layers={self.num_layers}, "
                f"bias={self.bias}, batch_first={self.batch_first}, dropout={self.dropout}")


class LSTM(_RecurrentStack):
    """Multi-layer LSTM (gates i, f, g, o): ``output, (h_n, c_n) = lstm(x, (h_0, c_0))``."""

    gates = 4

    def forward(self, x: Tensor, state: tuple[Tensor, Tensor] | None = None  # type: ignore[override]
                ) -> tuple[Tensor, tuple[Tensor, Tensor]]:
        seq = self._sequence(x)
        batch = seq.shape[1]
        h0 = self._state(state[0] if state else None, batch, seq.dtype)
        c0 = self._state(state[1] if state else None, batch, seq.dtype)
        h_last, c_last = [], []
        hs = seq
        for k in range(self.num_layers):
            out = lstm(seq, h0[k], c0[k], *self.layer_weights(k))  # (T, B, 2, H): h_t and c_t
            hs = out[:, :, 0]
            h_last.append(out[-1, :, 0])
            c_last.append(out[-1, :, 1])
            seq = self._between_layers(hs, k)
        return self._result(hs), (stack(h_last, 0), stack(c_last, 0))

    def __call__(self, x: Tensor, state: tuple[Tensor, Tensor] | None = None  # type: ignore[override]
                 ) -> tuple[Tensor, tuple[Tensor, Tensor]]:
        return self.forward(x, state)


class GRU(_RecurrentStack):
    """Multi-layer GRU (gates r, u, n; PyTorch's formulation): ``output, h_n = gru(x, h_0)``."""

    gates = 3

    def forward(self, x: Tensor, h0: Tensor | None = None) -> tuple[Tensor, Tensor]:  # type: ignore[override]
        seq = self._sequence(x)
        state = self._state(h0, seq.shape[1], seq.dtype)
        last = []
        hs = seq
        for k in range(self.num_layers):
            hs = gru(seq, state[k], *self.layer_weights(k))
            last.append(hs[-1])
            seq = self._between_layers(hs, k)
        return self._result(hs), stack(last, 0)

    def __call__(self, x: Tensor, h0: Tensor | None = None) -> tuple[Tensor, Tensor]:  # type: ignore[override]
        return self.forward(x, h0)


class RNN(_RecurrentStack):
    """Multi-layer Elman RNN, ``h_t = act(x_t W_ih^T + b_ih + h_{t-1} W_hh^T + b_hh)`` with
    ``act`` tanh or relu: ``output, h_n = rnn(x, h_0)``."""

    gates = 1

    def __init__(self, input_size: int, hidden_size: int, num_layers: int = 1,
                 nonlinearity: str = "tanh", bias: bool = True, batch_first: bool = False,
                 dropout: float = 0.0) -> None:
        if nonlinearity not in ("tanh", "relu"):
            raise ValueError(f"nonlinearity must be 'tanh' or 'relu', got {nonlinearity!r}")
        super().__init__(input_size, hidden_size, num_layers, bias, batch_first, dropout)
        self.nonlinearity = nonlinearity

    def forward(self, x: Tensor, h0: Tensor | None = None) -> tuple[Tensor, Tensor]:  # type: ignore[override]
        seq = self._sequence(x)
        state = self._state(h0, seq.shape[1], seq.dtype)
        last = []
        hs = seq
        for k in range(self.num_layers):
            hs = rnn(seq, state[k], *self.layer_weights(k), nonlinearity=self.nonlinearity)
            last.append(hs[-1])
            seq = self._between_layers(hs, k)
        return self._result(hs), stack(last, 0)

    def __call__(self, x: Tensor, h0: Tensor | None = None) -> tuple[Tensor, Tensor]:  # type: ignore[override]
        return self.forward(x, h0)

    def extra_repr(self) -> str:
        return super().extra_repr() + f", nonlinearity={self.nonlinearity!r}"
