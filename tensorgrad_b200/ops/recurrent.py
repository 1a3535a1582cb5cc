"""LSTM and GRU sequence ops with backpropagation through time (the reference's
ops/recurrent.py:223-437).

Each op runs a whole time-major sequence as one graph node and one C-ABI call per direction:
the host loop over time steps is C++ inside the library, which launches the per-step
recurrent GEMM (tensor cores for fp32) and the gate kernel. Weight layouts and gate order are
the reference's (PyTorch's): LSTM rows (i, f, g, o), GRU rows (r, u, n).

Under ``create_graph=True`` the VJP differentiates the same recurrence unrolled in
differentiable ops (one input projection, then per step the recurrent product, the gates and
the state update), so BPTT gradients are differentiable again, as the reference's graph VJPs
are (ops/recurrent.py:294-332, 405-437).
"""

from __future__ import annotations

from collections.abc import Sequence
from typing import Any

import numpy as np

from tensorgrad_b200 import device
from tensorgrad_b200._lib import check, lib
from tensorgrad_b200.device import DeviceArray, dtype_code
from tensorgrad_b200.ops._util import Need, as_tensor, graph_by_composite, make_result
from tensorgrad_b200.ops.elementwise import cast_array
from tensorgrad_b200.profiler import profiled
from tensorgrad_b200.tensor import Tensor

__all__ = ["gru", "lstm", "rnn"]

_GATES = {"rnn": 1, "lstm": 4, "gru": 3}


def _prepare(kind: str, x: Any, states: Sequence[Any], w_ih: Any, w_hh: Any, b_ih: Any,
             b_hh: Any) -> tuple[tuple[Tensor, ...], list[DeviceArray]]:
    """Validate shapes (ops/recurrent.py:40-75) and return the parents
    ``(x, *states, w_ih, w_hh[, b_ih, b_hh])`` with their data in one floating dtype."""
    if (b_ih is None) != (b_hh is None):
        raise ValueError(f"{kind}: pass both biases or neither")
    tx, tw_ih, tw_hh = as_tensor(x), as_tensor(w_ih), as_tensor(w_hh)
    tstates = [as_tensor(s) for s in states]
    tbiases = [] if b_ih is None else [as_tensor(b_ih), as_tensor(b_hh)]
    if tx.ndim != 3 or tx.shape[0] == 0:
        raise ValueError(
            f"{kind}: expected a non-empty (T, B, input_size) sequence, got {tx.shape}"
        )
    hidden = tw_hh.shape[-1] if tw_hh.ndim == 2 else -1
    rows = _GATES[kind] * hidden
    if tw_hh.shape != (rows, hidden) or tw_ih.shape != (rows, tx.shape[2]):
        raise ValueError(
            f"{kind}: weights {tw_ih.shape} and {tw_hh.shape} do not fit input size "
            f"{tx.shape[2]} ({_GATES[kind]} gate(s) of the hidden size {hidden})"
        )
    for b in tbiases:
        if b.shape != (rows,):
            raise ValueError(f"{kind}: bias of shape {b.shape} should be ({rows},)")
    for s in tstates:
        if s.shape != (tx.shape[1], hidden):
            raise ValueError(f"{kind}: initial state {s.shape} should be {(tx.shape[1], hidden)}")
    parents = (tx, *tstates, tw_ih, tw_hh, *tbiases)
    dt = np.result_type(np.float32, *(p.dtype for p in parents))
    return parents, [p.data if p.dtype == dt else cast_array(p.data, dt) for p in parents]


def _ptr(a: DeviceArray | None) -> int | None:
    return None if a is None else a.ptr


def _cols(z: Tensor, start: int, stop: int) -> Tensor:
    from tensorgrad_b200.ops.shape import getitem

    return getitem(z, (slice(None), slice(start, stop)))


def _lstm_composite(x: Tensor, h0: Tensor, c0: Tensor, w_ih: Tensor, w_hh: Tensor,
                    b_ih: Tensor | None = None, b_hh: Tensor | None = None) -> Tensor:
    """The LSTM recurrence in differentiable ops, ``(T, B, 2, H)`` like :func:`lstm`."""
    from tensorgrad_b200.ops import elementwise as E
    from tensorgrad_b200.ops.layers import linear
    from tensorgrad_b200.ops.shape import getitem, stack

    hid = h0.shape[1]
    xw = linear(x, w_ih, b_ih)
    h, c = h0, c0
    steps = []
    for t in range(x.shape[0]):
        z = E.add(getitem(xw, t), linear(h, w_hh, b_hh))
        i, f = E.sigmoid(_cols(z, 0, hid)), E.sigmoid(_cols(z, hid, 2 * hid))
        g, o = E.tanh(_cols(z, 2 * hid, 3 * hid)), E.sigmoid(_cols(z, 3 * hid, 4 * hid))
        c = E.add(E.mul(f, c), E.mul(i, g))
        h = E.mul(o, E.tanh(c))
        steps.append(stack([h, c], 1))
    return stack(steps, 0)


def _gru_composite(x: Tensor, h0: Tensor, w_ih: Tensor, w_hh: Tensor,
                   b_ih: Tensor | None = None, b_hh: Tensor | None = None) -> Tensor:
    """The GRU recurrence in differentiable ops, ``(T, B, H)`` like :func:`gru`."""
    from tensorgrad_b200.ops import elementwise as E
    from tensorgrad_b200.ops.layers import linear
    from tensorgrad_b200.ops.shape import getitem, stack

    hid = h0.shape[1]
    xw = linear(x, w_ih, b_ih)
    h = h0
    steps = []
    for t in range(x.shape[0]):
        a, b = getitem(xw, t), linear(h, w_hh, b_hh)
        r = E.sigmoid(E.add(_cols(a, 0, hid), _cols(b, 0, hid)))
        u = E.sigmoid(E.add(_cols(a, hid, 2 * hid), _cols(b, hid, 2 * hid)))
        n = E.tanh(E.add(_cols(a, 2 * hid, 3 * hid), E.mul(r, _cols(b, 2 * hid, 3 * hid))))
        h = E.add(E.mul(E.sub(1.0, u), n), E.mul(u, h))
        steps.append(h)
    return stack(steps, 0)


@profiled("lstm")
def lstm(x: Any, h0: Any, c0: Any, w_ih: Any, w_hh: Any, b_ih: Any = None,
         b_hh: Any = None) -> Tensor:
    """Long short-term memory over a ``(T, B, input_size)`` sequence. Returns ``(T, B, 2, H)``:
    ``[:, :, 0]`` the hidden states ``h_1 .. h_T``, ``[:, :, 1]`` the cell states."""
    parents, arrays = _prepare("lstm", x, (h0, c0), w_ih, w_hh, b_ih, b_hh)
    xd, h0d, c0d, w_ihd, w_hhd = arrays[:5]
    bias = arrays[5:] if len(arrays) > 5 else [None, None]
    steps, batch, width = xd.shape
    hid = h0d.shape[1]
    dt = xd.dtype
    code = dtype_code(dt)
    acts = device.empty((steps, batch, 4 * hid), dt)
    out = device.empty((steps, batch, 2, hid), dt)
    tanh_c = device.empty((steps, batch, hid), dt)
    scratch = device.scratch(lib.tg_lstm_forward_scratch_bytes(code, steps, batch, width, hid))
    check(lib.tg_lstm_forward(code, steps, batch, width, hid, xd.ptr, h0d.ptr, c0d.ptr,
                              w_ihd.ptr, w_hhd.ptr, _ptr(bias[0]), _ptr(bias[1]), acts.ptr,
                              out.ptr, tanh_c.ptr, scratch.ptr, device.stream()), "lstm")
    has_bias = len(arrays) > 5

    def backward(g: DeviceArray, need: Need) -> tuple[DeviceArray | None, ...]:
        if g.dtype != dt:
            g = cast_array(g, dt)

        def want(k: int, shape: tuple[int, ...]) -> DeviceArray | None:
            return device.empty(shape, dt) if need[k] else None

        dx = want(0, xd.shape)
        dh0, dc0 = want(1, h0d.shape), want(2, c0d.shape)
        dw_ih, dw_hh = want(3, w_ihd.shape), want(4, w_hhd.shape)
        db_ih = want(5, (4 * hid,)) if has_bias else None
        db_hh = want(6, (4 * hid,)) if has_bias else None
        scr = device.scratch(lib.tg_lstm_backward_scratch_bytes(code, steps, batch, width, hid))
        check(lib.tg_lstm_backward(
            code, steps, batch, width, hid, g.ptr, xd.ptr, h0d.ptr, c0d.ptr, w_ihd.ptr,
            w_hhd.ptr, acts.ptr, out.ptr, tanh_c.ptr, _ptr(dx), _ptr(dh0), _ptr(dc0),
            _ptr(dw_ih), _ptr(dw_hh), _ptr(db_ih), _ptr(db_hh), scr.ptr, device.stream()),
            "lstm backward")
        grads = [dx, dh0, dc0, dw_ih, dw_hh]
        return tuple(grads + [db_ih, db_hh] if has_bias else grads)

    def graph(g: Tensor, y: Tensor, need: Need) -> tuple[Tensor | None, ...]:
        return graph_by_composite(parents, _lstm_composite, g, need)

    return make_result(out, parents, backward, "lstm", graph)


@profiled("gru")
def gru(x: Any, h0: Any, w_ih: Any, w_hh: Any, b_ih: Any = None, b_hh: Any = None) -> Tensor:
    """Gated recurrent unit over a ``(T, B, input_size)`` sequence in PyTorch's formulation;
    returns the hidden states ``h_1 .. h_T``, ``(T, B, H)``."""
    parents, arrays = _prepare("gru", x, (h0,), w_ih, w_hh, b_ih, b_hh)
    xd, h0d, w_ihd, w_hhd = arrays[:4]
    bias = arrays[4:] if len(arrays) > 4 else [None, None]
    steps, batch, width = xd.shape
    hid = h0d.shape[1]
    dt = xd.dtype
    code = dtype_code(dt)
    acts = device.empty((steps, batch, 3 * hid), dt)
    hn = device.empty((steps, batch, hid), dt)
    out = device.empty((steps, batch, hid), dt)
    scratch = device.scratch(lib.tg_gru_forward_scratch_bytes(code, steps, batch, width, hid))
    check(lib.tg_gru_forward(code, steps, batch, width, hid, xd.ptr, h0d.ptr, w_ihd.ptr,
                             w_hhd.ptr, _ptr(bias[0]), _ptr(bias[1]), acts.ptr, hn.ptr, out.ptr,
                             scratch.ptr, device.stream()), "gru")
    has_bias = len(arrays) > 4

    def backward(g: DeviceArray, need: Need) -> tuple[DeviceArray | None, ...]:
        if g.dtype != dt:
            g = cast_array(g, dt)

        def want(k: int, shape: tuple[int, ...]) -> DeviceArray | None:
            return device.empty(shape, dt) if need[k] else None

        dx, dh0 = want(0, xd.shape), want(1, h0d.shape)
        dw_ih, dw_hh = want(2, w_ihd.shape), want(3, w_hhd.shape)
        db_ih = want(4, (3 * hid,)) if has_bias else None
        db_hh = want(5, (3 * hid,)) if has_bias else None
        scr = device.scratch(lib.tg_gru_backward_scratch_bytes(code, steps, batch, width, hid))
        check(lib.tg_gru_backward(
            code, steps, batch, width, hid, g.ptr, xd.ptr, h0d.ptr, w_ihd.ptr, w_hhd.ptr,
            acts.ptr, hn.ptr, out.ptr, _ptr(dx), _ptr(dh0), _ptr(dw_ih), _ptr(dw_hh),
            _ptr(db_ih), _ptr(db_hh), scr.ptr, device.stream()), "gru backward")
        grads = [dx, dh0, dw_ih, dw_hh]
        return tuple(grads + [db_ih, db_hh] if has_bias else grads)

    def graph(g: Tensor, y: Tensor, need: Need) -> tuple[Tensor | None, ...]:
        return graph_by_composite(parents, _gru_composite, g, need)

    return make_result(out, parents, backward, "gru", graph)


def _rnn_composite(x: Tensor, h0: Tensor, w_ih: Tensor, w_hh: Tensor,
                   b_ih: Tensor | None = None, b_hh: Tensor | None = None, *,
                   relu: bool = False) -> Tensor:
    """The Elman recurrence in differentiable ops, ``(T, B, H)`` like :func:`rnn`."""
    from tensorgrad_b200.ops import elementwise as E
    from tensorgrad_b200.ops.layers import linear
    from tensorgrad_b200.ops.shape import getitem, stack

    xw = linear(x, w_ih, b_ih)
    h = h0
    steps = []
    for t in range(x.shape[0]):
        pre = E.add(getitem(xw, t), linear(h, w_hh, b_hh))
        h = E.relu(pre) if relu else E.tanh(pre)
        steps.append(h)
    return stack(steps, 0)


@profiled("rnn")
def rnn(x: Any, h0: Any, w_ih: Any, w_hh: Any, b_ih: Any = None, b_hh: Any = None, *,
        nonlinearity: str = "tanh") -> Tensor:
    """Elman RNN ``h_t = act(x_t W_ih^T + b_ih + h_{t-1} W_hh^T + b_hh)`` over a
    ``(T, B, input_size)`` sequence, ``act`` tanh or relu (ops/recurrent.py:140-219); returns
    ``h_1 .. h_T``, ``(T, B, H)``."""
    if nonlinearity not in ("tanh", "relu"):
        raise ValueError(f"nonlinearity must be 'tanh' or 'relu', got {nonlinearity!r}")
    relu = int(nonlinearity == "relu")
    parents, arrays = _prepare("rnn", x, (h0,), w_ih, w_hh, b_ih, b_hh)
    xd, h0d, w_ihd, w_hhd = arrays[:4]
    bias = arrays[4:] if len(arrays) > 4 else [None, None]
    steps, batch, width = xd.shape
    hid = h0d.shape[1]
    dt = xd.dtype
    code = dtype_code(dt)
    out = device.empty((steps, batch, hid), dt)
    scratch = device.scratch(lib.tg_rnn_forward_scratch_bytes(code, steps, batch, width, hid))
    check(lib.tg_rnn_forward(code, relu, steps, batch, width, hid, xd.ptr, h0d.ptr, w_ihd.ptr,
                             w_hhd.ptr, _ptr(bias[0]), _ptr(bias[1]), out.ptr, scratch.ptr,
                             device.stream()), "rnn")
    has_bias = len(arrays) > 4

    def backward(g: DeviceArray, need: Need) -> tuple[DeviceArray | None, ...]:
        if g.dtype != dt:
            g = cast_array(g, dt)

        def want(k: int, shape: tuple[int, ...]) -> DeviceArray | None:
            return device.empty(shape, dt) if need[k] else None

        dx, dh0 = want(0, xd.shape), want(1, h0d.shape)
        dw_ih, dw_hh = want(2, w_ihd.shape), want(3, w_hhd.shape)
        db_ih = want(4, (hid,)) if has_bias else None
        db_hh = want(5, (hid,)) if has_bias else None
        scr = device.scratch(lib.tg_rnn_backward_scratch_bytes(code, steps, batch, width, hid))
        check(lib.tg_rnn_backward(
            code, relu, steps, batch, width, hid, g.ptr, xd.ptr, h0d.ptr, w_ihd.ptr,
            w_hhd.ptr, out.ptr, _ptr(dx), _ptr(dh0), _ptr(dw_ih), _ptr(dw_hh), _ptr(db_ih),
            _ptr(db_hh), scr.ptr, device.stream()), "rnn backward")
        grads = [dx, dh0, dw_ih, dw_hh]
        return tuple(grads + [db_ih, db_hh] if has_bias else grads)

    def graph(g: Tensor, y: Tensor, need: Need) -> tuple[Tensor | None, ...]:
        return graph_by_composite(
            parents, lambda *ps: _rnn_composite(*ps, relu=bool(relu)), g, need)

    return make_result(out, parents, backward, "rnn", graph)
