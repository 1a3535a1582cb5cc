"""Elementwise arithmetic and pointwise non-linearities (the reference's ops/elementwise.py).

Forward values and VJPs follow ops/elementwise.py:43-343; each runs as one device kernel.
"""

from __future__ import annotations

import math
from typing import Any

import numpy as np

from tensorgrad_b200 import device
from tensorgrad_b200._lib import (
    ADD, DIV, EXP, F32, F64, FILL, LOG, MUL, NEG, POW, POWS, SIGMOID, SQRT, SUB, TANH, check,
    int64_array, lib,
)
from tensorgrad_b200.device import DeviceArray, dtype_code
from tensorgrad_b200.ops._util import (
    Need, as_tensor, coerce_pair, constant, make_result, unbroadcast,
)
from tensorgrad_b200.profiler import profiled
from tensorgrad_b200.tensor import Tensor

__all__ = ["add", "astype", "div", "exp", "gelu", "log", "mul", "neg", "pow", "relu", "sigmoid",
           "sqrt", "sub", "tanh"]

_CAST_CODES = {np.dtype(np.float32): F32, np.dtype(np.float64): F64, np.dtype(np.int64): 2}


def cast_array(x: DeviceArray, dtype: np.dtype[Any]) -> DeviceArray:
    out = device.empty(x.shape, dtype)
    check(lib.tg_cast(_CAST_CODES[x.dtype], _CAST_CODES[np.dtype(dtype)], x.size, x.ptr, out.ptr,
                      device.stream()), "astype")
    return out


def _promote(a: DeviceArray, b: DeviceArray) -> tuple[DeviceArray, DeviceArray, np.dtype[Any]]:
    if a.dtype == b.dtype and a.dtype.kind == "f":
        return a, b, a.dtype
    dt = np.result_type(a.dtype, b.dtype)
    if dt.kind != "f":
        dt = np.dtype(np.float64)
    return (a if a.dtype == dt else cast_array(a, dt)), (b if b.dtype == dt else cast_array(b, dt)), dt


def _bcast_strides(shape: tuple[int, ...], out_shape: tuple[int, ...]) -> list[int]:
    strides = device.contiguous_strides(shape)
    pad = len(out_shape) - len(shape)
    res = [0] * pad
    for i, n in enumerate(shape):
        res.append(0 if (n == 1 and out_shape[pad + i] != 1) else strides[i])
    return res


def binary_array(a: DeviceArray, b: DeviceArray, op: int, out: DeviceArray | None = None) -> DeviceArray:
    """``a op b`` with NumPy broadcasting, into a new array (or ``out``)."""
    a, b, dt = _promote(a, b)
    shape = a.shape if a.shape == b.shape else tuple(np.broadcast_shapes(a.shape, b.shape))
    if out is None:
        out = device.empty(shape, dt)
    sa = _bcast_strides(a.shape, shape) if a.shape != shape else device.contiguous_strides(shape)
    sb = _bcast_strides(b.shape, shape) if b.shape != shape else device.contiguous_strides(shape)
    check(lib.tg_binary(dtype_code(dt), op, len(shape), int64_array(shape), a.ptr,
                        int64_array(sa), b.ptr, int64_array(sb), out.ptr, device.stream()),
          "binary op")
    return out


def scale_array(x: DeviceArray, alpha: float) -> DeviceArray:
    out = device.empty(x.shape, x.dtype)
    check(lib.tg_axpby(dtype_code(x.dtype), x.size, alpha, x.ptr, 0.0, None, out.ptr,
                       device.stream()), "scale")
    return out


def _unary(x: DeviceArray, op: int, alpha: float = 0.0) -> DeviceArray:
    out = device.empty(x.shape, x.dtype)
    check(lib.tg_unary(dtype_code(x.dtype), op, x.size, x.ptr, alpha, out.ptr, device.stream()),
          "unary op")
    return out


def _unary_bwd(op: int, g: DeviceArray, x: DeviceArray | None, y: DeviceArray | None,
               alpha: float = 0.0) -> DeviceArray:
    out = device.empty(g.shape, g.dtype)
    check(lib.tg_unary_backward(dtype_code(g.dtype), op, g.size, g.ptr,
                                x.ptr if x is not None else None,
                                y.ptr if y is not None else None, alpha, out.ptr,
                                device.stream()), "unary backward")
    return out


def _sum_to(g: Tensor, shape: tuple[int, ...]) -> Tensor:
    """Differentiable sum of a gradient tensor down to an input's shape (graph VJPs)."""
    if g.shape == tuple(shape):
        return g
    from tensorgrad_b200.ops.shape import sum_to

    return sum_to(g, shape)


def _float_input(t: Tensor) -> DeviceArray:
    return t.data if t.dtype.kind == "f" else cast_array(t.data, np.dtype(np.float64))


@profiled("add")
def add(a: Any, b: Any) -> Tensor:
    """``a + b`` with broadcasting (ops/elementwise.py:43-60)."""
    ta, tb = coerce_pair(a, b)
    sa, sb = ta.shape, tb.shape

    def backward(g: DeviceArray, need: Need) -> tuple[DeviceArray | None, DeviceArray | None]:
        return (unbroadcast(g, sa) if need[0] else None, unbroadcast(g, sb) if need[1] else None)

    def graph(g: Tensor, y: Tensor, need: Need) -> tuple[Tensor | None, Tensor | None]:
        return (_sum_to(g, sa) if need[0] else None, _sum_to(g, sb) if need[1] else None)

    return make_result(binary_array(ta.data, tb.data, ADD), (ta, tb), backward, "add", graph)


@profiled("sub")
def sub(a: Any, b: Any) -> Tensor:
    """``a - b`` (ops/elementwise.py:63-80)."""
    ta, tb = coerce_pair(a, b)
    sa, sb = ta.shape, tb.shape

    def backward(g: DeviceArray, need: Need) -> tuple[DeviceArray | None, DeviceArray | None]:
        return (unbroadcast(g, sa) if need[0] else None,
                unbroadcast(scale_array(g, -1.0), sb) if need[1] else None)

    def graph(g: Tensor, y: Tensor, need: Need) -> tuple[Tensor | None, Tensor | None]:
        return (_sum_to(g, sa) if need[0] else None, _sum_to(neg(g), sb) if need[1] else None)

    return make_result(binary_array(ta.data, tb.data, SUB), (ta, tb), backward, "sub", graph)


@profiled("mul")
def mul(a: Any, b: Any) -> Tensor:
    """``a * b`` (ops/elementwise.py:83-100)."""
    ta, tb = coerce_pair(a, b)

    def backward(g: DeviceArray, need: Need) -> tuple[DeviceArray | None, DeviceArray | None]:
        return (unbroadcast(binary_array(g, tb.data, MUL), ta.shape) if need[0] else None,
                unbroadcast(binary_array(g, ta.data, MUL), tb.shape) if need[1] else None)

    def graph(g: Tensor, y: Tensor, need: Need) -> tuple[Tensor | None, Tensor | None]:
        return (_sum_to(mul(g, tb), ta.shape) if need[0] else None,
                _sum_to(mul(g, ta), tb.shape) if need[1] else None)

    return make_result(binary_array(ta.data, tb.data, MUL), (ta, tb), backward, "mul", graph)


@profiled("div")
def div(a: Any, b: Any) -> Tensor:
    """``a / b`` (ops/elementwise.py:103-121)."""
    ta, tb = coerce_pair(a, b)
    out = binary_array(ta.data, tb.data, DIV)

    def backward(g: DeviceArray, need: Need) -> tuple[DeviceArray | None, DeviceArray | None]:
        ga = unbroadcast(binary_array(g, tb.data, DIV), ta.shape) if need[0] else None
        gb = None
        if need[1]:
            t = binary_array(binary_array(g, out, MUL), tb.data, DIV)
            gb = unbroadcast(scale_array(t, -1.0), tb.shape)
        return ga, gb

    def graph(g: Tensor, y: Tensor, need: Need) -> tuple[Tensor | None, Tensor | None]:
        return (_sum_to(div(g, tb), ta.shape) if need[0] else None,
                _sum_to(neg(div(mul(g, y), tb)), tb.shape) if need[1] else None)

    return make_result(out, (ta, tb), backward, "div", graph)


@profiled("neg")
def neg(a: Any) -> Tensor:
    """``-a`` (ops/elementwise.py:124-135)."""
    ta = as_tensor(a)

    def backward(g: DeviceArray, need: Need) -> tuple[DeviceArray]:
        return (scale_array(g, -1.0),)

    def graph(g: Tensor, y: Tensor, need: Need) -> tuple[Tensor]:
        return (neg(g),)

    return make_result(scale_array(ta.data, -1.0), (ta,), backward, "neg", graph)


@profiled("pow")
def pow(base: Any, exponent: Any) -> Tensor:  # noqa: A001
    """``base ** exponent`` (ops/elementwise.py:138-167). A Python-number exponent runs as one
    kernel. The gradient with respect to a tensor exponent, ``out * log(base)``, exists for
    positive bases only and is zero elsewhere, as in the reference."""
    if isinstance(exponent, int | float) and isinstance(base, Tensor):
        tb = base
        e = float(exponent)
        x = _float_input(tb)

        def backward(g: DeviceArray, need: Need) -> tuple[DeviceArray]:
            return (_unary_bwd(POWS, g, x, None, e),)

        def graph(g: Tensor, y: Tensor, need: Need) -> tuple[Tensor]:
            return (mul(g, mul(pow(tb, e - 1.0), e)),)

        return make_result(_unary(x, POWS, e), (tb,), backward, "pow", graph)
    tb, te = coerce_pair(base, exponent)
    out = binary_array(tb.data, te.data, POW)

    def positive() -> Tensor:
        from tensorgrad_b200.ops.compare import compare

        return compare(tb, 0.0, "gt")  # a constant mask: log(base) exists where base > 0

    def backward2(g: DeviceArray, need: Need) -> tuple[DeviceArray | None, DeviceArray | None]:
        from tensorgrad_b200.ops.shape import where_array

        g_base = g_exp = None
        if need[0]:
            em1 = binary_array(te.data, device.scalar_like(1.0, te.dtype), SUB)
            d = binary_array(binary_array(g, te.data, MUL), binary_array(tb.data, em1, POW), MUL)
            g_base = unbroadcast(d, tb.shape)
        if need[1]:
            mask = positive().data
            one, zero = (device.scalar_like(v, out.dtype) for v in (1.0, 0.0))
            log_base = _unary(where_array(mask, tb.data if tb.dtype == out.dtype
                                          else cast_array(tb.data, out.dtype), one), LOG)
            d = binary_array(binary_array(g, out, MUL), log_base, MUL)
            g_exp = unbroadcast(where_array(mask, d, zero), te.shape)
        return g_base, g_exp

    def graph2(g: Tensor, y: Tensor, need: Need) -> tuple[Tensor | None, Tensor | None]:
        from tensorgrad_b200.ops.shape import where

        g_base = _sum_to(mul(mul(g, te), pow(tb, sub(te, 1.0))), tb.shape) if need[0] else None
        g_exp = None
        if need[1]:
            mask = positive()
            log_base = log(where(mask, tb, 1.0))
            g_exp = _sum_to(where(mask, mul(mul(g, y), log_base), 0.0), te.shape)
        return g_base, g_exp

    return make_result(out, (tb, te), backward2, "pow", graph2)


def _unary_op(name: str, op: int, use_out: bool) -> Any:
    @profiled(name)
    def fn(a: Any) -> Tensor:
        ta = as_tensor(a)
        x = _float_input(ta)
        out = _unary(x, op)

        def backward(g: DeviceArray, need: Need) -> tuple[DeviceArray]:
            return (_unary_bwd(op, g, None if use_out else x, out if use_out else None),)

        def graph(g: Tensor, y: Tensor, need: Need) -> tuple[Tensor]:
            return (_unary_graph(op, g, ta, y),)

        return make_result(out, (ta,), backward, name, graph)

    fn.__name__ = name
    return fn


def _unary_graph(op: int, g: Tensor, x: Tensor, y: Tensor) -> Tensor:
    """The unary VJPs in differentiable ops, from the input ``x`` or the output ``y``."""
    if op == EXP:
        return mul(g, y)
    if op == LOG:
        return div(g, x)
    if op == SQRT:
        return div(mul(g, 0.5), y)
    if op == TANH:
        return mul(g, sub(1.0, mul(y, y)))
    if op == SIGMOID:
        return mul(g, mul(y, sub(1.0, y)))
    raise NotImplementedError(f"no differentiable VJP for unary op {op}")


exp = _unary_op("exp", EXP, True)        # ops/elementwise.py:170-181
log = _unary_op("log", LOG, False)       # :184-195
sqrt = _unary_op("sqrt", SQRT, True)     # :198-210
tanh = _unary_op("tanh", TANH, True)     # :213-225
sigmoid = _unary_op("sigmoid", SIGMOID, True)  # :240-252


@profiled("relu")
def relu(a: Any) -> Tensor:
    """``max(a, 0)``; the VJP is ``g * (a > 0)`` (ops/elementwise.py:255-268)."""
    ta = as_tensor(a)
    x = ta.data

    def backward(g: DeviceArray, need: Need) -> tuple[DeviceArray]:
        out = device.empty(g.shape, g.dtype)
        check(lib.tg_relu_backward(dtype_code(g.dtype), g.size, g.ptr, x.ptr, out.ptr,
                                   device.stream()), "relu backward")
        return (out,)

    def graph(g: Tensor, y: Tensor, need: Need) -> tuple[Tensor]:
        # g times the constant mask (x > 0), the mask being the VJP of a ones gradient.
        return (mul(g, constant(backward(_unary(x, FILL, 1.0), need)[0])),)

    return make_result(_unary(x, 6), (ta,), backward, "relu", graph)


@profiled("gelu")
def gelu(a: Any) -> Tensor:
    """Tanh-approximate GELU; the VJP recomputes ``tanh`` from the saved input instead of
    storing it (ops/elementwise.py:275-320)."""
    ta = as_tensor(a)
    x = _float_input(ta)
    out = device.empty(x.shape, x.dtype)
    check(lib.tg_gelu_forward(dtype_code(x.dtype), x.size, x.ptr, out.ptr, device.stream()),
          "gelu")

    def backward(g: DeviceArray, need: Need) -> tuple[DeviceArray]:
        gx = device.empty(g.shape, g.dtype)
        check(lib.tg_gelu_backward(dtype_code(g.dtype), g.size, g.ptr, x.ptr, gx.ptr,
                                   device.stream()), "gelu backward")
        return (gx,)

    def graph(g: Tensor, y: Tensor, need: Need) -> tuple[Tensor]:
        # d gelu / dx = 0.5 (1 + t) + 0.5 x (1 - t^2) c (1 + 3 k x^2), t = tanh(c (x + k x^3)).
        c, k = math.sqrt(2.0 / math.pi), 0.044715
        x2 = mul(ta, ta)
        t = tanh(mul(add(ta, mul(mul(x2, ta), k)), c))
        slope = mul(mul(mul(ta, sub(1.0, mul(t, t))), add(mul(x2, 3.0 * k), 1.0)), 0.5 * c)
        return (mul(g, add(mul(add(t, 1.0), 0.5), slope)),)

    return make_result(out, (ta,), backward, "gelu", graph)


@profiled("astype")
def astype(a: Any, dtype: Any) -> Tensor:
    """Dtype conversion; integer results are constants (ops/elementwise.py:323-343)."""
    ta = as_tensor(a)
    source = ta.dtype
    dt = np.dtype(dtype)
    out = ta.data.copy() if dt == source else cast_array(ta.data, dt)
    if dt.kind != "f":
        return Tensor._wrap(out)

    def backward(g: DeviceArray, need: Need) -> tuple[DeviceArray]:
        return (g if g.dtype == source else cast_array(g, source),)

    def graph(g: Tensor, y: Tensor, need: Need) -> tuple[Tensor]:
        return (g if g.dtype == source else astype(g, source),)

    return make_result(out, (ta,), backward, "astype", graph)


# NEG kept for symmetry with the C enum (used by callers that negate in place).
_ = NEG
