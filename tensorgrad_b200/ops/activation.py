"""Softmax, log-softmax and log-sum-exp along an axis (the reference's ops/activation.py).

Each is one graph node over device kernels: the row maximum (``tg_reduce_extremum``; a row
whose maximum is not finite is shifted by 0, so an all ``-inf`` row gives NaN as in the
reference), the shifted exponentials and their sums, with the closed-form VJPs
``s (g - sum(g s))``, ``g - exp(y) sum(g)`` and ``g exp(x - lse)``. Their graph VJPs are the
same formulas in differentiable ops. None of them is on a measured training step (the
language models fuse softmax into attention and cross entropy).
"""

from __future__ import annotations

from typing import Any

from tensorgrad_b200._lib import ADD, DIV, EXP, FINITE_OR_ZERO, LOG, MUL, SUB
from tensorgrad_b200.device import DeviceArray
from tensorgrad_b200.ops._util import Need, as_tensor, make_result, normalize_axis
from tensorgrad_b200.ops.elementwise import _unary, binary_array, cast_array
from tensorgrad_b200.ops.reduce import _drop, expand_array, extremum_array, sum_array
from tensorgrad_b200.profiler import profiled
from tensorgrad_b200.tensor import Tensor

__all__ = ["log_softmax", "logsumexp", "softmax"]


def _float(t: Tensor) -> DeviceArray:
    import numpy as np

    return t.data if t.dtype.kind == "f" else cast_array(t.data, np.dtype(np.float64))


def _shifted(x: DeviceArray, ax: int) -> tuple[DeviceArray, DeviceArray]:
    """``x - m`` and ``m``, the row maximum along ``ax`` (kept axis), 0 where not finite."""
    m = _unary(extremum_array(x, (ax,), False), FINITE_OR_ZERO)
    return binary_array(x, m, SUB), m


@profiled("softmax")
def softmax(a: Any, axis: int = -1) -> Tensor:
    """``exp(x) / sum(exp(x))`` along ``axis`` (ops/activation.py:27-45)."""
    ta = as_tensor(a)
    ax = normalize_axis(axis, ta.ndim)
    e = _unary(_shifted(_float(ta), ax)[0], EXP)
    s = binary_array(e, sum_array(e, (ax,)), DIV)

    def backward(g: DeviceArray, need: Need) -> tuple[DeviceArray]:
        dot = sum_array(binary_array(g, s, MUL), (ax,))
        return (binary_array(s, binary_array(g, dot, SUB), MUL),)

    def graph(g: Tensor, y: Tensor, need: Need) -> tuple[Tensor]:
        return (y * (g - (g * y).sum(axis=ax, keepdims=True)),)

    return make_result(s, (ta,), backward, "softmax", graph)


@profiled("log_softmax")
def log_softmax(a: Any, axis: int = -1) -> Tensor:
    """``x - logsumexp(x)`` along ``axis`` with the max shift (ops/activation.py:55-72)."""
    ta = as_tensor(a)
    ax = normalize_axis(axis, ta.ndim)
    shifted, _ = _shifted(_float(ta), ax)
    lse = _unary(sum_array(_unary(shifted, EXP), (ax,)), LOG)
    out = binary_array(shifted, lse, SUB)

    def backward(g: DeviceArray, need: Need) -> tuple[DeviceArray]:
        total = sum_array(g, (ax,))
        return (binary_array(g, binary_array(_unary(out, EXP), total, MUL), SUB),)

    def graph(g: Tensor, y: Tensor, need: Need) -> tuple[Tensor]:
        from tensorgrad_b200.ops.elementwise import exp

        return (g - exp(y) * g.sum(axis=ax, keepdims=True),)

    return make_result(out, (ta,), backward, "log_softmax", graph)


@profiled("logsumexp")
def logsumexp(a: Any, axis: int = -1, keepdims: bool = False) -> Tensor:
    """Stable ``log(sum(exp(x)))`` along ``axis``; its gradient is ``softmax(x)``
    (ops/activation.py:75-93)."""
    ta = as_tensor(a)
    ax = normalize_axis(axis, ta.ndim)
    x = _float(ta)
    shifted, m = _shifted(x, ax)
    kept = binary_array(_unary(sum_array(_unary(shifted, EXP), (ax,)), LOG), m, ADD)
    out = _drop(kept, (ax,), keepdims)

    def backward(g: DeviceArray, need: Need) -> tuple[DeviceArray]:
        g_kept = expand_array(g, ta.shape, (ax,))
        return (binary_array(g_kept, _unary(binary_array(x, kept, SUB), EXP), MUL),)

    def graph(g: Tensor, y: Tensor, need: Need) -> tuple[Tensor]:
        from tensorgrad_b200.ops.shape import unsqueeze

        g_kept = g if keepdims else unsqueeze(g, ax)
        return (g_kept * softmax(ta, ax),)

    return make_result(out, (ta,), backward, "logsumexp", graph)
