"""Reductions with ``keepdims`` (the reference's ops/reduce.py): sum, mean, var."""

from __future__ import annotations

import builtins
import math
from typing import Any

import numpy as np

from tensorgrad_b200 import device
from tensorgrad_b200._lib import MUL, SUB, check, int64_array, int_array, lib
from tensorgrad_b200.device import DeviceArray, dtype_code
from tensorgrad_b200.ops._util import Need, as_tensor, make_result, normalize_axes
from tensorgrad_b200.ops.elementwise import binary_array, scale_array
from tensorgrad_b200.profiler import profiled
from tensorgrad_b200.tensor import Tensor

__all__ = ["max", "mean", "min", "sum", "var"]


def _kept_shape(shape: tuple[int, ...], axes: tuple[int, ...]) -> tuple[int, ...]:
    return tuple(1 if i in axes else n for i, n in enumerate(shape))


def sum_array(x: DeviceArray, axes: tuple[int, ...]) -> DeviceArray:
    """Sum over ``axes``; the result has the kept (size-1) axes."""
    kept = _kept_shape(x.shape, axes)
    code = dtype_code(x.dtype)
    out = device.empty(kept, x.dtype)
    if len(axes) == x.ndim:
        scratch = device.scratch(lib.tg_sum_all_scratch_bytes())
        check(lib.tg_sum_all(code, x.ptr, out.ptr, x.size, scratch.ptr, device.stream()), "sum")
        return out
    keep = [0 if i in axes else 1 for i in range(x.ndim)]
    check(lib.tg_reduce_sum(code, x.ndim, int64_array(x.shape), int_array(keep), x.ptr, out.ptr,
                            device.stream()), "sum")
    return out


def expand_array(g: DeviceArray, shape: tuple[int, ...], axes: tuple[int, ...]) -> DeviceArray:
    """Re-insert the reduced axes of ``g`` and broadcast it back to ``shape``."""
    from tensorgrad_b200.ops.shape import broadcast_array

    return broadcast_array(g.reshape(_kept_shape(shape, axes)), shape)


def _expand(g: Tensor, shape: tuple[int, ...], axes: tuple[int, ...]) -> Tensor:
    """``expand_array`` in differentiable ops (the graph VJP of the reductions)."""
    from tensorgrad_b200.ops.shape import broadcast_to, reshape

    return broadcast_to(reshape(g, _kept_shape(shape, axes)), shape)


def _drop(a: DeviceArray, axes: tuple[int, ...], keepdims: bool) -> DeviceArray:
    if keepdims:
        return a
    return a.reshape(tuple(n for i, n in enumerate(a.shape) if i not in axes))


@profiled("sum")
def sum(a: Any, axis: Any = None, keepdims: bool = False) -> Tensor:  # noqa: A001
    """Sum over ``axis`` (ops/reduce.py:31-45)."""
    ta = as_tensor(a)
    axes = normalize_axes(axis, ta.ndim)
    out = _drop(sum_array(ta.data, axes), axes, keepdims)

    def backward(g: DeviceArray, need: Need) -> tuple[DeviceArray]:
        return (expand_array(g, ta.shape, axes),)

    def graph(g: Tensor, y: Tensor, need: Need) -> tuple[Tensor]:
        return (_expand(g, ta.shape, axes),)

    return make_result(out, (ta,), backward, "sum", graph)


@profiled("mean")
def mean(a: Any, axis: Any = None, keepdims: bool = False) -> Tensor:
    """Arithmetic mean over ``axis`` (ops/reduce.py:55-69)."""
    ta = as_tensor(a)
    axes = normalize_axes(axis, ta.ndim)
    n = math.prod(ta.shape[i] for i in axes)
    out = _drop(scale_array(sum_array(ta.data, axes), 1.0 / n if n else float("nan")), axes,
                keepdims)

    def backward(g: DeviceArray, need: Need) -> tuple[DeviceArray]:
        return (expand_array(scale_array(g, 1.0 / n), ta.shape, axes),)

    def graph(g: Tensor, y: Tensor, need: Need) -> tuple[Tensor]:
        from tensorgrad_b200.ops.elementwise import mul

        return (_expand(mul(g, 1.0 / n), ta.shape, axes),)

    return make_result(out, (ta,), backward, "mean", graph)


@profiled("var")
def var(a: Any, axis: Any = None, keepdims: bool = False, correction: int = 1) -> Tensor:
    """``sum((x - mean)**2) / (N - correction)``; VJP ``g * 2 (x - mean) / (N - correction)``
    (ops/reduce.py:108-132)."""
    ta = as_tensor(a)
    axes = normalize_axes(axis, ta.ndim)
    n = math.prod(ta.shape[i] for i in axes)
    denom = builtins.max(n - correction, 0)
    m = scale_array(sum_array(ta.data, axes), 1.0 / n)
    centered = binary_array(ta.data, m, SUB)
    sq = binary_array(centered, centered, MUL)
    out = _drop(scale_array(sum_array(sq, axes), 1.0 / denom if denom else float("nan")), axes,
                keepdims)
    scale = 2.0 / denom if denom else float("nan")

    def backward(g: DeviceArray, need: Need) -> tuple[DeviceArray]:
        return (binary_array(expand_array(scale_array(g, scale), ta.shape, axes), centered, MUL),)

    def graph(g: Tensor, y: Tensor, need: Need) -> tuple[Tensor]:
        from tensorgrad_b200.ops.elementwise import mul, sub

        return (mul(_expand(mul(g, scale), ta.shape, axes),
                    sub(ta, mean(ta, axes, keepdims=True))),)

    return make_result(out, (ta,), backward, "var", graph)


def extremum_array(x: DeviceArray, axes: tuple[int, ...], is_min: bool) -> DeviceArray:
    """Max (or min) over ``axes``, NaN-propagating; the result keeps the reduced axes."""
    out = device.empty(_kept_shape(x.shape, axes), x.dtype)
    keep = [0 if i in axes else 1 for i in range(x.ndim)]
    check(lib.tg_reduce_extremum(dtype_code(x.dtype), int(is_min), x.ndim,
                                 int64_array(x.shape), int_array(keep), x.ptr, out.ptr,
                                 device.stream()), "min" if is_min else "max")
    return out


def _extremum(a: Any, axis: Any, keepdims: bool, is_min: bool, op: str) -> Tensor:
    """Max / min over ``axis`` (ops/reduce.py:70-105): tied extrema share the gradient
    equally, a valid subgradient; the share is a constant mask under ``create_graph``."""
    from tensorgrad_b200._lib import DIV, EQ
    from tensorgrad_b200.ops.elementwise import cast_array

    ta = as_tensor(a)
    axes = normalize_axes(axis, ta.ndim)
    xd = ta.data if ta.dtype.kind == "f" else cast_array(ta.data, np.dtype(np.float64))
    kept = extremum_array(xd, axes, is_min)
    out = _drop(kept, axes, keepdims)
    if ta.dtype.kind != "f":
        out = cast_array(out, ta.dtype)

    def share() -> DeviceArray:
        winners = binary_array(xd, kept, EQ)
        return binary_array(winners, sum_array(winners, axes), DIV)

    def backward(g: DeviceArray, need: Need) -> tuple[DeviceArray]:
        return (binary_array(expand_array(g, ta.shape, axes), share(), MUL),)

    def graph(g: Tensor, y: Tensor, need: Need) -> tuple[Tensor]:
        from tensorgrad_b200.ops._util import constant
        from tensorgrad_b200.ops.elementwise import mul

        return (mul(_expand(g, ta.shape, axes), constant(share())),)

    return make_result(out, (ta,), backward, op, graph)


@profiled("max")
def max(a: Any, axis: Any = None, keepdims: bool = False) -> Tensor:  # noqa: A001
    """Maximum over ``axis``; tied maxima share the gradient equally."""
    return _extremum(a, axis, keepdims, False, "max")


@profiled("min")
def min(a: Any, axis: Any = None, keepdims: bool = False) -> Tensor:  # noqa: A001
    """Minimum over ``axis``; tied minima share the gradient equally."""
    return _extremum(a, axis, keepdims, True, "min")
