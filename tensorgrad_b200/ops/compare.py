"""Non-differentiable tensor queries on the device: comparisons into boolean tensors, and
``all`` / ``any`` / ``argmax`` (the reference's tensor.py comparison operators and
tensor.py:418-435). Results are device tensors outside every graph.
"""

from __future__ import annotations

from typing import Any

import numpy as np

from tensorgrad_b200 import device
from tensorgrad_b200._lib import check, int64_array, int_array, lib
from tensorgrad_b200.device import DeviceArray, dtype_code
from tensorgrad_b200.ops._util import normalize_axes
from tensorgrad_b200.tensor import Tensor

__all__ = ["argmax", "compare", "truth"]

#: Tensor comparison operators and their kernel codes.
OPS = {"eq": 0, "ne": 1, "lt": 2, "le": 3, "gt": 4, "ge": 5}
_TRUTH_CODES = {np.dtype(np.bool_): -1, np.dtype(np.float32): 0, np.dtype(np.float64): 1,
                np.dtype(np.int64): 2}


def _as_float(a: DeviceArray) -> DeviceArray:
    """A floating view of ``a`` for the comparison kernels (booleans as 0 / 1)."""
    from tensorgrad_b200.ops.elementwise import cast_array
    from tensorgrad_b200.ops.shape import where_array

    if a.dtype.kind == "f":
        return a
    if a.dtype == np.bool_:
        one, zero = (device.scalar_like(v, np.dtype(np.float64)) for v in (1.0, 0.0))
        return where_array(a, one, zero)
    return cast_array(a, np.dtype(np.float64))


def _operand(x: Any, like: DeviceArray) -> DeviceArray:
    if isinstance(x, Tensor):
        return x.data
    if isinstance(x, DeviceArray):
        return x
    arr = np.asarray(x)
    dt = like.dtype if like.dtype.kind == "f" and arr.dtype.kind in "biuf" else None
    return device.from_numpy(arr, dt)


def _bcast(shape: tuple[int, ...], out: tuple[int, ...]) -> list[int]:
    strides = device.contiguous_strides(shape)
    pad = len(out) - len(shape)
    return [0] * pad + [0 if (n == 1 and out[pad + i] != 1) else strides[i]
                        for i, n in enumerate(shape)]


def compare(a: Tensor, other: Any, op: str) -> Tensor:
    """``a <op> other`` elementwise with broadcasting, as a boolean tensor."""
    x = _as_float(a.data)
    y = _as_float(_operand(other, a.data))
    dt = np.result_type(x.dtype, y.dtype)
    if x.dtype != dt:
        x = x.astype(dt)
    if y.dtype != dt:
        y = y.astype(dt)
    shape = tuple(np.broadcast_shapes(x.shape, y.shape))
    out = device.empty(shape, np.bool_)
    check(lib.tg_compare(dtype_code(dt), OPS[op], len(shape), int64_array(shape), x.ptr,
                         int64_array(_bcast(x.shape, shape)), y.ptr,
                         int64_array(_bcast(y.shape, shape)), out.ptr, device.stream()),
          "compare")
    return Tensor._wrap(out)


def _kept(shape: tuple[int, ...], axes: tuple[int, ...], keepdims: bool) -> tuple[int, ...]:
    if keepdims:
        return tuple(1 if i in axes else n for i, n in enumerate(shape))
    return tuple(n for i, n in enumerate(shape) if i not in axes)


def truth(a: Tensor, axis: Any, keepdims: bool, is_all: bool) -> Tensor:
    """``all`` / ``any`` over ``axis``: whether every / some element is nonzero."""
    x = a.data
    if x.dtype not in _TRUTH_CODES:
        x = _as_float(x)
    axes = normalize_axes(axis, x.ndim)
    out = device.empty(_kept(x.shape, axes, keepdims), np.bool_)
    keep = [0 if i in axes else 1 for i in range(x.ndim)]
    check(lib.tg_reduce_truth(_TRUTH_CODES[x.dtype], int(is_all), x.ndim, int64_array(x.shape),
                              int_array(keep), x.ptr, out.ptr, device.stream()),
          "all" if is_all else "any")
    return Tensor._wrap(out)


def argmax(a: Tensor, axis: int | None, keepdims: bool) -> Tensor:
    """Index of the first maximum along ``axis`` (over the flattened tensor for ``None``)."""
    x = _as_float(a.data)
    if axis is None:
        axes = tuple(range(x.ndim))
        shape = tuple(1 for _ in x.shape) if keepdims else ()
    else:
        axes = normalize_axes(axis, x.ndim)
        shape = _kept(x.shape, axes, keepdims)
    out = device.empty(shape, np.int64)
    keep = [0 if i in axes else 1 for i in range(x.ndim)]
    check(lib.tg_argmax(dtype_code(x.dtype), x.ndim, int64_array(x.shape), int_array(keep),
                        x.ptr, out.ptr, device.stream()), "argmax")
    return Tensor._wrap(out)
